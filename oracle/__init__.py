"""ctypes loaders for the CPU checkers (test infrastructure only).

`Oracle` wraps oracle/_build/libqms_oracle.so, the C restatement of qms's MoE path.
`Reference` wraps oracle/_ref/libqms_ref_*.so, the reference compiled from its own sources
(oracle/Makefile, target `ref`). Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm import this package; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libqms_oracle.so"
REF_DIR = HERE / "_ref"

T_F32, T_F16, T_Q4_0, T_Q4_1, T_Q8_0, T_Q6_K = 0, 1, 2, 3, 8, 14

# OrcQ8 / QmsQ8: float d; float ds; int16 s16[2]; int8 q[32]  (44 bytes, src/kernels.h:7-12)
Q8_DTYPE = np.dtype([("d", "<f4"), ("ds", "<f4"), ("s16", "<i2", (2,)), ("q", "i1", (32,))])
assert Q8_DTYPE.itemsize == 44


def row_bytes(typ: int, ne0: int) -> int:
    """Bytes per row of ne0 elements (src/gguf.c:85-96)."""
    return {T_F32: ne0 * 4, T_F16: ne0 * 2,
            T_Q4_0: ne0 // 32 * 18 if ne0 % 32 == 0 else 0,
            T_Q4_1: ne0 // 32 * 20 if ne0 % 32 == 0 else 0,
            T_Q8_0: ne0 // 32 * 34 if ne0 % 32 == 0 else 0,
            T_Q6_K: ne0 // 256 * 210 if ne0 % 256 == 0 else 0}.get(typ, 0)


def _p(a: np.ndarray):
    return C.c_void_p(a.ctypes.data) if a is not None else None


def _build_oracle():
    if not ORACLE_SO.exists():
        import subprocess
        subprocess.run(["make", "-C", str(HERE), "all"], check=True, capture_output=True)


class Oracle:
    """The C restatement (kind "port")."""

    def __init__(self):
        _build_oracle()
        self.lib = L = C.CDLL(str(ORACLE_SO))
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_dequant_row.argtypes = [i32, vp, vp, i64]
        L.orc_dequant_row.restype = i32
        L.orc_quantize_q8.argtypes = [vp, i64, vp]
        L.orc_vec_dot_q8.argtypes = [i32, vp, vp, i64]
        L.orc_vec_dot_q8.restype = C.c_float
        L.orc_vec_dot_f32.argtypes = [vp, vp, i64]
        L.orc_vec_dot_f32.restype = C.c_float
        L.orc_matmul.argtypes = [i32, i64, i64, vp, vp, i32, vp]
        L.orc_matmul_q8.argtypes = [i32, i64, i64, vp, vp, i32, vp]
        L.orc_sample.argtypes = [vp, i32, C.c_float, C.c_float, i32, C.POINTER(C.c_uint64)]
        L.orc_sample.restype = i32
        L.orc_route.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp, vp]
        L.orc_moe.argtypes = [vp, vp, i32, vp, vp, vp, vp]
        L.orc_moe.restype = i32
        L.orc_swiglu.argtypes = [vp, vp, i64, vp]
        L.orc_set_threads.argtypes = [i32]

    def set_threads(self, n: int):
        self.lib.orc_set_threads(int(n))

    def f16_to_f32(self, h: int) -> float:
        return self.lib.orc_f16_to_f32(h)

    def dequant_row(self, typ: int, src: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        if self.lib.orc_dequant_row(typ, _p(np.ascontiguousarray(src)), _p(out), n) != 0:
            raise ValueError("unsupported type or size")
        return out

    def quantize_q8(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.size // 32, Q8_DTYPE)
        self.lib.orc_quantize_q8(_p(x), x.size, _p(out))
        return out

    def vec_dot_q8(self, typ: int, w: np.ndarray, xq: np.ndarray, n: int) -> float:
        return self.lib.orc_vec_dot_q8(typ, _p(np.ascontiguousarray(w)), _p(xq), n)

    def vec_dot_f32(self, w: np.ndarray, x: np.ndarray) -> float:
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        return self.lib.orc_vec_dot_f32(_p(w), _p(x), x.size)

    def matmul(self, typ: int, rows: int, cols: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        y = np.empty((x.shape[0], rows), np.float32)
        self.lib.orc_matmul(typ, rows, cols, _p(np.ascontiguousarray(w)), _p(x), x.shape[0], _p(y))
        return y

    def matmul_q8(self, typ: int, rows: int, cols: int, w: np.ndarray, xq: np.ndarray) -> np.ndarray:
        """matmul from quantised rows: xq holds T * cols/32 QmsQ8 records."""
        xq = np.ascontiguousarray(xq).view(Q8_DTYPE).reshape(-1)
        T = xq.size // (cols // 32)
        y = np.empty((T, rows), np.float32)
        self.lib.orc_matmul_q8(typ, rows, cols, _p(np.ascontiguousarray(w)), _p(xq), T, _p(y))
        return y

    def sample(self, logits: np.ndarray, temp: float, top_p: float, top_k: int, rng: int) -> tuple[int, int]:
        """The chat sampler (src/chat.c:36-69) restated: (token, advanced rng state)."""
        l = np.ascontiguousarray(logits, np.float32)
        st = C.c_uint64(rng)
        t = self.lib.orc_sample(_p(l), l.size, temp, top_p, top_k, C.byref(st))
        return t, st.value

    def route(self, router: np.ndarray, K: int, xn: np.ndarray):
        X, E = router.shape
        xn = np.ascontiguousarray(xn, np.float32).reshape(-1, E)
        T = xn.shape[0]
        logits = np.empty((T, X), np.float32)
        sel = np.empty((T, K), np.int32)
        w = np.empty((T, K), np.float32)
        self.lib.orc_route(_p(np.ascontiguousarray(router, np.float32)), X, E, K, _p(xn), T,
                           _p(logits), _p(sel), _p(w))
        return logits, sel, w

    def swiglu(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        a = np.empty_like(g)
        self.lib.orc_swiglu(_p(g), _p(u), g.size, _p(a))
        return a

    def moe(self, layer, xn: np.ndarray):
        """layer: synth.MoeLayer-like object. Returns (out, sel, w, logits)."""
        E, X, K = layer.n_embd, layer.n_expert, layer.n_used
        xn = np.ascontiguousarray(xn, np.float32).reshape(-1, E)
        T = xn.shape[0]
        out = np.empty((T, E), np.float32)
        sel = np.empty((T, K), np.int32)
        w = np.empty((T, K), np.float32)
        logits = np.empty((T, X), np.float32)

        class Desc(C.Structure):
            _fields_ = [("n_embd", C.c_int), ("n_expert", C.c_int), ("n_used", C.c_int),
                        ("n_ff", C.c_int), ("gate_type", C.c_int), ("up_type", C.c_int),
                        ("down_type", C.c_int), ("router", C.c_void_p), ("gate", C.c_void_p),
                        ("up", C.c_void_p), ("down", C.c_void_p)]
        d = Desc(E, X, K, layer.n_ff, layer.gate_type, layer.up_type, layer.down_type,
                 layer.router.ctypes.data, layer.gate.ctypes.data, layer.up.ctypes.data,
                 layer.down.ctypes.data)
        if self.lib.orc_moe(C.byref(d), _p(xn), T, _p(out), _p(sel), _p(w), _p(logits)) != 0:
            raise ValueError("layer does not take the integer fast path")
        return out, sel, w, logits


def ref_variant() -> str | None:
    """Pick the reference build this host can run: v4 (AVX-512 VNNI) when the CPU has it."""
    flags = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = line
                    break
    except OSError:
        pass
    need_v4 = ("avx512f", "avx512bw", "avx512dq", "avx512vl", "avx512cd", "avx512_vnni")
    for v in (["v4", "v3"] if all(n in flags.split() for n in need_v4) else ["v3"]):
        if (REF_DIR / f"libqms_ref_{v}.so").exists():
            return v
    return None


def reference_available() -> bool:
    return ref_variant() is not None


class Reference:
    """The reference's own code (kind "reference"), built from its sources by oracle/Makefile."""

    def __init__(self, variant: str | None = None):
        v = variant or ref_variant()
        if v is None:
            raise FileNotFoundError("oracle/_ref was not built (make -C oracle ref)")
        self.variant = v
        self.lib = L = C.CDLL(str(REF_DIR / f"libqms_ref_{v}.so"))
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        L.ref_set_threads.argtypes = [i32]
        L.ref_get_threads.restype = i32
        L.ref_set_exact.argtypes = [i32]
        L.ref_moe.argtypes = [i32] * 7 + [vp] * 5 + [i32, vp, vp, vp]
        L.ref_moe.restype = i32
        L.qms_quantize_q8.argtypes = [vp, i64, vp]
        L.qms_vec_dot_q8.argtypes = [i32, vp, vp, i64]
        L.qms_vec_dot_q8.restype = C.c_float
        L.qms_vec_dot_f32.argtypes = [vp, vp, i64]
        L.qms_vec_dot_f32.restype = C.c_float
        L.qms_dequant_row.argtypes = [i32, vp, vp, i64]
        L.qms_dequant_row.restype = i32
        L.qms_matmul.argtypes = [vp, vp, i32, vp]
        L.ref_model_new.argtypes = [i32] * 9 + [C.c_float, C.c_double, i32]
        L.ref_model_new.restype = vp
        L.ref_model_set_trunk.argtypes = [vp, i32, vp, vp, i32, vp]
        L.ref_model_set_layer.argtypes = [vp, i32, vp, vp, vp, vp, i32, vp, vp, vp, i32, vp, vp, i32, vp, vp, i32, vp]
        L.ref_forward.argtypes = [vp, vp, i32, i32, vp, i32]
        L.ref_forward.restype = i32
        L.ref_model_free.argtypes = [vp]

    def model(self, cfg, tensors: dict, ctx: int) -> "RefModel":
        """The reference's own qms_forward on a model held in host arrays (GGUF names and layouts,
        as large_model_b200.synth.model_tensors lists them)."""
        return RefModel(self, cfg, tensors, ctx)

    def set_threads(self, n: int):
        self.lib.ref_set_threads(int(n))

    def threads(self) -> int:
        return self.lib.ref_get_threads()

    def quantize_q8(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.size // 32, Q8_DTYPE)
        self.lib.qms_quantize_q8(_p(x), x.size, _p(out))
        return out

    def vec_dot_q8(self, typ: int, w: np.ndarray, xq: np.ndarray, n: int) -> float:
        return self.lib.qms_vec_dot_q8(typ, _p(np.ascontiguousarray(w)), _p(xq), n)

    def vec_dot_f32(self, w: np.ndarray, x: np.ndarray) -> float:
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        return self.lib.qms_vec_dot_f32(_p(w), _p(x), x.size)

    def dequant_row(self, typ: int, src: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        if self.lib.qms_dequant_row(typ, _p(np.ascontiguousarray(src)), _p(out), n) != 0:
            raise ValueError("unsupported type or size")
        return out

    def moe(self, layer, xn: np.ndarray, trace: bool = False):
        """Returns out [T][E] (and the --trace expert list when trace=True)."""
        E, X = layer.n_embd, layer.n_expert
        xn = np.ascontiguousarray(xn, np.float32).reshape(-1, E)
        T = xn.shape[0]
        out = np.empty((T, E), np.float32)
        tr = np.zeros(X, np.int32) if trace else None
        ntr = C.c_int(0)
        rc = self.lib.ref_moe(E, X, layer.n_used, layer.n_ff, layer.gate_type, layer.up_type,
                              layer.down_type, layer.router.ctypes.data, layer.gate.ctypes.data,
                              layer.up.ctypes.data, layer.down.ctypes.data, _p(xn), T, _p(out),
                              _p(tr), C.byref(ntr) if trace else None)
        if rc != 0:
            raise RuntimeError(f"reference moe() returned {rc}")
        return (out, tr[: ntr.value].copy()) if trace else out


class RefModel:
    """A QmsModel built from host arrays by oracle/ref_harness.c; forward() is the reference's
    qms_forward (src/model.c:1252-1296). The arrays are referenced, not copied: keep them alive."""

    def __init__(self, ref: Reference, cfg, tensors: dict, ctx: int):
        self.ref, self.cfg, self.keep = ref, cfg, tensors
        L = ref.lib
        c = cfg
        self.h = L.ref_model_new(c.n_layer, c.n_embd, c.n_head, c.n_head_kv, c.head_dim, c.n_expert, c.n_used,
                                 c.n_ff, c.vocab, float(c.eps), float(c.rope_base), int(ctx))
        if not self.h:
            raise MemoryError("ref_model_new failed")
        t = tensors
        out = t.get("output.weight")
        L.ref_model_set_trunk(self.h, T_Q4_0, _p(t["token_embd.weight"]), _p(t["output_norm.weight"]),
                              getattr(c, "output_type", T_Q6_K), None if out is None else _p(out))
        for l in range(c.n_layer):
            b = lambda n: _p(t[f"blk.{l}.{n}.weight"])
            L.ref_model_set_layer(self.h, l, b("attn_norm"), b("attn_q_norm"), b("attn_k_norm"), b("ffn_norm"),
                                  T_Q4_0, b("attn_q"), b("attn_k"), b("attn_v"), T_Q4_0, b("attn_output"),
                                  b("ffn_gate_inp"), T_Q4_0, b("ffn_gate_exps"), b("ffn_up_exps"), T_Q4_0,
                                  b("ffn_down_exps"))

    def forward(self, ids, pos0: int, all_logits: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        T = ids.shape[0]
        logits = np.empty((T, self.cfg.vocab) if all_logits else (self.cfg.vocab,), np.float32)
        if self.ref.lib.ref_forward(self.h, _p(ids), T, int(pos0), _p(logits), int(all_logits)) != 0:
            raise RuntimeError("reference qms_forward failed")
        return logits

    def close(self):
        if getattr(self, "h", None):
            self.ref.lib.ref_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


class RefSampler:
    """The reference's own sample() (src/chat.c:36-69) from oracle/_ref/libqms_ref_sample.so."""

    def __init__(self):
        path = HERE / "_ref" / "libqms_ref_sample.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} is missing: make -C oracle ref")
        self.lib = C.CDLL(str(path))
        self.lib.ref_sample.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_int, C.POINTER(C.c_uint64)]
        self.lib.ref_sample.restype = C.c_int

    def sample(self, logits: np.ndarray, temp: float, top_p: float, top_k: int, rng: int) -> tuple[int, int]:
        l = np.ascontiguousarray(logits, np.float32)
        st = C.c_uint64(rng)
        t = self.lib.ref_sample(l.ctypes.data_as(C.c_void_p), l.size, temp, top_p, top_k, C.byref(st))
        return t, st.value

