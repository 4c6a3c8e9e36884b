"""large_model_b200 - B200-native (sm_100a) Qwen3-MoE feed-forward path of qms.

The product is the C-ABI library `libqms_cuda.so` (include/qms_cuda.h). This module binds it
with ctypes and mirrors the reference's operator interface for tests and benchmarks:

    quantize_q8(x)               qms_quantize_q8   (src/kernels.h:15)
    matvec_q8(type, W, xq, ...)  qms_matmul fast path / qms_vec_dot_q8 (src/quant.h:23)
    matvec_f32(W, x)             qms_vec_dot_f32   (src/kernels.h:21)
    MoeLayer(...).forward(xn)    moe()             (src/model.c:1032)
    Model(...).forward(ids, pos) qms_forward       (src/model.c:1252), the whole token step

Device buffers are torch CUDA tensors (plumbing only); every computation runs in
libqms_cuda's kernels. There is no CPU fallback: if the library is missing or no sm_100 GPU is
present, the calls raise.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libqms_cuda.so"
HEADER = PKG.parent / "include" / "qms_cuda.h"

T_F32, T_F16, T_Q4_0, T_Q4_1, T_Q8_0, T_Q6_K = 0, 1, 2, 3, 8, 14
OK, EINVAL, ECUDA, ENOMEM, EUNSUPPORTED, ENODEV, ETIMEOUT = 0, -1, -2, -3, -4, -5, -6

Q8_DTYPE = np.dtype([("d", "<f4"), ("ds", "<f4"), ("s16", "<i2", (2,)), ("q", "i1", (32,))])


class QmsCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libqms_cuda error {code}: {msg}")
        self.code = code


class MoeDesc(C.Structure):
    _fields_ = [("n_embd", C.c_int), ("n_expert", C.c_int), ("n_used", C.c_int), ("n_ff", C.c_int),
                ("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int),
                ("router", C.c_void_p), ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("src_on_device", C.c_int)]


class ModelDesc(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_embd", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("head_dim", C.c_int), ("n_expert", C.c_int), ("n_used", C.c_int), ("n_ff", C.c_int),
                ("vocab", C.c_int), ("eps", C.c_float), ("rope_base", C.c_double), ("ctx", C.c_int),
                ("embd_type", C.c_int), ("embd", C.c_void_p), ("out_norm", C.c_void_p),
                ("output_type", C.c_int), ("output", C.c_void_p), ("src_on_device", C.c_int)]


class LayerDesc(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("ffn_norm", C.c_void_p), ("q_type", C.c_int), ("k_type", C.c_int), ("v_type", C.c_int),
                ("o_type", C.c_int), ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
                ("o", C.c_void_p), ("moe", MoeDesc)]


_lib = None


def lib() -> C.CDLL:
    """Load libqms_cuda.so (built by large_model_b200.build); raises when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `python -m large_model_b200.build`")
    L = C.CDLL(str(LIB_PATH))
    vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
    L.qms_cuda_last_error.restype = C.c_char_p
    L.qms_cuda_init.argtypes = [i32]
    L.qms_cuda_stream_sync.argtypes = [vp]
    L.qms_cuda_quantize_q8.argtypes = [vp, i64, i64, vp, vp]
    L.qms_cuda_matvec_q8.argtypes = [i32, vp, i64, i64, vp, i32, vp, vp]
    L.qms_cuda_matvec_f32.argtypes = [vp, i64, i64, vp, i32, vp, vp]
    L.qms_cuda_moe_create.argtypes = [C.POINTER(MoeDesc), C.POINTER(vp)]
    L.qms_cuda_moe_destroy.argtypes = [vp]
    L.qms_cuda_moe_destroy.restype = None
    L.qms_cuda_moe_device_bytes.argtypes = [vp]
    L.qms_cuda_moe_device_bytes.restype = i64
    L.qms_cuda_moe_reserve.argtypes = [vp, i32]
    L.qms_cuda_moe_forward.argtypes = [vp, vp, i32, vp, vp, vp, vp, vp, vp]
    L.qms_cuda_moe_forward_host.argtypes = [vp, vp, i32, vp, vp, vp, vp]
    L.qms_cuda_moe_set_kernel_events.argtypes = [vp, C.POINTER(vp)]
    L.qms_cuda_moe_status.argtypes = [vp]
    L.qms_cuda_moe_create_shard.argtypes = [C.POINTER(MoeDesc), i32, i32, C.POINTER(vp)]
    L.qms_cuda_moe_route.argtypes = [vp, vp, i32, vp, vp, vp, vp]
    L.qms_cuda_moe_experts.argtypes = [vp, vp, vp, i32, vp, vp]
    L.qms_cuda_moe_experts_q8.argtypes = [vp, vp, vp, i32, vp, vp]
    L.qms_cuda_sample.argtypes = [vp, i32, C.c_float, C.c_float, i32, vp, vp, vp]
    L.qms_cuda_moe_combine.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp]
    L.qms_cuda_ep_pack.argtypes = [vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]
    L.qms_cuda_ep_combine.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp]
    L.qms_cuda_model_create.argtypes = [C.POINTER(ModelDesc), C.POINTER(vp)]
    L.qms_cuda_model_set_layer.argtypes = [vp, i32, C.POINTER(LayerDesc)]
    L.qms_cuda_model_free.argtypes = [vp]
    L.qms_cuda_model_free.restype = None
    L.qms_cuda_model_device_bytes.argtypes = [vp]
    L.qms_cuda_model_device_bytes.restype = i64
    L.qms_cuda_forward.argtypes = [vp, vp, i32, i32, vp, i32, vp]
    L.qms_cuda_forward_dev.argtypes = [vp, vp, i32, vp, vp, i32, vp]
    L.qms_cuda_decode_step.argtypes = [vp, vp, vp, vp, vp]
    L.qms_cuda_model_set_sequences.argtypes = [vp, i32]
    L.qms_cuda_model_copy_sequence.argtypes = [vp, i32, i32, i32]
    L.qms_cuda_model_set_kv_type.argtypes = [vp, i32]
    L.qms_cuda_forward_seq.argtypes = [vp, i32, vp, i32, i32, vp, i32, vp]
    L.qms_cuda_forward_batch.argtypes = [vp, i32, vp, vp, vp]
    L.qms_cuda_decode_batch.argtypes = [vp, i32, vp, vp, vp, vp]
    L.qms_cuda_model_reserve.argtypes = [vp, i32]
    L.qms_cuda_model_status.argtypes = [vp]
    L.qms_cuda_model_profile.argtypes = [vp, i32, vp]
    L.qms_cuda_moe_route_noalloc.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp, vp, vp]
    _lib = L
    return L


def check(rc: int):
    if rc != OK:
        raise QmsCudaError(rc, lib().qms_cuda_last_error().decode())


def declared_functions() -> list[str]:
    """Function names declared in include/*.h (the exported C ABI)."""
    import re
    names = []
    for h in sorted((PKG.parent / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(qms_cuda_\w+)\s*\(", text)
    return sorted(set(names))


# ---- torch plumbing ----------------------------------------------------------------------------

def _torch():
    import torch
    return torch


def _ptr(t) -> C.c_void_p | None:
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream=None) -> C.c_void_p:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def init(device: int = 0):
    check(lib().qms_cuda_init(device))


def quantize_q8(x):
    """x: CUDA float32 [rows][n] -> uint8 [rows][n/32*44] holding QmsQ8 blocks."""
    torch = _torch()
    x = x.contiguous()
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty((rows, n // 32 * 44), dtype=torch.uint8, device=x.device)
    check(lib().qms_cuda_quantize_q8(_ptr(x), n, rows, _ptr(out), _stream()))
    return out


def sample(logits, temp: float, top_p: float, top_k: int, rng=None, token=None, stream=None):
    """One draw of the chat sampler on the device (qms_cuda_sample): logits CUDA float32 [vocab];
    rng a CUDA int64 [1] holding the uint64 generator state (advanced in place; may be None when
    temp <= 0). Returns the CUDA int32 [1] token tensor."""
    torch = _torch()
    if token is None:
        token = torch.empty((1,), dtype=torch.int32, device=logits.device)
    check(lib().qms_cuda_sample(_ptr(logits.contiguous()), logits.numel(), float(temp), float(top_p), int(top_k),
                                _ptr(rng), _ptr(token), _stream(stream)))
    return token


def matvec_q8(typ: int, w, rows: int, cols: int, xq, T: int):
    torch = _torch()
    y = torch.empty((T, rows), dtype=torch.float32, device=w.device)
    check(lib().qms_cuda_matvec_q8(typ, _ptr(w), rows, cols, _ptr(xq), T, _ptr(y), _stream()))
    return y


def matvec_f32(w, x):
    torch = _torch()
    rows, cols = w.shape
    x = x.reshape(-1, cols).contiguous()
    y = torch.empty((x.shape[0], rows), dtype=torch.float32, device=w.device)
    check(lib().qms_cuda_matvec_f32(_ptr(w), rows, cols, _ptr(x), x.shape[0], _ptr(y), _stream()))
    return y


class MoeLayer:
    """One resident MoE layer (the reference's moe(), src/model.c:1032)."""

    def __init__(self, n_embd: int, n_expert: int, n_used: int, n_ff: int, router, gate, up, down,
                 gate_type: int = T_Q4_0, up_type: int = T_Q4_0, down_type: int = T_Q4_0, shard=None):
        """shard = (expert_base, n_local): gate/up/down hold only those experts (a shard for expert
        parallelism, qms_cuda_moe_create_shard); the router always has all n_expert rows."""
        on_dev = not isinstance(router, np.ndarray)
        self._keep = (router, gate, up, down)
        ptr = (lambda a: a.ctypes.data) if not on_dev else (lambda t: t.data_ptr())
        d = MoeDesc(n_embd, n_expert, n_used, n_ff, gate_type, up_type, down_type,
                    ptr(router), ptr(gate), ptr(up), ptr(down), int(on_dev))
        h = C.c_void_p()
        if shard is None:
            check(lib().qms_cuda_moe_create(C.byref(d), C.byref(h)))
        else:
            check(lib().qms_cuda_moe_create_shard(C.byref(d), int(shard[0]), int(shard[1]), C.byref(h)))
        self._keep = None
        self.h = h
        self.n_embd, self.n_expert, self.n_used, self.n_ff = n_embd, n_expert, n_used, n_ff
        self.expert_base, self.n_local = (0, n_expert) if shard is None else (int(shard[0]), int(shard[1]))

    @classmethod
    def shard_from_synth(cls, layer, expert_base: int, n_local: int) -> "MoeLayer":
        """Experts [expert_base, expert_base + n_local) of a synth layer (host arrays)."""
        E, F = layer.n_embd, layer.n_ff
        gu_bytes = F * (E // 32) * 18
        dn_bytes = E * (F // 32) * (20 if layer.down_type == T_Q4_1 else 18)
        sl = lambda a, per: np.ascontiguousarray(a[expert_base * per:(expert_base + n_local) * per])
        return cls(E, layer.n_expert, layer.n_used, F, layer.router, sl(layer.gate, gu_bytes), sl(layer.up, gu_bytes),
                   sl(layer.down, dn_bytes), layer.gate_type, layer.up_type, layer.down_type,
                   shard=(expert_base, n_local))

    @classmethod
    def from_synth(cls, layer) -> "MoeLayer":
        return cls(layer.n_embd, layer.n_expert, layer.n_used, layer.n_ff, layer.router, layer.gate,
                   layer.up, layer.down, layer.gate_type, layer.up_type, layer.down_type)

    def close(self):
        if getattr(self, "h", None):
            lib().qms_cuda_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        return lib().qms_cuda_moe_device_bytes(self.h)

    def status(self):
        """Raise if a bounded wait inside the layer's kernels gave up since the last check."""
        check(lib().qms_cuda_moe_status(self.h))

    def reserve(self, T: int):
        check(lib().qms_cuda_moe_reserve(self.h, T))

    def set_kernel_events(self, events):
        """events: 6 torch.cuda.Event(enable_timing=True) recorded around the three kernels of
        every following forward (or None to stop)."""
        if events is None:
            check(lib().qms_cuda_moe_set_kernel_events(self.h, None))
            return
        torch = _torch()
        for e in events:                      # torch creates the CUDA event on its first record
            if not e.cuda_event:
                e.record(torch.cuda.current_stream())
        torch.cuda.current_stream().synchronize()
        arr = (C.c_void_p * 6)(*[C.c_void_p(e.cuda_event) for e in events])
        self._events = events
        check(lib().qms_cuda_moe_set_kernel_events(self.h, arr))

    def forward(self, xn, out=None, sel=None, wts=None, logits=None, resid=None, stream=None):
        """xn: CUDA float32 [T][n_embd]. Returns out (CUDA float32 [T][n_embd])."""
        torch = _torch()
        xn = xn.reshape(-1, self.n_embd)
        T = xn.shape[0]
        if out is None:
            out = torch.empty_like(xn)
        check(lib().qms_cuda_moe_forward(self.h, _ptr(xn), T, _ptr(out), _ptr(sel), _ptr(wts), _ptr(logits),
                                          _ptr(resid), _stream(stream)))
        return out

    def route(self, xn):
        """Forward that also returns (out, sel, wts, logits) as CUDA tensors."""
        torch = _torch()
        xn = xn.reshape(-1, self.n_embd)
        T = xn.shape[0]
        sel = torch.empty((T, self.n_used), dtype=torch.int32, device=xn.device)
        wts = torch.empty((T, self.n_used), dtype=torch.float32, device=xn.device)
        logits = torch.empty((T, self.n_expert), dtype=torch.float32, device=xn.device)
        out = self.forward(xn, sel=sel, wts=wts, logits=logits)
        return out, sel, wts, logits

    def route_only(self, xn, stream=None):
        """Routing of T tokens (qms_cuda_moe_route): (sel, wts) CUDA int32 / float32 [T][n_used]."""
        torch = _torch()
        xn = xn.reshape(-1, self.n_embd)
        T = xn.shape[0]
        sel = torch.empty((T, self.n_used), dtype=torch.int32, device=xn.device)
        wts = torch.empty((T, self.n_used), dtype=torch.float32, device=xn.device)
        check(lib().qms_cuda_moe_route(self.h, _ptr(xn), T, _ptr(sel), _ptr(wts), None, _stream(stream)))
        return sel, wts

    def experts(self, x, expert, dn=None, stream=None):
        """Expert FFNs of rows x [S][n_embd] with local expert ids expert [S] (qms_cuda_moe_experts):
        returns dn [S][n_embd], the unweighted down rows."""
        torch = _torch()
        S = x.shape[0]
        if dn is None:
            dn = torch.empty((S, self.n_embd), dtype=torch.float32, device=x.device)
        check(lib().qms_cuda_moe_experts(self.h, _ptr(x), _ptr(expert), S, _ptr(dn), _stream(stream)))
        return dn

    def experts_q8(self, xq, expert, dn=None, stream=None):
        """The same from quantised rows (qms_cuda_moe_experts_q8): xq uint8 [S][n_embd/32 * 44], QmsQ8
        blocks as quantize_q8 returns them."""
        torch = _torch()
        S = xq.shape[0]
        if dn is None:
            dn = torch.empty((S, self.n_embd), dtype=torch.float32, device=xq.device)
        check(lib().qms_cuda_moe_experts_q8(self.h, _ptr(xq), _ptr(expert), S, _ptr(dn), _stream(stream)))
        return dn

    def forward_host(self, xn: np.ndarray, out: np.ndarray | None = None, with_routing: bool = False):
        """Host-buffer entry point (copies in, runs, copies out, waits)."""
        xn = np.ascontiguousarray(xn, np.float32).reshape(-1, self.n_embd)
        T = xn.shape[0]
        if out is None:
            out = np.empty_like(xn)
        sel = np.empty((T, self.n_used), np.int32) if with_routing else None
        wts = np.empty((T, self.n_used), np.float32) if with_routing else None
        p = lambda a: None if a is None else C.c_void_p(a.ctypes.data)
        check(lib().qms_cuda_moe_forward_host(self.h, p(xn), T, p(out), p(sel), p(wts), None))
        return (out, sel, wts) if with_routing else out


def combine(dn, wts, resid=None, out=None, stream=None):
    """out[t] = resid[t] + sum_j wts[t][j] * dn[t*K + j] in selection order (qms_cuda_moe_combine)."""
    torch = _torch()
    T, K = wts.shape
    E = dn.shape[-1]
    if out is None:
        out = torch.empty((T, E), dtype=torch.float32, device=dn.device)
    check(lib().qms_cuda_moe_combine(_ptr(dn), _ptr(wts), T, K, E, _ptr(resid), _ptr(out), _stream(stream)))
    return out


def ep_pack(xn, sel, n_expert: int, n_rank: int, cap: int, err=None, stream=None):
    """Expert-parallel dispatch buffers on the device (qms_cuda_ep_pack): xn CUDA float32 [T][E],
    sel CUDA int32 [T][K]. Returns (send_x uint8 [n_rank * cap][E/32 * 44] of QmsQ8 rows,
    send_e int32 [n_rank * cap] local expert ids or -1, slot int32 [T][K] entry of each slot or -1);
    err (CUDA int32 [1] or None) gets bit 0 set when a slot does not fit its segment."""
    torch = _torch()
    xn, sel = xn.contiguous(), sel.contiguous()
    T, K = sel.shape
    E = xn.shape[-1]
    send_x = torch.empty((n_rank * cap, E // 32 * 44), dtype=torch.uint8, device=xn.device)
    send_e = torch.empty((n_rank * cap,), dtype=torch.int32, device=xn.device)
    slot = torch.empty((T, K), dtype=torch.int32, device=xn.device)
    check(lib().qms_cuda_ep_pack(_ptr(xn), _ptr(sel), T, K, E, n_expert, n_rank, cap, _ptr(send_x), _ptr(send_e),
                                 _ptr(slot), _ptr(err), _stream(stream)))
    return send_x, send_e, slot


def ep_combine(ret, slot, wts, resid=None, out=None, stream=None):
    """out[t] = resid[t] + sum_j wts[t][j] * ret[slot[t][j]] in selection order (qms_cuda_ep_combine)."""
    torch = _torch()
    T, K = wts.shape
    E = ret.shape[-1]
    if out is None:
        out = torch.empty((T, E), dtype=torch.float32, device=ret.device)
    check(lib().qms_cuda_ep_combine(_ptr(ret), _ptr(slot), _ptr(wts), T, K, E, _ptr(resid), _ptr(out),
                                    _stream(stream)))
    return out


# ---- the whole model (qms_model_load / qms_forward, src/model.h:135-141) ------------------------------

class Model:
    """A Qwen3-MoE model resident on the current device (qms_cuda_model_*).

    cfg: an object with the config fields of synth.ModelCfg. Tensors are added with the GGUF names
    and layouts qms_model_load reads (src/model.c:314-387): `trunk` holds token_embd.weight,
    output_norm.weight and (unless tied) output.weight; set_layer(l, tensors) takes layer l's
    blk.{l}.* tensors. Arrays are numpy (host) or torch CUDA tensors (device)."""

    def __init__(self, cfg, trunk: dict, ctx: int, embd_type: int = T_Q4_0, output_type: int | None = None):
        on_dev = not isinstance(trunk["token_embd.weight"], np.ndarray)
        ptr = (lambda a: a.ctypes.data) if not on_dev else (lambda t: t.data_ptr())
        out = trunk.get("output.weight")
        otype = (cfg.output_type if output_type is None else output_type) if out is not None else embd_type
        d = ModelDesc(cfg.n_layer, cfg.n_embd, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.n_expert, cfg.n_used,
                      cfg.n_ff, cfg.vocab, float(cfg.eps), float(cfg.rope_base), int(ctx), embd_type,
                      ptr(trunk["token_embd.weight"]), ptr(trunk["output_norm.weight"]), otype,
                      None if out is None else ptr(out), int(on_dev))
        h = C.c_void_p()
        check(lib().qms_cuda_model_create(C.byref(d), C.byref(h)))
        self.h = h
        self.cfg = cfg
        self.ctx = ctx

    def set_layer(self, l: int, t: dict, types: dict | None = None):
        """t: the layer's tensors by their short names (attn_norm, attn_q_norm, attn_k_norm, ffn_norm,
        attn_q, attn_k, attn_v, attn_output, ffn_gate_inp, ffn_gate_exps, ffn_up_exps, ffn_down_exps)."""
        types = types or {}
        on_dev = not isinstance(t["attn_q"], np.ndarray)
        ptr = (lambda a: a.ctypes.data) if not on_dev else (lambda x: x.data_ptr())
        c = self.cfg
        ty = lambda k: types.get(k, T_Q4_0)
        moe = MoeDesc(c.n_embd, c.n_expert, c.n_used, c.n_ff, ty("ffn_gate_exps"), ty("ffn_up_exps"),
                      ty("ffn_down_exps"), ptr(t["ffn_gate_inp"]), ptr(t["ffn_gate_exps"]), ptr(t["ffn_up_exps"]),
                      ptr(t["ffn_down_exps"]), int(on_dev))
        ld = LayerDesc(ptr(t["attn_norm"]), ptr(t["attn_q_norm"]), ptr(t["attn_k_norm"]), ptr(t["ffn_norm"]),
                       ty("attn_q"), ty("attn_k"), ty("attn_v"), ty("attn_output"), ptr(t["attn_q"]),
                       ptr(t["attn_k"]), ptr(t["attn_v"]), ptr(t["attn_output"]), moe)
        check(lib().qms_cuda_model_set_layer(self.h, int(l), C.byref(ld)))

    @classmethod
    def from_synth(cls, cfg, seed: int, ctx: int) -> "Model":
        """The seeded synthetic model of synth.write_gguf (same bytes), uploaded tensor by tensor."""
        from . import synth
        names = synth.model_tensors(cfg)
        trunk = {}
        i = 0
        while i < len(names) and not names[i][0].startswith("blk."):
            trunk[names[i][0]] = np.ascontiguousarray(synth.tensor_data(cfg, seed, i))
            i += 1
        m = cls(cfg, trunk, ctx)
        del trunk
        for l in range(cfg.n_layer):
            t = {}
            while i < len(names) and names[i][0].startswith(f"blk.{l}."):
                t[names[i][0].split(".")[2]] = np.ascontiguousarray(synth.tensor_data(cfg, seed, i))
                i += 1
            m.set_layer(l, t)
        return m

    def close(self):
        if getattr(self, "h", None):
            lib().qms_cuda_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        return lib().qms_cuda_model_device_bytes(self.h)

    def reserve(self, T: int):
        check(lib().qms_cuda_model_reserve(self.h, T))

    def status(self):
        check(lib().qms_cuda_model_status(self.h))

    def profile(self, on: bool = True):
        """Switch the section timers; returns the sums since the last read (ms: qkv, attn, o_proj,
        router, fetch, moe, output)."""
        ms = (C.c_double * 7)()
        check(lib().qms_cuda_model_profile(self.h, int(on), ms))
        return list(ms)

    def forward(self, ids, pos0: int, all_logits: bool = False, trace: bool = False, seq: int = 0):
        """qms_forward on host buffers (sequence seq's KV cache): returns logits (numpy [vocab] or
        [T][vocab]) and, with trace, the selected experts [n_layer][T][n_used]."""
        ids = np.ascontiguousarray(ids, np.int32)
        T = ids.shape[0]
        V = self.cfg.vocab
        logits = np.empty((T, V) if all_logits else (V,), np.float32)
        sel = np.empty((self.cfg.n_layer, T, self.cfg.n_used), np.int32) if trace else None
        check(lib().qms_cuda_forward_seq(self.h, int(seq), C.c_void_p(ids.ctypes.data), T, int(pos0),
                                         C.c_void_p(logits.ctypes.data), int(all_logits),
                                         None if sel is None else C.c_void_p(sel.ctypes.data)))
        return (logits, sel) if trace else logits

    def set_sequences(self, n_seq: int):
        """KV caches for n_seq sequences (qms_cuda_model_set_sequences; caches cleared)."""
        check(lib().qms_cuda_model_set_sequences(self.h, int(n_seq)))

    def set_kv_type(self, kv_type: int):
        """KV cache elements: T_F32 (the reference's) or T_F16 (compacted); caches cleared."""
        check(lib().qms_cuda_model_set_kv_type(self.h, int(kv_type)))

    def copy_sequence(self, src: int, dst: int, npos: int):
        check(lib().qms_cuda_model_copy_sequence(self.h, int(src), int(dst), int(npos)))

    def forward_batch(self, ids, pos):
        """One token for each of B sequences (host ids[B], pos[B]): returns logits [B][vocab]."""
        ids = np.ascontiguousarray(ids, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        B = ids.shape[0]
        assert pos.shape == (B,)
        logits = np.empty((B, self.cfg.vocab), np.float32)
        check(lib().qms_cuda_forward_batch(self.h, B, C.c_void_p(ids.ctypes.data), C.c_void_p(pos.ctypes.data),
                                           C.c_void_p(logits.ctypes.data)))
        return logits

    def decode_batch(self, tok, pos, logits=None, stream=None):
        """One greedy step for B sequences on the device: tok / pos torch CUDA int32 [B], updated
        in place (qms_cuda_decode_batch)."""
        check(lib().qms_cuda_decode_batch(self.h, tok.numel(), _ptr(tok), _ptr(pos), _ptr(logits), _stream(stream)))

    def forward_dev(self, ids, pos, logits, all_logits: bool = False, stream=None):
        """Device buffers (torch CUDA int32 ids [T], int32 pos [1], float32 logits)."""
        check(lib().qms_cuda_forward_dev(self.h, _ptr(ids), ids.numel(), _ptr(pos), _ptr(logits), int(all_logits),
                                         _stream(stream)))

    def decode_step(self, tok, pos, logits=None, stream=None):
        """One greedy step on the device: tok / pos torch CUDA int32 [1], updated in place."""
        check(lib().qms_cuda_decode_step(self.h, _ptr(tok), _ptr(pos), _ptr(logits), _stream(stream)))
