"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

No public dataset or checkpoint is involved: every tensor is drawn from numpy's PCG64
(`default_rng(seed)`) exactly as the configs describe — Q4_0 nibbles uniform 0..15, fp16
block scales U(0.002, 0.006), F32 router ~N(0, 0.02), hidden vectors ~N(0, 1). Tensors use
the GGUF layout the reference loads (stacked experts, ggml block structs), so the same bytes
feed libqms_cuda, the oracle and the reference build.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

T_F32, T_F16, T_Q4_0, T_Q4_1, T_Q8_0, T_Q6_K = 0, 1, 2, 3, 8, 14

# name: (n_embd, n_expert, n_used, n_ff)
MOE_SHAPES = {
    "tiny": (512, 32, 4, 256),          # config 1's MoE block
    "30b": (2048, 128, 8, 768),         # Qwen3-30B-A3B
    "235b": (4096, 128, 8, 1536),       # Qwen3-235B-A22B (config 2)
}


def q4_0_blocks(rng: np.random.Generator, nblocks: int, lo: float = 0.002, hi: float = 0.006) -> np.ndarray:
    """nblocks ggml Q4_0 blocks {f16 d; u8 qs[16]} as a flat uint8 array."""
    blk = np.empty((nblocks, 18), np.uint8)
    d = rng.uniform(lo, hi, nblocks).astype(np.float16)
    blk[:, 0:2] = d.view(np.uint8).reshape(nblocks, 2)
    blk[:, 2:] = np.frombuffer(rng.bytes(nblocks * 16), np.uint8).reshape(nblocks, 16)
    return blk.reshape(-1)


def q4_1_blocks(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    """nblocks ggml Q4_1 blocks {f16 d; f16 m; u8 qs[16]}: d as Q4_0, m = -8 d (centred)."""
    blk = np.empty((nblocks, 20), np.uint8)
    d = rng.uniform(0.002, 0.006, nblocks).astype(np.float32)
    m = (-8.0 * d * rng.uniform(0.9, 1.1, nblocks)).astype(np.float16)
    blk[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    blk[:, 2:4] = m.view(np.uint8).reshape(nblocks, 2)
    blk[:, 4:] = np.frombuffer(rng.bytes(nblocks * 16), np.uint8).reshape(nblocks, 16)
    return blk.reshape(-1)


@dataclass
class MoeLayer:
    """One MoE layer in GGUF layout (reference src/model.h:229-243)."""
    n_embd: int
    n_expert: int
    n_used: int
    n_ff: int
    router: np.ndarray          # F32 [n_expert][n_embd]
    gate: np.ndarray            # uint8, [n_expert][n_ff] rows of n_embd
    up: np.ndarray              # uint8, [n_expert][n_ff] rows of n_embd
    down: np.ndarray            # uint8, [n_expert][n_embd] rows of n_ff
    gate_type: int = T_Q4_0
    up_type: int = T_Q4_0
    down_type: int = T_Q4_0

    @property
    def expert_bytes(self) -> int:
        return self.gate.nbytes // self.n_expert + self.up.nbytes // self.n_expert + \
            self.down.nbytes // self.n_expert

    def bytes_per_token(self) -> int:
        """Algorithmic bytes one decode token reads: n_used experts plus the F32 router."""
        return self.n_used * self.expert_bytes + self.router.nbytes


def make_moe_layer(shape: str | tuple, seed: int = 0, down_type: int = T_Q4_0,
                   router_std: float = 0.02) -> MoeLayer:
    E, X, K, F = MOE_SHAPES[shape] if isinstance(shape, str) else shape
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((X, E), dtype=np.float32) * np.float32(router_std)).astype(np.float32)
    gate = q4_0_blocks(rng, X * F * E // 32)
    up = q4_0_blocks(rng, X * F * E // 32)
    down = q4_1_blocks(rng, X * E * F // 32) if down_type == T_Q4_1 else q4_0_blocks(rng, X * E * F // 32)
    return MoeLayer(E, X, K, F, router, gate, up, down, down_type=down_type)


def make_hidden(n_embd: int, T: int, seed: int = 1) -> np.ndarray:
    """T post-RMSNorm hidden vectors ~N(0, 1), fp32 [T][n_embd]."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((T, n_embd), dtype=np.float32)


def zipf_layer_and_hidden(layer: MoeLayer, T: int, s: float = 1.1, seed: int = 7, mu: float = 4.0):
    """Config 5's skewed routing: expert popularity follows Zipf(s) over the experts. The router is
    bias-free (a plain matmul, src/model.c:1043), so the popularity comes from a component shared by
    every token: hidden x_t = z_t + mu * u with z_t ~ N(0, 1) and u a random unit vector, and router
    rows w_e + (b_e / mu) u with b_e = sigma * s * log(1 / rank_e) (sigma = the logits' own spread,
    0.02 * sqrt(n_embd)), so logit_e = w_e.z_t + b_e + small terms: the noise of the top-k plays the
    Gumbel noise of Plackett-Luce sampling and expert e is picked with probability ~ rank_e^-s.
    Returns (layer with the biased router, hidden [T][n_embd])."""
    rng = np.random.default_rng(seed)
    X, E = layer.router.shape
    rank = rng.permutation(X) + 1
    sigma = 0.02 * np.sqrt(E)
    b = (sigma * s * -np.log(rank)).astype(np.float64)
    u = rng.standard_normal(E)
    u /= np.linalg.norm(u)
    router = (layer.router.astype(np.float64) + (b / mu)[:, None] * u[None, :]).astype(np.float32)
    z = rng.standard_normal((T, E), dtype=np.float32)
    x = (z + np.float32(mu) * u.astype(np.float32)[None, :]).astype(np.float32)
    return (MoeLayer(layer.n_embd, layer.n_expert, layer.n_used, layer.n_ff, np.ascontiguousarray(router),
                     layer.gate, layer.up, layer.down, layer.gate_type, layer.up_type, layer.down_type), x)


# ---- whole models (configs 1, 3 and 4) ------------------------------------------------------------
# Architecture hyper-parameters of BASELINE.json's full-model configs. Every tensor is drawn from
# its own generator, default_rng([seed, tensor index]), so any tensor can be produced on its own
# (streamed into a GGUF file, or uploaded layer by layer) and always has the same bytes.

@dataclass(frozen=True)
class ModelCfg:
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_expert: int
    n_used: int
    n_ff: int
    vocab: int
    eps: float = 1e-6
    rope_base: float = 1e6
    output_type: int = T_Q6_K      # T_Q6_K, or -1 for tied embeddings (no output.weight)


MODEL_CONFIGS = {
    "tiny": ModelCfg(2, 512, 8, 2, 64, 32, 4, 256, 4096),                 # config 1
    "tiny-tied": ModelCfg(2, 512, 8, 2, 64, 32, 4, 256, 4096, output_type=-1),
    "30b": ModelCfg(48, 2048, 32, 4, 128, 128, 8, 768, 151936),           # config 3 (Qwen3-30B-A3B)
    "235b": ModelCfg(94, 4096, 64, 4, 128, 128, 8, 1536, 151936),         # config 4 (Qwen3-235B-A22B)
}


def _raw_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    """n uniform random bytes from full-range 64-bit integer draws (an order of magnitude faster
    than Generator.bytes, which matters for the 16-124 GiB full models)."""
    w = rng.integers(0, np.iinfo(np.uint64).max, (n + 7) // 8, dtype=np.uint64, endpoint=True)
    return w.view(np.uint8)[:n]


def q4_0_blocks_model(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    """Q4_0 blocks for the full-model configs: the distributions of q4_0_blocks, nibble bytes
    from 64-bit integer draws."""
    blk = np.empty((nblocks, 18), np.uint8)
    blk[:, 0:2] = rng.uniform(0.002, 0.006, nblocks).astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    blk[:, 2:] = _raw_bytes(rng, nblocks * 16).reshape(nblocks, 16)
    return blk.reshape(-1)


def q6_k_blocks(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    """nblocks ggml Q6_K super-blocks {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d} (210 bytes):
    6-bit values uniform 0..63, sub-scales uniform 2..8, d U(1.5e-4, 3e-4), so the weights have
    about the magnitude of the Q4_0 tensors (gguf-py cannot quantise Q6_K; these are raw blocks)."""
    blk = np.empty((nblocks, 210), np.uint8)
    blk[:, :192] = _raw_bytes(rng, nblocks * 192).reshape(nblocks, 192)
    blk[:, 192:208] = rng.integers(2, 9, (nblocks, 16), dtype=np.int8).view(np.uint8)
    blk[:, 208:210] = rng.uniform(1.5e-4, 3e-4, nblocks).astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    return blk.reshape(-1)


_ROW_BYTES = {T_F32: (1, 4), T_F16: (1, 2), T_Q4_0: (32, 18), T_Q4_1: (32, 20), T_Q8_0: (32, 34), T_Q6_K: (256, 210)}


def tensor_nbytes(typ: int, ne: tuple) -> int:
    per, nbytes = _ROW_BYTES[typ]
    n = int(np.prod(ne))
    return n // per * nbytes


def model_tensors(cfg: ModelCfg) -> list[tuple[str, int, tuple]]:
    """(name, ggml type, ne) of every tensor, in file order; ne[0] is the contiguous dimension
    (the layout qms_model_load expects, src/model.c:314-387)."""
    E, D, H, Hk, X, F, V = cfg.n_embd, cfg.head_dim, cfg.n_head, cfg.n_head_kv, cfg.n_expert, cfg.n_ff, cfg.vocab
    t = [("token_embd.weight", T_Q4_0, (E, V)), ("output_norm.weight", T_F32, (E,))]
    if cfg.output_type >= 0:
        t.append(("output.weight", cfg.output_type, (E, V)))
    for l in range(cfg.n_layer):
        b = f"blk.{l}."
        t += [(b + "attn_norm.weight", T_F32, (E,)), (b + "attn_q_norm.weight", T_F32, (D,)),
              (b + "attn_k_norm.weight", T_F32, (D,)), (b + "attn_q.weight", T_Q4_0, (E, H * D)),
              (b + "attn_k.weight", T_Q4_0, (E, Hk * D)), (b + "attn_v.weight", T_Q4_0, (E, Hk * D)),
              (b + "attn_output.weight", T_Q4_0, (H * D, E)), (b + "ffn_norm.weight", T_F32, (E,)),
              (b + "ffn_gate_inp.weight", T_F32, (E, X)), (b + "ffn_gate_exps.weight", T_Q4_0, (E, F, X)),
              (b + "ffn_up_exps.weight", T_Q4_0, (E, F, X)), (b + "ffn_down_exps.weight", T_Q4_0, (F, E, X))]
    return t


def tensor_data(cfg: ModelCfg, seed: int, index: int) -> np.ndarray:
    """Bytes (uint8) or values (float32) of tensor `index` of model_tensors(cfg)."""
    name, typ, ne = model_tensors(cfg)[index]
    rng = np.random.default_rng([seed, index])
    n = int(np.prod(ne))
    if typ == T_F32:
        if "ffn_gate_inp" in name:                       # router ~N(0, 0.02)
            return (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)).reshape(ne[::-1])
        return (1.0 + rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    if typ == T_Q4_0:
        return q4_0_blocks_model(rng, n // 32)
    if typ == T_Q6_K:
        return q6_k_blocks(rng, n // 256)
    raise ValueError(f"no generator for type {typ}")


def iter_model(cfg: ModelCfg, seed: int):
    """Yield (name, type, ne, data) in file order."""
    for i, (name, typ, ne) in enumerate(model_tensors(cfg)):
        yield name, typ, ne, tensor_data(cfg, seed, i)


def write_gguf(path, cfg: ModelCfg, seed: int, alignment: int = 32) -> int:
    """Write a GGUF v3 qwen3moe file with the seeded tensors (the keys read_cfg requires,
    src/model.c:279-312). Tensors are generated one at a time, so memory stays at one tensor.
    Returns the file size."""
    import struct

    def s_str(b: str) -> bytes:
        e = b.encode()
        return struct.pack("<Q", len(e)) + e

    U32, F32, STR = 4, 6, 8
    kv = [("general.architecture", STR, "qwen3moe"), ("general.alignment", U32, alignment),
          ("qwen3moe.block_count", U32, cfg.n_layer), ("qwen3moe.embedding_length", U32, cfg.n_embd),
          ("qwen3moe.attention.head_count", U32, cfg.n_head),
          ("qwen3moe.attention.head_count_kv", U32, cfg.n_head_kv),
          ("qwen3moe.attention.key_length", U32, cfg.head_dim),
          ("qwen3moe.attention.value_length", U32, cfg.head_dim),
          ("qwen3moe.expert_count", U32, cfg.n_expert), ("qwen3moe.expert_used_count", U32, cfg.n_used),
          ("qwen3moe.expert_feed_forward_length", U32, cfg.n_ff),
          ("qwen3moe.attention.layer_norm_rms_epsilon", F32, cfg.eps),
          ("qwen3moe.rope.freq_base", F32, cfg.rope_base)]
    tensors = model_tensors(cfg)
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for key, vt, val in kv:
        head += s_str(key) + struct.pack("<I", vt)
        head += s_str(val) if vt == STR else struct.pack("<I" if vt == U32 else "<f", val)
    off = 0
    offsets = []
    for name, typ, ne in tensors:
        offsets.append(off)
        head += s_str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
        head += struct.pack("<IQ", typ, off)
        off += (tensor_nbytes(typ, ne) + alignment - 1) // alignment * alignment
    head += b"\0" * ((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        for i, (name, typ, ne) in enumerate(tensors):
            data = tensor_data(cfg, seed, i)
            raw = data.tobytes()
            assert len(raw) == tensor_nbytes(typ, ne), name
            f.write(raw)
            f.write(b"\0" * ((-len(raw)) % alignment))
        return f.tell()


def model_bytes(cfg: ModelCfg) -> int:
    return sum(tensor_nbytes(t, ne) for _, t, ne in model_tensors(cfg))


def random_ids(vocab: int, n: int, seed: int) -> list[int]:
    """Uniform random prompt ids (the configs' random-id prompts)."""
    return [int(v) for v in np.random.default_rng(seed).integers(0, vocab, n)]
