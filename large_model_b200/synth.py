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


def zipf_router(layer: MoeLayer, s: float = 1.1, seed: int = 7, scale: float = 2.0) -> MoeLayer:
    """Bias the router rows so expert popularity follows Zipf(s) (config 5): adding a mean
    direction with per-expert strength log(1/rank^s) makes popular experts win more often."""
    rng = np.random.default_rng(seed)
    X, E = layer.router.shape
    rank = rng.permutation(X) + 1
    bias = (-s * np.log(rank)).astype(np.float32)
    direction = rng.standard_normal(E, dtype=np.float32)
    direction /= np.linalg.norm(direction)
    router = layer.router + (scale * bias[:, None] * direction[None, :] / 8.0).astype(np.float32)
    return MoeLayer(layer.n_embd, layer.n_expert, layer.n_used, layer.n_ff,
                    np.ascontiguousarray(router, np.float32), layer.gate, layer.up, layer.down,
                    layer.gate_type, layer.up_type, layer.down_type)
