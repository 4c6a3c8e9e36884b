"""Seeded input cases shared by tests/golden/make_golden.py and the tests that read its fixtures.

The draws follow the reference's own kernel test (tests/test_kernels.c:22-39, 65-68): random
block bytes with positive fp16 scales of controlled exponent, activations uniform in
[-10000, 10000]/3000 with an all-zero 32-block every fifth trial, sizes {256 .. 8192}.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from large_model_b200 import synth  # noqa: E402

T_F32, T_F16, T_Q4_0, T_Q4_1, T_Q8_0, T_Q6_K = 0, 1, 2, 3, 8, 14
BLOCK = {T_Q4_0: (32, 18), T_Q4_1: (32, 20), T_Q6_K: (256, 210), T_Q8_0: (32, 34)}
NAMES = {T_Q4_0: "q4_0", T_Q4_1: "q4_1", T_Q6_K: "q6_k", T_Q8_0: "q8_0"}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).view(np.uint8).tobytes())
    return h.hexdigest()


def f16_bits(sign: int, exp: np.ndarray, mant: np.ndarray) -> np.ndarray:
    return ((sign << 15) | (exp << 10) | mant).astype(np.uint16)


def random_rows(rng: np.random.Generator, typ: int, n: int, rows: int) -> np.ndarray:
    """rows weight rows of n elements: random bytes, then positive fp16 scales as in
    tests/test_kernels.c:26-37 (exponent 9..12 for Q4, 5..7 for Q6_K super-scales)."""
    per, bs = BLOCK[typ]
    nb = n // per
    w = np.frombuffer(rng.bytes(rows * nb * bs), np.uint8).copy().reshape(rows, nb, bs)
    if typ in (T_Q4_0, T_Q4_1):
        d = f16_bits(0, rng.integers(9, 13, (rows, nb)), rng.integers(0, 1024, (rows, nb)))
        w[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
        if typ == T_Q4_1:
            m = f16_bits(1, rng.integers(9, 13, (rows, nb)), rng.integers(0, 1024, (rows, nb)))
            w[:, :, 2:4] = m.view(np.uint8).reshape(rows, nb, 2)
    elif typ == T_Q6_K:
        w[:, :, 192:208] = (rng.integers(0, 128, (rows, nb, 16)) - 64).astype(np.int8).view(np.uint8)
        d = f16_bits(0, rng.integers(5, 8, (rows, nb)), rng.integers(0, 1024, (rows, nb)))
        w[:, :, 208:210] = d.view(np.uint8).reshape(rows, nb, 2)
    elif typ == T_Q8_0:
        d = f16_bits(0, rng.integers(9, 13, (rows, nb)), rng.integers(0, 1024, (rows, nb)))
        w[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    return w.reshape(rows, nb * bs)


def activations(rng: np.random.Generator, n: int, rows: int) -> np.ndarray:
    x = ((rng.integers(0, 20001, (rows, n)).astype(np.float32) - 10000.0) / 3000.0).astype(np.float32)
    x[::5, :32] = 0.0
    return x


def quant_cases() -> dict:
    rng = np.random.default_rng(101)
    x = rng.standard_normal(8192).astype(np.float32)
    x[:32] = 0.0                        # amax == 0: d = 0, id = 0
    x[64:96] = 1e-30                    # tiny amax
    x[128] = 127.0 * 0.5                # exact .5 products exercise round-half-even
    y = activations(rng, 4096, 1)[0]
    return {"normal": x, "kernel_test": y}


def dot_cases() -> dict:
    rng = np.random.default_rng(202)
    out = {}
    for typ in (T_Q4_0, T_Q4_1, T_Q6_K):
        for n in (256, 768, 1536, 2048, 4096, 8192):
            rows = 10
            w = random_rows(rng, typ, n, rows)
            x = activations(rng, n, rows)
            out[f"{NAMES[typ]}_{n}"] = (typ, n, w, x)
    return out


def f32_cases() -> dict:
    rng = np.random.default_rng(303)
    out = {}
    for n in (16, 256, 4096, 4100, 33):
        w = rng.standard_normal((8, n)).astype(np.float32) * np.float32(0.02)
        x = rng.standard_normal(n).astype(np.float32)
        out[f"n{n}"] = (w, x)
    return out


def deq_cases() -> dict:
    rng = np.random.default_rng(404)
    out = {}
    for typ in (T_Q4_0, T_Q4_1, T_Q8_0, T_Q6_K):
        n = 512
        out[NAMES[typ]] = (typ, n, random_rows(rng, typ, n, 1)[0])
    return out


def moe_cases() -> dict:
    """MoE layers in the benchmark distributions, small enough for the CPU suite."""
    out = {}
    tiny = synth.make_moe_layer("tiny", seed=7)
    out["tiny_t4"] = (tiny, synth.make_hidden(tiny.n_embd, 4, seed=8))
    mid = synth.make_moe_layer((1024, 64, 8, 512), seed=9)
    out["mid_t2"] = (mid, synth.make_hidden(mid.n_embd, 2, seed=10))
    return out


def sampler_cases() -> dict:
    """Logit rows and sampler settings for the chat sampler (src/chat.c:36-69): vocabularies from
    5 to Qwen3's 151,936, ties at the top and rows of rounded values (many ties at the K-th),
    greedy, default top_k (0 -> 1024), small and large top_k, top_p below and at 1."""
    rng = np.random.default_rng(90)
    out = {}
    for i in range(48):
        V = int([5, 37, 1000, 4096, 151936][i % 5])
        scale = float([0.5, 2.0, 8.0][i % 3])
        l = (rng.standard_normal(V) * scale).astype(np.float32)
        if i % 7 == 0:
            l[rng.integers(0, V, 6)] = l.max()
        if i % 6 == 1:
            l = np.round(l).astype(np.float32)
        temp = float([0.0, 0.3, 0.7, 1.0, 1.5][i % 5 if i % 9 else 0])
        top_p = float([0.5, 0.9, 0.95, 1.0][i % 4])
        top_k = int([0, 1, 5, 40, 1024, 0][i % 6])
        seed = int(rng.integers(0, 2**63))
        out[f"s{i:02d}"] = (l, temp, top_p, top_k, seed)
    return out
