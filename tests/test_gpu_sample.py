"""The chat sampler on a B200 (qms_cuda_sample, src/chat.c:36-69) through the C ABI: the same
token and generator state as the reference's draws (tests/golden/sampler_golden.npz, made by
the reference's own sample()) and as the oracle's restatement on further seeded rows, with the
generator state carried on the device from one draw to the next."""
from __future__ import annotations

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu


def _draws(cuda, l, temp, top_p, top_k, seed, n=2):
    import torch
    x = torch.from_numpy(l).cuda()
    st = torch.tensor([np.int64(np.uint64(seed).view(np.int64))], dtype=torch.int64, device="cuda")
    out = []
    for _ in range(n):
        t = cuda.sample(x, temp, top_p, top_k, rng=st)
        torch.cuda.synchronize()
        out.append((int(t.item()), int(np.int64(st.item()).view(np.uint64))))
    return out


def test_sample_matches_reference_golden(cuda):
    from conftest import ROOT
    g = np.load(ROOT / "tests" / "golden" / "sampler_golden.npz")
    for name, (l, temp, top_p, top_k, seed) in cases.sampler_cases().items():
        for k, (t, st) in enumerate(_draws(cuda, l, temp, top_p, top_k, seed)):
            assert t == int(g[f"{name}/tokens"][k]), f"{name} draw {k}"
            if temp > 0:
                assert st == int(g[f"{name}/states"][k]), f"{name} draw {k}: generator state"


def test_sample_matches_oracle(cuda, oracle):
    rng = np.random.default_rng(17)
    for i in range(60):
        V = int(rng.choice([2, 31, 1024, 1025, 50000, 151936]))
        l = (rng.standard_normal(V) * rng.choice([0.2, 1.0, 6.0])).astype(np.float32)
        if i % 4 == 0:
            l = np.round(l).astype(np.float32)              # ties at the K-th candidate
        if i % 9 == 0:
            l[:] = 1.5                                      # all equal
        temp, top_p = float(rng.choice([0.0, 0.4, 1.0, 3.0])), float(rng.choice([0.2, 0.8, 1.0]))
        top_k, seed = int(rng.choice([0, 1, 3, 100, 1024])), int(rng.integers(0, 2**63))
        st, want = seed, []
        for _ in range(3):
            t, st = oracle.sample(l, temp, top_p, top_k, st)
            want.append((t, st if temp > 0 else seed))
        got = _draws(cuda, l, temp, top_p, top_k, seed, n=3)
        assert got == want, f"case {i}: V={V} temp={temp} top_p={top_p} top_k={top_k}"


def test_sample_rejects_large_top_k(cuda):
    import torch
    x = torch.zeros(5000, device="cuda")
    st = torch.zeros(1, dtype=torch.int64, device="cuda")
    with pytest.raises(cuda.QmsCudaError):
        cuda.sample(x, 1.0, 0.9, 2000, rng=st)
    assert int(cuda.sample(x, 0.0, 0.9, 2000).item()) == 0      # greedy needs no candidates
