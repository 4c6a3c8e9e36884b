"""Kernel-level parity on a B200: libqms_cuda's mirrors of src/kernels.h against the oracle.

Bars: Q8 quantisation and the F32 router dot are bit-exact (same arithmetic, same order); the
Q4/Q6 integer dots meet the reference's own kernel-test criterion |got-ref|/sum|terms| < 1e-5
(tests/test_kernels.c:71-83), ref = double dot of dequantised weights and int8 activations.
"""
from __future__ import annotations

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu


def test_quantize_q8_bit_exact(cuda, oracle, golden):
    import torch
    for name, x in cases.quant_cases().items():
        got = cuda.quantize_q8(torch.from_numpy(x.reshape(1, -1)).cuda()).cpu().numpy().reshape(-1)
        assert np.array_equal(got, golden[f"quant/{name}/q8"]), name
    rng = np.random.default_rng(9)
    x = rng.standard_normal((37, 1536)).astype(np.float32) * 3
    x[5, 64:96] = 0.0
    got = cuda.quantize_q8(torch.from_numpy(x).cuda()).cpu().numpy().reshape(-1)
    want = oracle.quantize_q8(x).view(np.uint8)
    assert np.array_equal(got, want)


def test_matvec_f32_bit_exact(cuda, oracle, golden):
    import torch
    for name, (w, x) in cases.f32_cases().items():
        got = cuda.matvec_f32(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()).cpu().numpy()[0]
        assert np.array_equal(got.view(np.uint32), golden[f"f32/{name}/got"].view(np.uint32)), name
    rng = np.random.default_rng(10)
    w = (rng.standard_normal((128, 4096)) * 0.02).astype(np.float32)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    got = cuda.matvec_f32(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()).cpu().numpy()
    want = oracle.matmul(0, 128, 4096, w.view(np.uint8), x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("typ", [cases.T_Q4_0, cases.T_Q4_1, cases.T_Q6_K])
def test_matvec_q8_kernel_criterion(cuda, oracle, golden, typ):
    import torch
    worst = 0.0
    for name, (t, n, w, x) in cases.dot_cases().items():
        if t != typ:
            continue
        rows = len(w)
        xq = oracle.quantize_q8(x).reshape(rows, -1)
        xq_d = torch.from_numpy(xq.view(np.uint8).reshape(rows, -1).copy()).cuda()
        w_d = torch.from_numpy(np.ascontiguousarray(w)).cuda()
        # every weight row against every activation row: y[t][r]
        y = cuda.matvec_q8(typ, w_d, rows, n, xq_d, rows).cpu().numpy()
        for i in range(rows):
            wd = oracle.dequant_row(typ, w[i], n).astype(np.float64)
            xi = (xq[i]["q"].astype(np.float64) * xq[i]["d"][:, None]).reshape(-1)
            ref = float(np.dot(wd, xi))
            mag = float(np.abs(wd * xi).sum())
            worst = max(worst, abs(float(y[i, i]) - ref) / (mag + 1e-30))
            # and against the reference's own value from the golden file
            g = float(golden[f"dot/{name}/got"][i])
            worst = max(worst, abs(float(y[i, i]) - g) / (mag + 1e-30))
    assert worst < 1e-5, worst
