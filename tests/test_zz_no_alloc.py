"""qms_cuda_moe_route_noalloc: routing for callers that may not allocate device memory (code
under another framework's memory pool or allocator hooks, plugin hosts that forbid cudaMalloc
after start-up, deployments that reserve all of HBM up front). It must give what the normal
entry point reports (sel / wts / logits of qms_cuda_moe_forward) on consecutive calls, using
only the library's fixed scratch array. This file is collected last on purpose.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from large_model_b200 import synth

pytestmark = pytest.mark.gpu

ULP_TOL = 2     # renormalised weights, same bar as tests/test_gpu_moe.py


def _bind(L):
    f = L.qms_cuda_moe_route_noalloc
    f.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                  C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return f


def _ulps(a, b):
    a = a.view(np.int32).astype(np.int64)
    b = b.view(np.int32).astype(np.int64)
    return int(np.abs(a - b).max())


def test_route_noalloc_matches_forward_on_consecutive_calls(cuda):
    import torch
    L = cuda.lib()
    route = _bind(L)
    layer = synth.make_moe_layer("30b", seed=77)
    X, E, K = layer.n_expert, layer.n_embd, layer.n_used
    m = cuda.MoeLayer.from_synth(layer)
    router = torch.from_numpy(layer.router).cuda()
    stream = torch.cuda.current_stream()
    # two calls in a row: T=3 (top-k inside the router kernel) then T=20 (separate top-k kernel)
    for call, T in enumerate((3, 20)):
        xn = torch.from_numpy(synth.make_hidden(E, T, seed=500 + call)).cuda()
        _, sel_ref, wts_ref, logits_ref = m.route(xn)
        sel = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
        wts = torch.full((T, K), -1.0, dtype=torch.float32, device="cuda")
        logits = torch.empty((T, X), dtype=torch.float32, device="cuda")
        rc = route(router.data_ptr(), X, E, K, xn.data_ptr(), T, sel.data_ptr(), wts.data_ptr(),
                   logits.data_ptr(), C.c_void_p(stream.cuda_stream))
        assert rc == 0, L.qms_cuda_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(sel, sel_ref), f"call {call}: selected experts differ"
        assert torch.equal(logits.view(torch.int32), logits_ref.view(torch.int32)), f"call {call}: logits differ"
        assert _ulps(wts.cpu().numpy(), wts_ref.cpu().numpy()) <= ULP_TOL, f"call {call}: weights differ"
        # logits are optional: without them the library keeps its own copy in the fixed array
        sel2 = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
        wts2 = torch.full((T, K), -1.0, dtype=torch.float32, device="cuda")
        rc = route(router.data_ptr(), X, E, K, xn.data_ptr(), T, sel2.data_ptr(), wts2.data_ptr(), None,
                   C.c_void_p(stream.cuda_stream))
        assert rc == 0, L.qms_cuda_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(sel2, sel_ref) and torch.equal(wts2, wts)
    m.close()


def test_route_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    L = cuda.lib()
    route = _bind(L)
    E, X, K, T = 4096, 128, 8, 65
    router = torch.zeros((X, E), dtype=torch.float32, device="cuda")
    xn = torch.zeros((T, E), dtype=torch.float32, device="cuda")
    sel = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, K), dtype=torch.float32, device="cuda")
    rc = route(router.data_ptr(), X, E, K, xn.data_ptr(), T, sel.data_ptr(), wts.data_ptr(), None, None)
    assert rc == cuda.EINVAL
    assert "64 tokens" in L.qms_cuda_last_error().decode()
    rc = route(router.data_ptr(), X, 8192, K, xn.data_ptr(), 1, sel.data_ptr(), wts.data_ptr(), None, None)
    assert rc == cuda.EINVAL
