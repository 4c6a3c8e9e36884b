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


def _route_call(route, router, X, E, K, xn, T, stream):
    import torch
    sel = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
    wts = torch.full((T, K), -1.0, dtype=torch.float32, device="cuda")
    logits = torch.empty((T, X), dtype=torch.float32, device="cuda")
    return sel, wts, logits


def test_route_noalloc_matches_oracle_and_allocates_nothing(cuda, oracle):
    """Against the CPU restatement of the reference's routing (src/model.c:1043-1064): bit-identical
    logits and ids, weights within 2 ulps; two calls in a row (T = 5 and an xn that is not 16-byte
    aligned with T = 20, the tiled-router path); device free memory is the same before and after."""
    import torch
    L = cuda.lib()
    route = _bind(L)
    layer = synth.make_moe_layer("235b", seed=91)
    X, E, K = layer.n_expert, layer.n_embd, layer.n_used
    router = torch.from_numpy(layer.router).cuda()
    stream = torch.cuda.current_stream()
    cases = []
    for call, (T, offset) in enumerate(((5, 0), (20, 1))):
        x = synth.make_hidden(E, T, seed=700 + call)
        flat = torch.empty(T * E + 4, dtype=torch.float32, device="cuda")
        xn = flat[offset:offset + T * E].view(T, E)          # offset 1 float: 4-byte aligned only
        xn.copy_(torch.from_numpy(x))
        cases.append((T, x, xn) + _route_call(route, router, X, E, K, xn, T, stream))
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for T, x, xn, sel, wts, logits in cases:
        rc = route(router.data_ptr(), X, E, K, xn.data_ptr(), T, sel.data_ptr(), wts.data_ptr(), logits.data_ptr(),
                   C.c_void_p(stream.cuda_stream))
        assert rc == 0, L.qms_cuda_last_error().decode()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    for T, x, xn, sel, wts, logits in cases:
        o_logits, o_sel, o_w = oracle.route(layer.router, K, x)
        assert np.array_equal(logits.cpu().numpy().view(np.uint32), o_logits.view(np.uint32)), f"T={T}: logits"
        assert np.array_equal(sel.cpu().numpy(), o_sel), f"T={T}: selected experts"
        assert _ulps(wts.cpu().numpy(), o_w) <= ULP_TOL, f"T={T}: weights"


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
