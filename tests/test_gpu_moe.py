"""MoE block parity on a B200: qms_cuda_moe_forward (C ABI) against the oracle / reference.

Bars: identical selected expert ids in identical selection order, router
logits bit-identical, renormalised weights within 2 float ulps, and the block output within
1e-3 relative L2 of the reference's integer path (observed ~1e-6: only float summation order of
the int8 dots differs). Shapes: the tiny config's block, Qwen3-30B-A3B and Qwen3-235B-A22B.
"""
from __future__ import annotations

import numpy as np
import pytest

import cases
from conftest import rel_l2
from large_model_b200 import synth

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-3          # relative L2 of the block output
ULP_TOL = 2             # renormalised routing weights


def _ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return int(np.abs(a - b).max())


def _run(cuda, layer, xn):
    import torch
    m = cuda.MoeLayer.from_synth(layer)
    out, sel, w, logits = m.route(torch.from_numpy(xn).cuda())
    torch.cuda.synchronize()
    m.status()                       # no bounded wait inside the kernels gave up
    return m, out.cpu().numpy(), sel.cpu().numpy(), w.cpu().numpy(), logits.cpu().numpy()


def _check(oracle, layer, xn, out, sel, w, logits, tag=""):
    o_out, o_sel, o_w, o_logits = oracle.moe(layer, xn)
    assert np.array_equal(logits.view(np.uint32), o_logits.view(np.uint32)), f"{tag} router logits differ"
    assert np.array_equal(sel, o_sel), f"{tag} selected experts differ"
    assert _ulps(w, o_w) <= ULP_TOL, f"{tag} weights differ by {_ulps(w, o_w)} ulps"
    err = rel_l2(out, o_out)
    assert err < OUT_TOL, f"{tag} rel L2 {err:.3e}"
    return err


@pytest.mark.parametrize("shape,T", [("tiny", 1), ("tiny", 4), ("tiny", 13), ("30b", 1), ("30b", 5),
                                     ("235b", 1), ("235b", 3), ("235b", 9)])
def test_moe_matches_oracle(cuda, oracle, shape, T):
    layer = synth.make_moe_layer(shape, seed=31 + T)
    xn = synth.make_hidden(layer.n_embd, T, seed=41 + T)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    _check(oracle, layer, xn, out, sel, w, logits, f"{shape} T={T}")
    m.close()


@pytest.mark.parametrize("shape,T", [("tiny", 1), ("tiny", 7), ("30b", 1), ("30b", 4),
                                     ("235b", 1), ("235b", 6)])
def test_moe_q4_1_down_matches_oracle(cuda, oracle, shape, T):
    """ffn_down_exps stored as Q4_1 (per-block scale and minimum), batch 1 and batched kernels."""
    layer = synth.make_moe_layer(shape, seed=71 + T, down_type=synth.T_Q4_1)
    xn = synth.make_hidden(layer.n_embd, T, seed=81 + T)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    _check(oracle, layer, xn, out, sel, w, logits, f"q4_1 {shape} T={T}")
    m.close()


def test_moe_golden_reference(cuda, golden):
    """Against outputs produced by the reference's own moe() (tests/golden)."""
    for name, (layer, xn) in cases.moe_cases().items():
        m, out, sel, w, logits = _run(cuda, layer, xn)
        assert rel_l2(out, golden[f"moe/{name}/out"]) < OUT_TOL, name
        assert sorted(set(sel.ravel().tolist())) == golden[f"moe/{name}/trace"].tolist(), name
        m.close()


def test_moe_decode_sequence_235b(cuda, oracle):
    """64 consecutive bs1 calls on one layer (scratch reuse, self-resetting counters)."""
    import torch
    layer = synth.make_moe_layer("235b", seed=5)
    xn = synth.make_hidden(layer.n_embd, 64, seed=6)
    m = cuda.MoeLayer.from_synth(layer)
    xd = torch.from_numpy(xn).cuda()
    outs, sels = [], []
    for t in range(64):
        o, s, _, _ = m.route(xd[t:t + 1])
        outs.append(o)
        sels.append(s)
    out = torch.cat(outs).cpu().numpy()
    sel = torch.cat(sels).cpu().numpy()
    m.status()
    o_out, o_sel, _, _ = oracle.moe(layer, xn)
    assert np.array_equal(sel, o_sel)
    assert rel_l2(out, o_out) < OUT_TOL
    m.close()


def test_moe_edge_cases(cuda, oracle):
    import torch
    layer = synth.make_moe_layer("tiny", seed=3)
    E = layer.n_embd
    # all-zero input: every logit 0 -> ties -> experts 0..k-1, equal weights, zero output
    xn = np.zeros((2, E), np.float32)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    _check(oracle, layer, xn, out, sel, w, logits, "zeros")
    assert sel.tolist() == [[0, 1, 2, 3]] * 2 and np.all(out == 0)
    # zero 32-blocks inside a token (d == 0 blocks) and huge / tiny magnitudes; at x1e4 every
    # probability but the top one underflows to 0.0 and the zeros tie (lower index first)
    xn = synth.make_hidden(E, 3, seed=4)
    xn[0, :64] = 0.0
    xn[1] *= 1e4
    xn[2] *= 1e-4
    out, sel, w, logits = [a.cpu().numpy() for a in m.route(torch.from_numpy(xn).cuda())]
    _check(oracle, layer, xn, out, sel, w, logits, "magnitudes")
    # tied router rows: experts 5 and 2 identical -> lower index first
    tied = synth.make_moe_layer("tiny", seed=3)
    tied.router[5] = tied.router[2]
    xt = synth.make_hidden(E, 16, seed=5)
    m2, out, sel, w, logits = _run(cuda, tied, xt)
    _check(oracle, tied, xt, out, sel, w, logits, "ties")
    # empty batch
    empty = torch.empty((0, E), dtype=torch.float32, device="cuda")
    assert m.forward(empty).shape == (0, E)
    m.close()
    m2.close()


@pytest.mark.parametrize("shape,T,down", [("tiny", 16, 2), ("tiny", 70, 3), ("tiny", 200, 3), ("30b", 16, 2),
                                          ("30b", 130, 2), ("235b", 16, 2), ("235b", 64, 3), ("235b", 200, 2),
                                          ("235b", 512, 2)])
def test_moe_grouped_mma_matches_oracle(cuda, oracle, monkeypatch, shape, T, down):
    """T >= 16: expert-grouped tcgen05 kind::i8 GEMMs against the oracle, with the batch bars: 16-slot
    tiles while experts average <= 24 slots, 64-slot tiles above (tiny T=200, 235B T=512); partial
    and multiple tiles per expert; Q4_0 and Q4_1 down. The grouped GEMV, which takes the 16-slot
    calls by default, is switched off for these layers."""
    monkeypatch.setenv("QMS_GEMV", "0")
    layer = synth.make_moe_layer(shape, seed=91 + T, down_type=down)
    xn = synth.make_hidden(layer.n_embd, T, seed=93 + T)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    _check(oracle, layer, xn, out, sel, w, logits, f"mma {shape} T={T} down={down}")
    m.close()


@pytest.mark.parametrize("shape,T,down", [("tiny", 16, 2), ("tiny", 40, 3), ("tiny", 150, 2), ("30b", 16, 2),
                                          ("30b", 64, 3), ("235b", 16, 2), ("235b", 64, 2), ("235b", 130, 3),
                                          ("235b", 300, 2)])
def test_moe_grouped_gemv_matches_oracle(cuda, oracle, shape, T, down):
    """Batched decode (experts average <= 24 slots): the expert-grouped GEMV kernels (one weight read
    per expert and call, dp4a over up to 16 slots per tile) against the oracle; Q4_0 and Q4_1 down;
    one tile per expert (235B T=16/64) up to several per expert (tiny T=150, 235B T=300)."""
    layer = synth.make_moe_layer(shape, seed=191 + T, down_type=down)
    xn = synth.make_hidden(layer.n_embd, T, seed=193 + T)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    _check(oracle, layer, xn, out, sel, w, logits, f"gemv {shape} T={T} down={down}")
    m.close()


@pytest.mark.parametrize("shape", ["tiny", "30b"])
def test_decode_routing_edge_cases(cuda, oracle, shape):
    """Batch-1 kernel (one call per token): its stream starts on the float ranking and is checked
    against the exact double ranking. Zeros tie everywhere (same experts); at 1e-30 every
    probability is exactly 1 in double and at 1e4 all but the top one underflow to 0, so the
    exact ranking takes the lowest indices while the float ranking does not: the kernel must
    restart its stream on the selected experts."""
    import torch
    layer = synth.make_moe_layer(shape, seed=12)
    E = layer.n_embd
    xs = synth.make_hidden(E, 6, seed=13)
    xs[0] = 0.0
    xs[1] *= 1e-30
    xs[2] *= 1e4
    xs[3, : E // 2] = 0.0
    xs[4] *= -3.0
    m = cuda.MoeLayer.from_synth(layer)
    xd = torch.from_numpy(xs).cuda()
    res = [m.route(xd[t:t + 1]) for t in range(xs.shape[0])]
    torch.cuda.synchronize()
    m.status()
    out, sel, w, logits = (torch.cat([r[i] for r in res]).cpu().numpy() for i in range(4))
    _check(oracle, layer, xs, out, sel, w, logits, f"decode edge {shape}")
    K = layer.n_used
    assert sel[0].tolist() == list(range(K)) and sel[1].tolist() == list(range(K))
    m.close()


def test_moe_host_entry_and_residual(cuda, oracle):
    import torch
    layer = synth.make_moe_layer("30b", seed=8)
    xn = synth.make_hidden(layer.n_embd, 2, seed=9)
    m = cuda.MoeLayer.from_synth(layer)
    out_h, sel_h, w_h = m.forward_host(xn, with_routing=True)
    o_out, o_sel, o_w, _ = oracle.moe(layer, xn)
    assert np.array_equal(sel_h, o_sel)
    assert rel_l2(out_h, o_out) < OUT_TOL
    resid = torch.from_numpy(synth.make_hidden(layer.n_embd, 2, seed=10)).cuda()
    xd = torch.from_numpy(xn).cuda()
    plain = m.forward(xd)
    fused = m.forward(xd, resid=resid)
    torch.cuda.synchronize()
    assert torch.equal(fused, resid + plain)           # h += moe(xn), src/model.c:1285
    # in place: out aliases the residual
    h = resid.clone()
    m.forward(xd, out=h, resid=h)
    assert torch.equal(h, fused)
    m.close()


def test_grouped_mma_residual_graph_and_determinism(cuda, oracle):
    """Tensor-core path (T = 48): fused residual, output aliasing the residual, CUDA-graph capture
    after reserve, bitwise reproducibility across calls."""
    import torch
    layer = synth.make_moe_layer("30b", seed=21)
    T = 48
    xn = synth.make_hidden(layer.n_embd, T, seed=22)
    m = cuda.MoeLayer.from_synth(layer)
    xd = torch.from_numpy(xn).cuda()
    plain = m.forward(xd)
    again = m.forward(xd)
    torch.cuda.synchronize()
    m.status()
    assert torch.equal(plain, again)
    o_out, _, _, _ = oracle.moe(layer, xn)
    assert rel_l2(plain.cpu().numpy(), o_out) < OUT_TOL
    resid = torch.from_numpy(synth.make_hidden(layer.n_embd, T, seed=23)).cuda()
    fused = m.forward(xd, resid=resid)
    h = resid.clone()
    m.forward(xd, out=h, resid=h)
    torch.cuda.synchronize()
    assert torch.equal(fused, resid + plain) and torch.equal(h, fused)
    m.reserve(T)
    s = torch.cuda.Stream()
    out = torch.empty_like(xd)
    with torch.cuda.stream(s):
        m.forward(xd, out=out, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        m.forward(xd, out=out, stream=s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    m.status()
    assert torch.equal(out, plain)
    del g
    m.close()


def test_moe_deterministic_and_expert_permutation(cuda):
    """Size-independent properties at the 235B shape: repeated calls are bit-identical, and
    storing the experts in a different order (router rows permuted alike) changes only the
    reported ids, not one bit of the output."""
    import torch
    layer = synth.make_moe_layer("235b", seed=12)
    xn = torch.from_numpy(synth.make_hidden(layer.n_embd, 4, seed=13)).cuda()
    m = cuda.MoeLayer.from_synth(layer)
    a, sa, _, _ = m.route(xn)
    b, sb, _, _ = m.route(xn)
    assert torch.equal(a, b) and torch.equal(sa, sb)
    X = layer.n_expert
    perm = np.random.default_rng(1).permutation(X)      # slot i of the new layer holds expert perm[i]
    per = lambda t: np.ascontiguousarray(t.reshape(X, -1)[perm]).reshape(-1)
    pl = synth.MoeLayer(layer.n_embd, X, layer.n_used, layer.n_ff, np.ascontiguousarray(layer.router[perm]),
                        per(layer.gate), per(layer.up), per(layer.down))
    mp = cuda.MoeLayer.from_synth(pl)
    c, sc, _, _ = mp.route(xn)
    assert torch.equal(a, c)
    assert np.array_equal(perm[sc.cpu().numpy()], sa.cpu().numpy())
    m.close()
    mp.close()


def test_moe_device_source_matches_host_source(cuda):
    """Creating from device-resident GGUF bytes gives the same layer as from host bytes."""
    import torch
    layer = synth.make_moe_layer("30b", seed=14)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (layer.router, layer.gate, layer.up, layer.down)]
    md = cuda.MoeLayer(layer.n_embd, layer.n_expert, layer.n_used, layer.n_ff, *dev)
    mh = cuda.MoeLayer.from_synth(layer)
    xn = torch.from_numpy(synth.make_hidden(layer.n_embd, 3, seed=15)).cuda()
    assert torch.equal(md.forward(xn), mh.forward(xn))
    md.close()
    mh.close()


@pytest.mark.parametrize("skew,T", [(None, 4096), (1.1, 4096), (4.0, 1024)])
def test_moe_prefill_sizes_and_skewed_routing(cuda, oracle, skew, T):
    """The grouped tensor-core path at config 5's call size (T = 4096 tokens, 32768 slots) and under
    skewed routing: Zipf(1.1) expert popularity (config 5: thousands of slots and dozens of 64-slot
    tiles on the top experts) and a sharper Zipf(4) where a few experts take almost every slot and
    most get fewer than 8. Same bars as the other block tests."""
    layer = synth.make_moe_layer("235b", seed=61)
    if skew is None:
        xn = synth.make_hidden(layer.n_embd, T, seed=62)
    else:
        layer, xn = synth.zipf_layer_and_hidden(layer, T, s=skew, seed=63)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    counts = np.bincount(sel.reshape(-1), minlength=layer.n_expert)
    if skew is not None:
        assert counts.max() >= 512, counts.max()               # the skew this case exists for
    o_out, o_sel, o_w, o_logits = oracle.moe(layer, xn)
    assert np.array_equal(logits.view(np.uint32), o_logits.view(np.uint32)), "router logits differ"
    assert np.array_equal(sel, o_sel), "selected experts differ"
    assert _ulps(w, o_w) <= ULP_TOL
    err = rel_l2(out, o_out)
    assert err < OUT_TOL, f"rel L2 {err:.3e}"
    # per token, not only over the whole block: the worst token is within the bar as well
    tok = np.linalg.norm(out - o_out, axis=1) / np.maximum(np.linalg.norm(o_out, axis=1), 1e-30)
    assert tok.max() < 10 * OUT_TOL, f"worst token rel L2 {tok.max():.2e} (block {err:.2e})"
    m.close()


@pytest.mark.parametrize("shape", ["tiny", "235b"])
def test_batch1_without_the_persistent_kernel_matches_oracle(cuda, oracle, shape, monkeypatch):
    """The batch-1 kernel needs its whole grid resident (its CTAs wait for one another); where an
    SM cannot hold one of its CTAs the layer runs the per-slot kernels instead. QMS_PERSISTENT=0
    forces that choice at creation: same results."""
    monkeypatch.setenv("QMS_PERSISTENT", "0")
    layer = synth.make_moe_layer(shape, seed=81)
    xn = synth.make_hidden(layer.n_embd, 1, seed=82)
    m, out, sel, w, logits = _run(cuda, layer, xn)
    _check(oracle, layer, xn, out, sel, w, logits, f"{shape} fallback")
    m.close()
