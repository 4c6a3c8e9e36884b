"""The oracle (C restatement) pinned against the reference: golden vectors produced by the
reference's own build (tests/golden/reference_golden.npz), its known-answer tests, and a live
comparison with oracle/_ref when that build is present. CPU only."""
from __future__ import annotations

import numpy as np
import pytest

import cases
from conftest import rel_l2


def test_f16_known_answers(oracle):
    # tests/test_smoke.c:36-39 of the reference
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0xC000) == -2.0
    assert oracle.f16_to_f32(0x7BFF) == 65504.0
    assert oracle.f16_to_f32(0x0001) == np.float32(5.9604644775390625e-08)


def test_f16_all_halves_match_numpy(oracle):
    h = np.arange(0, 1 << 16, 257, dtype=np.uint16)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h], np.float32)
    want = h.view(np.float16).astype(np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))


def test_quantize_golden(oracle, golden):
    for name, x in cases.quant_cases().items():
        assert str(golden[f"quant/{name}/sha"]) == cases.sha(x), "input generation drifted"
        got = oracle.quantize_q8(x).view(np.uint8)
        assert np.array_equal(got, golden[f"quant/{name}/q8"]), name


def test_dot_golden_bit_exact(oracle, golden):
    for name, (typ, n, w, x) in cases.dot_cases().items():
        assert str(golden[f"dot/{name}/sha"]) == cases.sha(w, x), "input generation drifted"
        xq = oracle.quantize_q8(x).reshape(len(w), -1)
        got = np.array([oracle.vec_dot_q8(typ, w[i], xq[i], n) for i in range(len(w))], np.float32)
        assert np.array_equal(got.view(np.uint32), golden[f"dot/{name}/got"].view(np.uint32)), name


def test_f32_dot_golden_bit_exact(oracle, golden):
    for name, (w, x) in cases.f32_cases().items():
        assert str(golden[f"f32/{name}/sha"]) == cases.sha(w, x)
        got = np.array([oracle.vec_dot_f32(w[i], x) for i in range(len(w))], np.float32)
        assert np.array_equal(got.view(np.uint32), golden[f"f32/{name}/got"].view(np.uint32)), name


def test_dequant_golden_bit_exact(oracle, golden):
    for name, (typ, n, blob) in cases.deq_cases().items():
        assert str(golden[f"deq/{name}/sha"]) == cases.sha(blob)
        got = oracle.dequant_row(typ, blob, n)
        assert np.array_equal(got.view(np.uint32), golden[f"deq/{name}/got"].view(np.uint32)), name


def test_kernel_criterion(oracle):
    """The reference's kernel test (tests/test_kernels.c:65-84): the integer dot against a double
    dot of dequantised weights and dequantised int8 activations, |got-ref|/sum|terms| < 1e-5."""
    worst = 0.0
    for name, (typ, n, w, x) in cases.dot_cases().items():
        xq = oracle.quantize_q8(x).reshape(len(w), -1)
        for i in range(len(w)):
            wd = oracle.dequant_row(typ, w[i], n).astype(np.float64)
            xi = (xq[i]["q"].astype(np.float64) * xq[i]["d"][:, None]).reshape(-1)
            ref = float(np.dot(wd, xi))
            mag = float(np.abs(wd * xi).sum())
            got = oracle.vec_dot_q8(typ, w[i], xq[i], n)
            worst = max(worst, abs(got - ref) / (mag + 1e-30))
    assert worst < 1e-5, worst


def test_moe_golden_bit_exact(oracle, golden):
    for name, (layer, xn) in cases.moe_cases().items():
        assert str(golden[f"moe/{name}/sha"]) == cases.sha(layer.router, layer.gate, layer.up, layer.down, xn)
        out, sel, w, logits = oracle.moe(layer, xn)
        assert np.array_equal(out.view(np.uint32), golden[f"moe/{name}/out"].view(np.uint32)), name
        # the reference's --trace lists the distinct experts of the call in ascending order
        assert sorted(set(sel.ravel().tolist())) == golden[f"moe/{name}/trace"].tolist(), name


def test_route_semantics(oracle):
    """Top-k ties go to the lower expert index; weights are renormalised over the top k."""
    X, E, K = 16, 256, 4
    router = np.zeros((X, E), np.float32)
    router[[3, 5, 9, 12, 14], 0] = 1.0           # five tied winners
    xn = np.zeros((1, E), np.float32)
    xn[0, 0] = 2.0
    logits, sel, w = oracle.route(router, K, xn)
    assert sel.tolist() == [[3, 5, 9, 12]]
    assert np.allclose(w, 0.25) and abs(float(w.sum()) - 1.0) < 1e-6
    _, sel0, w0 = oracle.route(router, K, np.zeros((1, E), np.float32))
    assert sel0.tolist() == [[0, 1, 2, 3]]       # all equal: lowest indices first
    assert np.all(w0 == np.float32(0.25))


def test_oracle_matches_reference_live(oracle, reference):
    """Bit-exact agreement with the reference build on fresh seeds (incl. the 235B shape)."""
    from large_model_b200 import synth
    for shape, T, seed in (("tiny", 6, 21), ("30b", 2, 22), ("235b", 1, 23)):
        layer = synth.make_moe_layer(shape, seed=seed)
        xn = synth.make_hidden(layer.n_embd, T, seed=seed + 100)
        out, sel, w, _ = oracle.moe(layer, xn)
        ref_out, trace = reference.moe(layer, xn, trace=True)
        assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32)), (shape, rel_l2(out, ref_out))
        assert sorted(set(sel.ravel().tolist())) == trace.tolist()
    x = np.random.default_rng(5).standard_normal(4096).astype(np.float32)
    assert oracle.quantize_q8(x).tobytes() == reference.quantize_q8(x).tobytes()


def test_oracle_matches_reference_q4_1_down(oracle, reference):
    """Q4_1 ffn_down_exps (src/kernels.c:109-121 dot, d*q + m blocks) bit-exact against the reference."""
    from large_model_b200 import synth
    for shape, T, seed in (("tiny", 5, 61), ("30b", 1, 62)):
        layer = synth.make_moe_layer(shape, seed=seed, down_type=synth.T_Q4_1)
        xn = synth.make_hidden(layer.n_embd, T, seed=seed + 100)
        out, sel, _, _ = oracle.moe(layer, xn)
        ref_out, trace = reference.moe(layer, xn, trace=True)
        assert np.array_equal(out.view(np.uint32), ref_out.view(np.uint32)), (shape, rel_l2(out, ref_out))
        assert sorted(set(sel.ravel().tolist())) == trace.tolist()


def test_moe_rejects_non_fast_shapes(oracle):
    from large_model_b200 import synth
    layer = synth.make_moe_layer((288, 4, 2, 64), seed=1)   # 288 % 256 != 0: reference uses exact math
    with pytest.raises(ValueError):
        oracle.moe(layer, synth.make_hidden(288, 1))


def _sampler_golden():
    from conftest import ROOT
    return np.load(ROOT / "tests" / "golden" / "sampler_golden.npz")


def test_sampler_golden(oracle):
    """The restated chat sampler (src/chat.c:36-69) against the reference's own draws: same
    token and same generator state after each of two draws in a row."""
    g = _sampler_golden()
    for name, (l, temp, top_p, top_k, seed) in cases.sampler_cases().items():
        assert str(g[f"{name}/sha"]) == cases.sha(l), f"{name}: input generation drifted"
        st = seed
        for k in range(2):
            t, st = oracle.sample(l, temp, top_p, top_k, st)
            assert t == int(g[f"{name}/tokens"][k]), f"{name} draw {k}"
            assert st == int(g[f"{name}/states"][k]), f"{name} draw {k}: generator state"


def test_sampler_random_vs_reference(oracle):
    """More seeded draws straight against the reference build, where it is present."""
    from oracle import RefSampler
    try:
        ref = RefSampler()
    except FileNotFoundError:
        pytest.skip("oracle/_ref/libqms_ref_sample.so is not present")
    rng = np.random.default_rng(7)
    for i in range(200):
        V = int(rng.choice([3, 64, 3000, 151936]))
        l = (rng.standard_normal(V) * rng.choice([0.3, 3.0])).astype(np.float32)
        if i % 5 == 0:
            l = np.round(l * 2).astype(np.float32)
        args = (float(rng.choice([0.0, 0.5, 1.0, 2.0])), float(rng.choice([0.3, 0.9, 1.0])),
                int(rng.choice([0, 2, 50, 1024, 3000])), int(rng.integers(0, 2**63)))
        assert oracle.sample(l, *args) == ref.sample(l, *args), f"case {i}"
