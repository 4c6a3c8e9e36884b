"""A whole token step on a B200: the device build of `qms run` and qms_cuda_forward against the
reference CLI's own outputs on the same seeded GGUF models (tests/golden/make_model_golden.py).

Bars (north star): greedy ids identical over every generated step, the same expert ids in every
layer of every step (md5 of the --trace records, src/model.c:1102-1110), every step's top-10
logprobs within LP_TOL of the reference's, and prompt logits within 1e-3 relative L2.

Why these and not bit-identity: the device reproduces the reference's integer arithmetic (the same
Q8 activations, exact int8 block dots) but sums the fp32 block terms in another order, so a
re-quantised activation sitting on a rounding boundary can land one int8 step away. On config 1's
random-weight model (n_ff 256) one such flip moves a token's logits by ~1e-3; the reference's own
integer path is 3.4e-3 (mean per-row relative L2) away from its fp32 path on the same prompts, and
logprobs 5e-3 apart. Config 3 (n_ff 768, 48 layers) meets 1e-3; config 1's logits are held to
three quarters of the reference's own integer-vs-fp32 spread. Greedy ids are compared where the
reference's top-2 margin exceeds that noise (the golden seeds are chosen by that rule); the
near-tie seed is compared with teacher forcing, as the reference's tools/cmp_ref.py does.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, rel_l2
from large_model_b200 import synth

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((ROOT / "tests" / "golden" / "model_golden.json").read_text())
ARRAYS = np.load(ROOT / "tests" / "golden" / "model_golden.npz")
CLI = ROOT / "large_model_b200" / "bin" / "qms"
LP_TOL = 5e-3          # absolute, per top-10 logprob (the reference's own int8-vs-fp32 spread)
LOGIT_TOL = 1e-3       # relative L2 of prompt logits (north star)
NEAR_TIE = 5e-3        # a reference top-2 margin below this is a near tie (int8 re-quantisation noise)


def _logit_tol(g):
    """1e-3, or for config 1 three quarters of the reference's own integer-vs-fp32 distance."""
    return max(LOGIT_TOL, 0.75 * g.get("int_vs_fp32_rel_l2_mean", 0.0))


def _make_gguf(case: str, tmp: Path) -> Path:
    import make_model_golden as mg
    cfg_name, seed = mg.CASES[case][:2]
    path = tmp / f"{case}.gguf"
    synth.write_gguf(path, synth.MODEL_CONFIGS[cfg_name], seed)
    assert mg.sha256_file(path) == GOLDEN[case]["gguf_sha256"], "the synthetic model generator drifted"
    return path


def _check_steps(steps, ref_steps):
    assert len(steps) == len(ref_steps)
    worst = 0.0
    for s, (a, b) in enumerate(zip(steps, ref_steps)):
        da, db = dict(a), dict((int(i), lp) for i, lp in b)
        assert a[0][0] == int(b[0][0]), f"step {s}: top-1 {a[0][0]} vs reference {b[0][0]}"
        common = set(da) & set(db)
        assert len(common) >= 8, f"step {s}: top-10 sets differ: {sorted(da)} vs {sorted(db)}"
        worst = max(worst, max(abs(da[i] - db[i]) for i in common))
    assert worst < LP_TOL, f"top-10 logprobs differ by {worst:.2e}"
    return worst


@pytest.mark.parametrize("case", ["tiny", "tiny-tied"])
def test_device_cli_matches_reference_cli(cuda, tmp_path, case):
    """`qms run` with qms_forward on the device: same ids, experts, top-10 and prompt logits."""
    import make_model_golden as mg
    if not CLI.exists():
        pytest.fail(f"{CLI} is missing: large_model_b200.build compiles it where the reference tree exists")
    g = GOLDEN[case]
    gguf = _make_gguf(case, tmp_path)
    out, logits = mg.run_cli(CLI, gguf, mg.prompt_of(case), g["gen"], g["ctx"], tmp_path)
    assert out["ids"] == g["ids"], "greedy ids differ from the reference CLI"
    assert out["trace_md5"] == g["trace_md5"], "selected experts (--trace records) differ"
    _check_steps(out["steps"], g["steps"])
    rows = ARRAYS[f"{case}_rows"]
    err = rel_l2(logits[rows], ARRAYS[f"{case}_logits"])
    assert err < _logit_tol(g), f"prompt logits rel L2 {err:.2e}"
    assert "device:" in out["stderr"] and "uploaded" in out["stderr"]


def test_near_tie_seed_teacher_forced(cuda):
    """Config 1 with seed 1, whose reference trajectory has a 1.6e-3 top-2 margin: the device runs
    the reference's own ids (teacher forcing, tools/cmp_ref.py's method) and must pick the same
    argmax at every step whose margin is not a near tie, with logprobs within LP_TOL."""
    import make_model_golden as mg
    g = GOLDEN["tiny-s1"]
    m = cuda.Model.from_synth(synth.MODEL_CONFIGS["tiny"], g["seed"], g["ctx"])
    ids, n = g["ids"], g["n_prompt"]
    assert ids[:n] == mg.prompt_of("tiny-s1")
    logits = m.forward(ids[:n], 0)
    ties = 0
    worst = 0.0
    for s, ref in enumerate(g["steps"]):
        lp = _log_softmax(logits)
        margin = ref[0][1] - ref[1][1]
        if margin >= NEAR_TIE:
            assert int(np.argmax(logits)) == ref[0][0], f"step {s}: argmax differs at margin {margin:.2e}"
        else:
            ties += 1
            assert int(np.argmax(logits)) in (ref[0][0], ref[1][0])
        worst = max(worst, max(abs(lp[int(i)] - v) for i, v in ref))
        if s + 1 < len(g["steps"]):
            logits = m.forward([ids[n + s]], n + s)
    m.status()
    assert worst < LP_TOL, f"logprobs differ by {worst:.2e}"
    assert ties >= 1                                      # the case this seed exists for
    m.close()


def _log_softmax(x):
    x = np.asarray(x, np.float64)
    m = x.max()
    return x - m - np.log(np.exp(x - m).sum())


def _greedy_run(model, prompt, gen):
    """main.c's inc-mode loop (src/main.c:181-207) through qms_cuda_forward: returns ids, top-10
    steps and every layer's selected experts per call."""
    logits, sel = model.forward(prompt, 0, trace=True)
    traces = [sel]
    ids = list(prompt)
    steps = []
    for s in range(gen):
        lp = _log_softmax(logits)
        top = np.argsort(-lp, kind="stable")[:10]
        steps.append([(int(i), float(lp[i])) for i in top])
        nxt = int(np.argmax(logits))
        ids.append(nxt)
        if s + 1 < gen:
            logits, sel = model.forward([nxt], len(ids) - 1, trace=True)
            traces.append(sel)
    return ids, steps, traces


def _trace_md5(traces, n_expert):
    """The reference's --trace bytes: per call and layer, {step, layer, expert} for every distinct
    expert in ascending order (src/model.c:1102-1110)."""
    h = hashlib.md5()
    for step, sel in enumerate(traces, start=1):
        for l in range(sel.shape[0]):
            for e in np.unique(sel[l]):
                h.update(np.array([step], "<i4").tobytes() + np.array([l, e], "<i2").tobytes())
    return h.hexdigest()


def test_30b_forward_matches_reference(cuda):
    """Config 3 (Qwen3-30B-A3B, 48 layers, Q6_K head): a 512-id prompt (two 256-token passes) and
    128 greedy steps through qms_cuda_forward, against the reference CLI on the same GGUF bytes."""
    import make_model_golden as mg
    g = GOLDEN["30b"]
    cfg = synth.MODEL_CONFIGS["30b"]
    m = cuda.Model.from_synth(cfg, g["seed"], g["ctx"])
    prompt = mg.prompt_of("30b")
    logits_all = m.forward(prompt, 0, all_logits=True)
    rows = ARRAYS["30b_rows"]
    idx, val = ARRAYS["30b_top_idx"], ARRAYS["30b_top_val"]
    for k, r in enumerate(rows):
        err = rel_l2(logits_all[r][idx[k]], val[k])
        assert err < LOGIT_TOL, f"prompt row {r}: top-256 logits rel L2 {err:.2e}"
    m.close()
    m = cuda.Model.from_synth(cfg, g["seed"], g["ctx"])
    ids, steps, traces = _greedy_run(m, prompt, g["gen"])
    m.status()
    assert ids == g["ids"], "greedy ids differ from the reference CLI"
    assert _trace_md5(traces, cfg.n_expert) == g["trace_md5"], "selected experts differ"
    _check_steps(steps, g["steps"])
    m.close()


def test_decode_step_graph_replays_greedy_decode(cuda):
    """qms_cuda_decode_step captured once in a CUDA graph and replayed: the argmax, the position
    and the next embedding stay on the device, and the tokens equal the reference's greedy ids."""
    import torch
    import make_model_golden as mg
    g = GOLDEN["tiny"]
    m = cuda.Model.from_synth(synth.MODEL_CONFIGS["tiny"], g["seed"], g["ctx"])
    prompt = mg.prompt_of("tiny")
    logits = m.forward(prompt, 0)
    tok = torch.tensor([int(np.argmax(logits))], dtype=torch.int32, device="cuda")
    pos = torch.tensor([len(prompt)], dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    out = [int(tok.item())]
    with torch.cuda.stream(s):
        m.decode_step(tok, pos, stream=s)            # warm-up step outside capture
        s.synchronize()
        out.append(int(tok.item()))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            m.decode_step(tok, pos, stream=s)
        for _ in range(g["gen"] - 2):
            graph.replay()
            s.synchronize()
            out.append(int(tok.item()))
    m.status()
    assert int(pos.item()) == len(prompt) + g["gen"] - 1
    assert prompt + out == g["ids"]
    del graph
    m.close()


def test_forward_refuses_bad_calls(cuda):
    g = GOLDEN["tiny"]
    m = cuda.Model.from_synth(synth.MODEL_CONFIGS["tiny"], g["seed"], 64)
    with pytest.raises(cuda.QmsCudaError) as e:
        m.forward([1, 2, 3], 62)                     # pos0 + T > ctx (src/model.c:1257)
    assert e.value.code == cuda.EINVAL and "context" in str(e.value)
    with pytest.raises(cuda.QmsCudaError) as e:
        m.forward([5, 4096], 0)                      # id outside the vocabulary (src/model.c:1264)
    assert e.value.code == cuda.EINVAL and "bad id" in str(e.value)
    m.forward([5, 6], 0)                             # still usable
    m.status()
    m.close()


def test_forward_before_layers_are_set_fails(cuda):
    cfg = synth.MODEL_CONFIGS["tiny"]
    names = synth.model_tensors(cfg)
    trunk = {names[i][0]: synth.tensor_data(cfg, 1, i) for i in range(3)}
    m = cuda.Model(cfg, trunk, 32)
    with pytest.raises(cuda.QmsCudaError) as e:
        m.forward([1], 0)
    assert "never set" in str(e.value)
    m.close()


def _teacher_forced(m_batch, m_single, prompts, steps):
    """Sequence b of m_batch and a single-sequence run on m_single see the same tokens (the single
    run's greedy ids); returns the relative L2 of every pair of logits rows and the number of steps
    whose argmax differs where the single run's top-2 margin is not a near tie."""
    B = len(prompts)
    singles = []
    for p in prompts:                                 # greedy single-sequence runs, host path
        lg = m_single.forward(p, 0)
        ids, rows = [int(np.argmax(lg))], [lg]
        for s in range(steps):
            lg = m_single.forward([ids[-1]], len(p) + s)
            rows.append(lg)
            ids.append(int(np.argmax(lg)))
        singles.append((ids, rows))
    errs, flips = [], 0
    for b, p in enumerate(prompts):
        lg = m_batch.forward(p, 0, seq=b)
        errs.append(rel_l2(lg, singles[b][1][0]))
    for s in range(steps):
        ids = [singles[b][0][s] for b in range(B)]
        pos = [len(prompts[b]) + s for b in range(B)]
        rows = m_batch.forward_batch(ids, pos)
        for b in range(B):
            ref = singles[b][1][s + 1]
            errs.append(rel_l2(rows[b], ref))
            top = np.sort(_log_softmax(ref))[-2:]
            if top[1] - top[0] >= NEAR_TIE and int(np.argmax(rows[b])) != int(np.argmax(ref)):
                flips += 1
    return np.array(errs), flips


def test_forward_batch_matches_single_sequences(cuda):
    """qms_cuda_forward_batch: B sequences at different positions in one pass give, row by row, the
    logits of qms_cuda_forward_seq on each sequence alone (teacher forcing, config 1 and config 3).
    The two paths sum fp32 terms in different orders (multi-token vs one-token kernels), so on
    config 1 a re-quantised activation can land one int8 step away (module docstring): there the mean
    row is held to three quarters, the worst row to all, of the reference's own int-vs-fp32 spread;
    config 3 to 1e-3. The argmax must agree wherever the margin is not a near tie."""
    rng = np.random.default_rng(5)
    for name, B, steps in (("tiny", 5, 12), ("30b", 3, 6)):
        cfg = synth.MODEL_CONFIGS[name]
        prompts = [[int(v) for v in rng.integers(0, cfg.vocab, n)] for n in (7, 19, 3, 40, 11)[:B]]
        mb = cuda.Model.from_synth(cfg, 1, 128)
        mb.set_sequences(B)
        ms = cuda.Model.from_synth(cfg, 1, 128)
        errs, flips = _teacher_forced(mb, ms, prompts, steps)
        mb.status()
        ms.status()
        mb.close()
        ms.close()
        spread = GOLDEN["tiny"]["int_vs_fp32_rel_l2_mean"] if name == "tiny" else LOGIT_TOL
        mean_bar, max_bar = (0.75 * spread, spread) if name == "tiny" else (LOGIT_TOL, LOGIT_TOL)
        assert errs.mean() < mean_bar, f"{name}: batch rows differ from single-sequence logits by {errs.mean():.2e} (mean)"
        assert errs.max() < max_bar, f"{name}: batch rows differ from single-sequence logits by {errs.max():.2e} (worst)"
        assert flips == 0, f"{name}: {flips} argmax differences outside near ties"


def test_decode_batch_graph_matches_reference_ids(cuda):
    """qms_cuda_decode_batch in a CUDA graph: sequences 0 and 2 hold the golden prompt (sequence 2
    through qms_cuda_model_copy_sequence), sequence 1 another prompt; 0 and 2 must produce the
    reference CLI's greedy ids, and sequence 1 must not disturb them."""
    import torch
    import make_model_golden as mg
    g = GOLDEN["tiny"]
    m = cuda.Model.from_synth(synth.MODEL_CONFIGS["tiny"], g["seed"], g["ctx"])
    m.set_sequences(3)
    prompt = mg.prompt_of("tiny")
    other = [int(v) for v in np.random.default_rng(9).integers(0, 4096, 23)]
    l0 = m.forward(prompt, 0, seq=0)
    l1 = m.forward(other, 0, seq=1)
    m.copy_sequence(0, 2, len(prompt))
    first = int(np.argmax(l0))
    tok = torch.tensor([first, int(np.argmax(l1)), first], dtype=torch.int32, device="cuda")
    pos = torch.tensor([len(prompt), len(other), len(prompt)], dtype=torch.int32, device="cuda")
    out = [[first], [], [first]]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.decode_batch(tok, pos, stream=s)            # warm-up step outside capture
        s.synchronize()
        t = tok.tolist()
        out[0].append(t[0])
        out[2].append(t[2])
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            m.decode_batch(tok, pos, stream=s)
        for _ in range(g["gen"] - 2):
            graph.replay()
            s.synchronize()
            t = tok.tolist()
            out[0].append(t[0])
            out[2].append(t[2])
    m.status()
    assert prompt + out[0] == g["ids"], "sequence 0 differs from the reference's greedy ids"
    assert out[2] == out[0], "the copied sequence differs"
    assert pos.tolist() == [len(prompt) + g["gen"] - 1, len(other) + g["gen"] - 1, len(prompt) + g["gen"] - 1]
    del graph
    m.close()


def test_fp16_kv_cache_close_to_fp32(cuda):
    """KV compaction (qms_cuda_model_set_kv_type F16): the prompt and 8 teacher-forced decode steps
    with an fp16 cache against the fp32 cache (the reference's). Each K / V value is rounded once
    to fp16, so the logits move by about that rounding through the softmax; the argmax must agree
    wherever the fp32 run's top-2 margin is above 0.05 (logprob). A batched step over fp16 caches
    must match single sequences on fp16 caches as the fp32 batch test does."""
    rng = np.random.default_rng(17)
    for name in ("tiny", "30b"):
        cfg = synth.MODEL_CONFIGS[name]
        prompt = [int(v) for v in rng.integers(0, cfg.vocab, 40)]
        m32 = cuda.Model.from_synth(cfg, 3, 96)
        m16 = cuda.Model.from_synth(cfg, 3, 96)
        m16.set_kv_type(cuda.T_F16)
        l32, l16 = m32.forward(prompt, 0, all_logits=True), m16.forward(prompt, 0, all_logits=True)
        errs = [rel_l2(l16[t], l32[t]) for t in range(len(prompt))]
        flips = 0
        tok = int(np.argmax(l32[-1]))
        for s in range(8):
            a32, a16 = m32.forward([tok], len(prompt) + s), m16.forward([tok], len(prompt) + s)
            errs.append(rel_l2(a16, a32))
            top = np.sort(_log_softmax(a32))[-2:]
            if top[1] - top[0] > 0.05 and int(np.argmax(a16)) != int(np.argmax(a32)):
                flips += 1
            tok = int(np.argmax(a32))
        m32.status()
        m16.status()
        m32.close()
        errs = np.array(errs)
        assert errs.mean() < 1e-2 and errs.max() < 5e-2, f"{name}: fp16 cache moves logits by {errs.mean():.2e} (mean), {errs.max():.2e} (worst)"
        assert flips == 0, f"{name}: {flips} argmax changes outside near ties"
        # batched decode over fp16 caches against single sequences on fp16 caches
        m16.set_sequences(2)
        ms = cuda.Model.from_synth(cfg, 3, 96)
        ms.set_kv_type(cuda.T_F16)
        berrs, bflips = _teacher_forced(m16, ms, [prompt[:13], prompt[13:]], 4)
        m16.close()
        ms.close()
        assert berrs.mean() < 3e-3 and bflips == 0, f"{name}: fp16 batch rows differ by {berrs.mean():.2e}"


def test_batch_calls_edge_cases(cuda):
    """Batch of one through the batched path; a sequence stepping past its context raises the
    device flag (EINVAL) while the others' rows stay valid; the model stays usable; host checks."""
    import torch
    cfg = synth.MODEL_CONFIGS["tiny"]
    ctx = 24
    m = cuda.Model.from_synth(cfg, 5, ctx)
    m.set_sequences(3)
    single = cuda.Model.from_synth(cfg, 5, ctx)
    p0, p1 = [7, 8, 9, 10], [11] * (ctx - 1)
    m.forward(p0, 0, seq=0)
    m.forward(p1, 0, seq=1)
    lb = m.forward_batch([3], [len(p0)])                       # B = 1
    single.forward(p0, 0)
    ls = single.forward([3], len(p0))
    assert rel_l2(lb[0], ls) < 1e-2                           # the multi-token vs one-token kernels (config 1 noise)
    # sequence 1 is at its last position: one step fits, the next one is refused
    tok = torch.tensor([4, 5], dtype=torch.int32, device="cuda")
    pos = torch.tensor([len(p0) + 1, ctx - 1], dtype=torch.int32, device="cuda")
    m.decode_batch(tok, pos)
    m.status()
    with pytest.raises(cuda.QmsCudaError) as e:               # host entry: checked before launch
        m.forward_batch([1, 2], [len(p0) + 2, ctx])
    assert e.value.code == cuda.EINVAL and "context" in str(e.value)
    m.decode_batch(tok, pos)                                  # device entry: pos[1] == ctx
    with pytest.raises(cuda.QmsCudaError) as e:
        m.status()
    assert e.value.code == cuda.EINVAL and "position" in str(e.value)
    rows = m.forward_batch([1], [len(p0) + 3])                # still usable after the flag
    assert np.isfinite(rows).all()
    m.status()
    for bad in (lambda: m.forward([1], 0, seq=3), lambda: m.copy_sequence(0, 0, 4),
                lambda: m.copy_sequence(0, 1, ctx + 1), lambda: m.forward_batch([1] * 4, [0] * 4),
                lambda: m.set_kv_type(cuda.T_Q4_0)):
        with pytest.raises(cuda.QmsCudaError):
            bad()
    m.close()
    single.close()
