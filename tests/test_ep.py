"""Expert parallelism (large_model_b200/ep.py): the dispatch / return / combine logic.

CPU: two and four gloo ranks, the compute steps from the oracle (the reference's integer path
restated in C: route, per-slot gate/up/SwiGLU/down, weighted sum); the sharded result (rows sent
as Q8 blocks) must equal the same backend run unsharded on one process from fp32 rows, bit for bit. GPU (two B200s, NCCL): shard layers through the
C ABI against the unsharded layer's grouped path.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from large_model_b200 import synth
from large_model_b200.ep import ExpertParallelMoe


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def pack_index(sel, n_expert: int, n_rank: int, cap: int):
    """qms_cuda_ep_pack's slot map restated on the host: slot t*K + j goes to entry o * cap + (its
    index among the slots owned by rank o, in slot order), o = expert // (n_expert / n_rank); ids
    holds each used entry's local expert id and -1 elsewhere; slots past `cap` are dropped (-1).
    Returns (slot [T][K], ids [n_rank * cap], dropped)."""
    T, K = sel.shape
    per = n_expert // n_rank
    slot = torch.full((T * K,), -1, dtype=torch.int32)
    ids = torch.full((n_rank * cap,), -1, dtype=torch.int32)
    fill = [0] * n_rank
    for i, e in enumerate(sel.reshape(-1).tolist()):
        o = e // per
        if fill[o] < cap:
            slot[i] = o * cap + fill[o]
            ids[o * cap + fill[o]] = e - o * per
        fill[o] += 1
    return slot.reshape(T, K), ids, max(fill) > cap


class OracleBackend:
    """The oracle's per-slot computation for experts [base, base + n_local) of a synth layer."""

    def __init__(self, layer, base: int, n_local: int):
        import oracle
        self.o = oracle.Oracle()
        self.layer, self.base, self.n_local = layer, base, n_local
        E, F = layer.n_embd, layer.n_ff
        self.gu_bytes = F * (E // 32) * 18
        self.dn_bytes = E * (F // 32) * (20 if layer.down_type == synth.T_Q4_1 else 18)

    def route(self, xn):
        if xn.shape[0] == 0:
            K = self.layer.n_used
            return torch.empty((0, K), dtype=torch.int32), torch.empty((0, K), dtype=torch.float32)
        _, sel, w = self.o.route(self.layer.router, self.layer.n_used, xn.numpy())
        return torch.from_numpy(sel), torch.from_numpy(w)

    def experts(self, x, local_expert):
        L, E, F = self.layer, self.layer.n_embd, self.layer.n_ff
        dn = np.empty((x.shape[0], E), np.float32)
        for i, (row, le) in enumerate(zip(x.numpy(), local_expert.tolist())):
            assert 0 <= le < self.n_local
            e = self.base + le
            gw = L.gate[e * self.gu_bytes:(e + 1) * self.gu_bytes]
            uw = L.up[e * self.gu_bytes:(e + 1) * self.gu_bytes]
            dw = L.down[e * self.dn_bytes:(e + 1) * self.dn_bytes]
            g = self.o.matmul(L.gate_type, F, E, gw, row)[0]
            u = self.o.matmul(L.up_type, F, E, uw, row)[0]
            dn[i] = self.o.matmul(L.down_type, E, F, dw, self.o.swiglu(g, u))[0]
        return torch.from_numpy(dn)

    def quantize(self, xn):
        rows = [self.o.quantize_q8(r).view(np.uint8) for r in xn.numpy()]
        return torch.from_numpy(np.stack(rows)) if rows else torch.empty((0, xn.shape[1] // 32 * 44), dtype=torch.uint8)

    def experts_q8(self, xq, local_expert):
        L, E, F = self.layer, self.layer.n_embd, self.layer.n_ff
        dn = np.zeros((xq.shape[0], E), np.float32)
        for i, (row, le) in enumerate(zip(xq.numpy(), local_expert.tolist())):
            if le == -1:                                        # an unused entry of a segment
                continue
            assert 0 <= le < self.n_local
            e = self.base + le
            gw = L.gate[e * self.gu_bytes:(e + 1) * self.gu_bytes]
            uw = L.up[e * self.gu_bytes:(e + 1) * self.gu_bytes]
            dw = L.down[e * self.dn_bytes:(e + 1) * self.dn_bytes]
            g = self.o.matmul_q8(L.gate_type, F, E, gw, row)[0]
            u = self.o.matmul_q8(L.up_type, F, E, uw, row)[0]
            dn[i] = self.o.matmul(L.down_type, E, F, dw, self.o.swiglu(g, u))[0]
        return torch.from_numpy(dn)

    def new_flag(self, device):
        return torch.zeros((1,), dtype=torch.int32)

    def pack(self, xn, sel, n_expert, n_rank, cap, err):
        T, K = sel.shape
        slot, send_e, dropped = pack_index(sel, n_expert, n_rank, cap)
        xq = self.quantize(xn)
        send_x = torch.zeros((n_rank * cap, xn.shape[1] // 32 * 44), dtype=torch.uint8)
        s = slot.reshape(-1).long()
        used = s >= 0
        send_x[s[used]] = xq[torch.arange(T * K)[used] // K]
        if dropped:
            err[0] |= 1
        return send_x, send_e, slot

    def combine_slots(self, ret, slot, wts, resid):
        s = slot.reshape(-1).long()
        dn = ret[s.clamp(min=0)]
        dn[s < 0] = float("nan")
        return self.combine(dn, wts, resid)

    def combine(self, dn, wts, resid):
        T, K = wts.shape
        d = dn.reshape(T, K, dn.shape[-1])
        out = torch.zeros((T, d.shape[-1]), dtype=torch.float32)
        for j in range(K):                                      # selection order
            out = out + wts[:, j:j + 1] * d[:, j]
        return out if resid is None else resid + out


def unsharded(backend, xn, resid=None):
    sel, wts = backend.route(xn)
    T, K = sel.shape
    dn = backend.experts(xn.repeat_interleave(K, dim=0), sel.reshape(-1).to(torch.int32))
    return backend.combine(dn, wts, resid)


def _cpu_rank(rank, world, port, shape, T, q, cap=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = synth.make_moe_layer(shape, seed=41)
        per = layer.n_expert // world
        ep = ExpertParallelMoe(OracleBackend(layer, rank * per, per), layer.n_expert, layer.n_used, layer.n_embd,
                               max_tokens=T + world, cap=cap)
        # ragged T per rank; rank 1 also makes a call with no tokens (it still takes part)
        xn = torch.from_numpy(synth.make_hidden(layer.n_embd, T + rank, seed=50 + rank))
        resid = torch.from_numpy(synth.make_hidden(layer.n_embd, T + rank, seed=60 + rank))
        out = ep.forward(xn, resid)
        empty = ep.forward(xn[:0] if rank == 1 else xn, None if rank == 1 else resid)
        ref = unsharded(OracleBackend(layer, 0, layer.n_expert), xn, resid)
        if cap is None:
            ok = torch.equal(out, ref) and (rank == 1 and empty.shape[0] == 0 or torch.equal(empty, ref))
            q.put((rank, bool(ok) and not ep.overflowed(), float((out - ref).abs().max())))
        else:                                  # dropped slots: flagged, their tokens NaN, the rest exact
            bad = torch.isnan(out).any(dim=1)
            ok = ep.overflowed() == bool(bad.any()) and torch.equal(out[~bad], ref[~bad])
            q.put((rank, bool(ok), int(bad.sum())))
    finally:
        dist.destroy_process_group()


def _run_cpu_ranks(world, T, cap=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank, args=(r, world, port, "tiny", T, q, cap)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_ep_dispatch_combine_gloo(world):
    for rank, equal, diff in _run_cpu_ranks(world, 5):
        assert equal, f"rank {rank}: EP differs from the unsharded layer by {diff}"


def test_ep_small_capacity_flags_dropped_slots_gloo():
    """cap = 3 entries per destination for 6-7 tokens of 4 slots: slots are dropped; the flag is
    raised exactly on the ranks whose slots were dropped, only their tokens are NaN."""
    res = _run_cpu_ranks(2, 6, cap=3)
    for rank, ok, n_bad in res:
        assert ok, f"rank {rank}: flag or the surviving tokens wrong ({n_bad} NaN tokens)"
    assert sum(n for _, _, n in res) > 0


def _gpu_rank(rank, world, port, shape, T, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import large_model_b200 as lmb
        from large_model_b200.ep import CudaBackend
        lmb.init(rank)
        layer = synth.make_moe_layer(shape, seed=42)
        per = layer.n_expert // world
        shard = lmb.MoeLayer.shard_from_synth(layer, rank * per, per)
        ep = ExpertParallelMoe(CudaBackend(shard), layer.n_expert, layer.n_used, layer.n_embd, max_tokens=T + 3)
        xn = torch.from_numpy(synth.make_hidden(layer.n_embd, T + 3 * rank, seed=70 + rank)).cuda()
        resid = torch.from_numpy(synth.make_hidden(layer.n_embd, T + 3 * rank, seed=80 + rank)).cuda()
        out = ep.forward(xn, resid)
        full = lmb.MoeLayer.from_synth(layer)
        ref = full.forward(xn, resid=resid)
        torch.cuda.synchronize()
        shard.status()
        full.status()
        q.put((rank, bool(torch.equal(out, ref)) and not ep.overflowed(), float((out - ref).abs().max())))
        shard.close()
        full.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_two_gpus_matches_unsharded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank, args=(r, 2, port, "30b", 40, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for rank, equal, diff in res:
        assert equal, f"rank {rank}: EP differs from the unsharded layer by {diff}"


@pytest.mark.gpu
@pytest.mark.parametrize("shape,T,parts", [("tiny", 20, 2), ("30b", 48, 4), ("235b", 64, 8)])
def test_shards_on_one_gpu_match_unsharded(shape, T, parts):
    """The EP building blocks on one GPU: `parts` shard layers, routing on shard 0, each slot's rows
    through its owner shard, combine - bitwise equal to the unsharded layer's grouped path."""
    import large_model_b200 as lmb
    lmb.init(0)
    layer = synth.make_moe_layer(shape, seed=43)
    per = layer.n_expert // parts
    shards = [lmb.MoeLayer.shard_from_synth(layer, p * per, per) for p in range(parts)]
    xn = torch.from_numpy(synth.make_hidden(layer.n_embd, T, seed=44)).cuda()
    sel, wts = shards[0].route_only(xn)
    K, E = layer.n_used, layer.n_embd
    flat = sel.reshape(-1).long()
    dn = torch.empty((T * K, E), dtype=torch.float32, device="cuda")
    rows = xn.repeat_interleave(K, dim=0)
    xq = lmb.quantize_q8(rows)
    for p, sh in enumerate(shards):
        idx = torch.nonzero(flat // per == p).flatten()
        if idx.numel():
            ids = (flat[idx] % per).to(torch.int32).contiguous()
            dn[idx] = sh.experts(rows[idx].contiguous(), ids)
            # the same rows sent as QmsQ8 blocks (the expert-parallel dispatch format)
            assert torch.equal(sh.experts_q8(xq[idx].contiguous(), ids), dn[idx])
    out = lmb.combine(dn, wts)
    full = lmb.MoeLayer.from_synth(layer)
    ref, ref_sel, _, _ = full.route(xn)
    torch.cuda.synchronize()
    for sh in shards:
        sh.status()
    assert torch.equal(sel, ref_sel)
    if T >= 16:
        assert torch.equal(out, ref)
    with pytest.raises(lmb.QmsCudaError):
        shards[0].forward(xn)                       # a shard has no whole-block path
    for sh in shards:
        sh.close()
    full.close()


@pytest.mark.gpu
@pytest.mark.parametrize("S", [24, 600])
def test_experts_leave_out_of_range_rows(S):
    """qms_cuda_moe_experts / _experts_q8 skip rows whose local expert id is out of range (their dn
    rows keep what the caller put there) and the other rows come out as in a run without them.
    S = 24 slots over 16 local experts runs the grouped GEMV, S = 600 the tensor-core GEMMs."""
    import large_model_b200 as lmb
    lmb.init(0)
    layer = synth.make_moe_layer("tiny", seed=45)
    per = layer.n_expert // 2
    sh = lmb.MoeLayer.shard_from_synth(layer, 0, per)
    g = torch.Generator().manual_seed(3)
    x = torch.from_numpy(synth.make_hidden(layer.n_embd, S, seed=46)).cuda()
    ids = torch.randint(0, per, (S,), generator=g).to(torch.int32)
    r = torch.arange(S)
    bad = r % 5 == 0
    ids[bad] = torch.where(r[bad] % 2 == 0, torch.full_like(r[bad], -1), torch.full_like(r[bad], per + 3)).to(torch.int32)
    ids, badc, okc = ids.cuda(), bad.cuda(), (~bad).cuda()
    ref = sh.experts(x[okc].contiguous(), ids[okc].contiguous())
    for run, rows in ((sh.experts, x), (sh.experts_q8, lmb.quantize_q8(x))):
        dn = torch.full((S, layer.n_embd), 7.0, device="cuda")
        run(rows, ids, dn=dn)
        torch.cuda.synchronize()
        sh.status()
        assert torch.all(dn[badc] == 7.0)
        assert torch.equal(dn[okc], ref)
    sh.close()


def _narrow(S: int, nx: int) -> bool:
    """The expert kernels' width rule: 16-slot tiles (the grouped GEMV) while S <= 24 slots per
    expert, else the 64-slot tensor-core tiles; the two differ in float summation order."""
    return S <= 24 * nx


@pytest.mark.gpu
@pytest.mark.parametrize("shape,Ts", [("tiny", (20, 7)), ("30b", (40, 43)), ("30b", (48, 45, 40, 0))])
def test_ep_pack_exchange_combine_on_one_gpu(shape, Ts):
    """Ranks emulated on one GPU (the all-to-alls done by slicing segments): qms_cuda_ep_pack's slot
    map and ids equal the host restatement, its rows equal quantize_q8 of the tokens, the unused
    entries carry -1 (a rank with no tokens included); qms_cuda_ep_combine equals
    qms_cuda_moe_combine on the gathered rows bit for bit; and the layer output equals the unsharded
    layer bit for bit where both pick the same expert-kernel width, else the oracle within 1e-3
    relative L2 (the MoE bar)."""
    import large_model_b200 as lmb
    import oracle as oracle_mod
    from conftest import rel_l2
    lmb.init(0)
    layer = synth.make_moe_layer(shape, seed=47)
    N, X, K, E = len(Ts), layer.n_expert, layer.n_used, layer.n_embd
    per = X // N
    shards = [lmb.MoeLayer.shard_from_synth(layer, r * per, per) for r in range(N)]
    full = lmb.MoeLayer.from_synth(layer)
    cap = max(Ts) * K
    err = torch.zeros((1,), dtype=torch.int32, device="cuda")
    xs = [torch.from_numpy(synth.make_hidden(E, max(T, 1), seed=90 + r))[:T].contiguous().cuda()
          for r, T in enumerate(Ts)]
    rs = [torch.from_numpy(synth.make_hidden(E, max(T, 1), seed=95 + r))[:T].contiguous().cuda()
          for r, T in enumerate(Ts)]
    packs = []
    for r, x in enumerate(xs):
        sel, wts = shards[r].route_only(x)
        sx, se, slot = lmb.ep_pack(x, sel, X, N, cap, err=err)
        ref_slot, ref_ids, dropped = pack_index(sel.cpu(), X, N, cap)
        assert not dropped
        assert torch.equal(slot.cpu(), ref_slot), f"rank {r}: slot map"
        assert torch.equal(se.cpu(), ref_ids), f"rank {r}: expert ids / unused entries"
        if Ts[r]:
            s = slot.reshape(-1).long()
            assert torch.equal(sx[s], lmb.quantize_q8(x).repeat_interleave(K, dim=0)), f"rank {r}: Q8 rows"
        packs.append((sel, wts, sx, se, slot))
    rets = [torch.empty((N * cap, E), dtype=torch.float32, device="cuda") for _ in range(N)]
    for o in range(N):                                   # rank o: segment o of every rank, in rank order
        recv_x = torch.cat([p[2][o * cap:(o + 1) * cap] for p in packs])
        recv_e = torch.cat([p[3][o * cap:(o + 1) * cap] for p in packs])
        dn = shards[o].experts_q8(recv_x, recv_e)
        for r in range(N):
            rets[r][o * cap:(o + 1) * cap] = dn[r * cap:(r + 1) * cap]
    orc = oracle_mod.Oracle()
    for r, (x, resid) in enumerate(zip(xs, rs)):
        sel, wts, _, _, slot = packs[r]
        out = lmb.ep_combine(rets[r], slot, wts, resid)
        assert torch.equal(out, lmb.combine(rets[r][slot.reshape(-1).long()], wts, resid)), f"rank {r}: combine"
        if not Ts[r]:
            continue
        if _narrow(Ts[r] * K, X) == _narrow(N * cap, per):
            ref = full.forward(x, resid=resid)
            assert torch.equal(out, ref), f"rank {r}: differs from the unsharded layer"
        else:
            o_out = orc.moe(layer, x.cpu().numpy())[0]
            got = lmb.ep_combine(rets[r], slot, wts).cpu().numpy()
            assert rel_l2(got, o_out) < 1e-3, f"rank {r}: rel L2 {rel_l2(got, o_out):.3e}"
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for sh in shards:
        sh.status()
    full.status()
    for sh in shards:
        sh.close()
    full.close()


@pytest.mark.gpu
def test_ep_pack_overflow_is_flagged_on_one_gpu():
    """cap below the worst case: qms_cuda_ep_pack drops the slots past each segment's capacity and
    sets the flag, exactly as the host restatement says; the dropped slots' tokens come out NaN and
    every other token equals the run with room for all slots."""
    import large_model_b200 as lmb
    lmb.init(0)
    layer = synth.make_moe_layer("30b", seed=48)
    N, X, K, E, T = 2, layer.n_expert, layer.n_used, layer.n_embd, 40
    per = X // N
    sh = lmb.MoeLayer.shard_from_synth(layer, 0, per)
    x = torch.from_numpy(synth.make_hidden(E, T, seed=49)).cuda()
    sel, wts = sh.route_only(x)
    runs = {}
    for cap in (T * K, 100):
        err = torch.zeros((1,), dtype=torch.int32, device="cuda")
        sx, se, slot = lmb.ep_pack(x, sel, X, N, cap, err=err)
        ref_slot, ref_ids, dropped = pack_index(sel.cpu(), X, N, cap)
        assert torch.equal(slot.cpu(), ref_slot) and torch.equal(se.cpu(), ref_ids)
        assert int(err.item()) == int(dropped)
        # every segment through the shard for rank 0's experts; the other owner's rows stand in
        # for rank 1's experts (the combine only reads entries, it does not check who made them)
        ret = torch.cat([sh.experts_q8(sx[o * cap:(o + 1) * cap], se[o * cap:(o + 1) * cap]) for o in range(N)])
        runs[cap] = (lmb.ep_combine(ret, slot, wts), slot, dropped)
    full_out, _, d0 = runs[T * K]
    out, slot, dropped = runs[100]
    assert not d0 and dropped
    lost = (slot < 0).any(dim=1)
    assert lost.any() and not lost.all()
    assert torch.isnan(out[lost]).all(dim=1).all()
    assert torch.equal(out[~lost], full_out[~lost])
    sh.close()


@pytest.mark.gpu
def test_expert_calls_beyond_the_token_scratch():
    """An expert call of 20000 rows (a rank's segments at prefill sizes; more than the 65535 / K
    tokens a forward call may reserve) runs, and each row equals the same rows run in 5000-row
    calls bit for bit (both sizes take the 64-slot tensor-core tiles)."""
    import large_model_b200 as lmb
    lmb.init(0)
    layer = synth.make_moe_layer("tiny", seed=52)
    per = layer.n_expert // 2
    sh = lmb.MoeLayer.shard_from_synth(layer, per, per)
    S = 20000
    g = torch.Generator().manual_seed(5)
    x = torch.from_numpy(synth.make_hidden(layer.n_embd, S, seed=53)).cuda()
    ids = torch.randint(-1, per, (S,), generator=g).to(torch.int32).cuda()    # -1: unused entries
    xq = lmb.quantize_q8(x)
    whole = sh.experts_q8(xq, ids, dn=torch.zeros((S, layer.n_embd), device="cuda"))
    parts = torch.zeros_like(whole)
    for c in range(0, S, 5000):
        sh.experts_q8(xq[c:c + 5000], ids[c:c + 5000], dn=parts[c:c + 5000])
    torch.cuda.synchronize()
    sh.status()
    assert torch.equal(whole, parts)
    used = ids >= 0
    assert bool(torch.isfinite(whole[used]).all()) and bool((whole[used] != 0).any())
    sh.close()


@pytest.mark.gpu
@pytest.mark.parametrize("cap", [5600, 700])
def test_ep_pack_many_chunks_matches_restatement(cap):
    """qms_cuda_ep_pack over 5600 slots (the index kernel's 1024-slot chunks carry each owner's
    running count from chunk to chunk) with skewed expert ids over 4 ranks: slot map, ids, rows
    and overflow flag equal the host restatement; cap 700 drops slots in later chunks."""
    import large_model_b200 as lmb
    lmb.init(0)
    T, K, E, X, N = 700, 8, 512, 128, 4
    g = torch.Generator().manual_seed(9)
    w = torch.arange(1, X + 1, dtype=torch.float64).pow(-1.1)                   # Zipf-like popularity
    sel = torch.multinomial(w.expand(T, X), K, replacement=False, generator=g).to(torch.int32)
    x = torch.from_numpy(synth.make_hidden(E, T, seed=54)).cuda()
    err = torch.zeros((1,), dtype=torch.int32, device="cuda")
    sx, se, slot = lmb.ep_pack(x, sel.cuda(), X, N, cap, err=err)
    ref_slot, ref_ids, dropped = pack_index(sel, X, N, cap)
    torch.cuda.synchronize()
    assert torch.equal(slot.cpu(), ref_slot)
    assert torch.equal(se.cpu(), ref_ids)
    assert int(err.item()) == int(dropped) and dropped == (cap == 700)     # owner 0 gets 4138 slots
    s = slot.reshape(-1).long()
    kept = s >= 0
    rows = lmb.quantize_q8(x).repeat_interleave(K, dim=0)
    assert torch.equal(sx[s[kept]], rows[kept])
