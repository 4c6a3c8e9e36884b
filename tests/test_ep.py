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
        dn = np.empty((xq.shape[0], E), np.float32)
        for i, (row, le) in enumerate(zip(xq.numpy(), local_expert.tolist())):
            assert 0 <= le < self.n_local
            e = self.base + le
            gw = L.gate[e * self.gu_bytes:(e + 1) * self.gu_bytes]
            uw = L.up[e * self.gu_bytes:(e + 1) * self.gu_bytes]
            dw = L.down[e * self.dn_bytes:(e + 1) * self.dn_bytes]
            g = self.o.matmul_q8(L.gate_type, F, E, gw, row)[0]
            u = self.o.matmul_q8(L.up_type, F, E, uw, row)[0]
            dn[i] = self.o.matmul(L.down_type, E, F, dw, self.o.swiglu(g, u))[0]
        return torch.from_numpy(dn)

    def combine(self, dn, wts, resid):
        T, K = wts.shape
        d = dn.reshape(T, K, -1)
        out = torch.zeros((T, d.shape[-1]), dtype=torch.float32)
        for j in range(K):                                      # selection order
            out = out + wts[:, j:j + 1] * d[:, j]
        return out if resid is None else resid + out


def unsharded(backend, xn, resid=None):
    sel, wts = backend.route(xn)
    T, K = sel.shape
    dn = backend.experts(xn.repeat_interleave(K, dim=0), sel.reshape(-1).to(torch.int32))
    return backend.combine(dn, wts, resid)


def _cpu_rank(rank, world, port, shape, T, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = synth.make_moe_layer(shape, seed=41)
        per = layer.n_expert // world
        ep = ExpertParallelMoe(OracleBackend(layer, rank * per, per), layer.n_expert, layer.n_used, layer.n_embd)
        xn = torch.from_numpy(synth.make_hidden(layer.n_embd, T + rank, seed=50 + rank))   # ragged T per rank
        resid = torch.from_numpy(synth.make_hidden(layer.n_embd, T + rank, seed=60 + rank))
        out = ep.forward(xn, resid)
        ref = unsharded(OracleBackend(layer, 0, layer.n_expert), xn, resid)
        q.put((rank, bool(torch.equal(out, ref)), float((out - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_dispatch_combine_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank, args=(r, world, port, "tiny", 5, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for rank, equal, diff in res:
        assert equal, f"rank {rank}: EP differs from the unsharded layer by {diff}"


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
        ep = ExpertParallelMoe(CudaBackend(shard), layer.n_expert, layer.n_used, layer.n_embd)
        xn = torch.from_numpy(synth.make_hidden(layer.n_embd, T + 3 * rank, seed=70 + rank)).cuda()
        resid = torch.from_numpy(synth.make_hidden(layer.n_embd, T + 3 * rank, seed=80 + rank)).cuda()
        out = ep.forward(xn, resid)
        full = lmb.MoeLayer.from_synth(layer)
        ref = full.forward(xn, resid=resid)
        torch.cuda.synchronize()
        shard.status()
        full.status()
        q.put((rank, bool(torch.equal(out, ref)), float((out - ref).abs().max())))
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
