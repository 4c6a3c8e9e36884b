"""Expert parallelism (EP) for batched decode and prefill: the experts of a layer are split over
the ranks of a process group, tokens stay on the rank that owns them.

Rank r holds experts [r * X/N, (r+1) * X/N) as a shard layer (qms_cuda_moe_create_shard) and the
full router. One call of a layer, on every rank:

1. route its own tokens (replicated router, src/model.c:1043-1064): sel / wts [T][K];
2. quantise its token rows once into Q8 blocks (the reference's QmsQ8, 44 bytes per 32 values,
   src/kernels.h:7-12) and send every (token, slot) row to the rank owning the slot's expert: an
   all-to-all of the per-rank counts, then of the Q8 rows and of the local expert ids, in slot order;
3. run the received rows through the local experts (the grouped kernels) into their unweighted
   down rows;
4. return those rows with the reverse all-to-all;
5. combine each token's K down rows in selection order, plus the residual (src/model.c:1152-1162).

Every per-slot computation is the same as in a single-GPU call, so the output is bitwise equal to
the unsharded layer's grouped path. Collectives go through torch.distributed (NCCL on GPUs, gloo in
the CPU tests); the compute steps come from a backend object so the dispatch logic can be tested
without a GPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class CudaBackend:
    """Compute steps on a B200 through the C ABI: a shard layer of large_model_b200."""

    def __init__(self, shard):
        self.layer = shard

    def route(self, xn):
        return self.layer.route_only(xn)

    def quantize(self, xn):
        from . import quantize_q8
        return quantize_q8(xn)

    def experts_q8(self, xq, local_expert):
        return self.layer.experts_q8(xq, local_expert)

    def combine(self, dn, wts, resid):
        from . import combine
        return combine(dn, wts, resid)


def _all_to_all(out, inp, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


class ExpertParallelMoe:
    """One MoE layer sharded by expert over `group` (every rank calls forward with its own tokens)."""

    def __init__(self, backend, n_expert: int, n_used: int, n_embd: int, group=None):
        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_expert % self.world:
            raise ValueError(f"{n_expert} experts do not split evenly over {self.world} ranks")
        self.per_rank = n_expert // self.world
        self.K, self.E = n_used, n_embd

    def forward(self, xn, resid=None):
        T = xn.shape[0]
        dev = xn.device
        sel, wts = self.backend.route(xn)                         # [T][K] global ids, weights
        flat = sel.reshape(-1).to(torch.int64)
        dest = flat // self.per_rank
        order = torch.argsort(dest, stable=True)                  # slots grouped by owner, slot order kept
        send_counts = torch.bincount(dest, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        S = sum(rc)
        xq = self.backend.quantize(xn)                            # [T][E/32 * 44] bytes
        send_x = xq[order // self.K].contiguous()
        send_e = (flat[order] % self.per_rank).to(torch.int32).contiguous()
        recv_x = torch.empty((S, xq.shape[1]), dtype=xq.dtype, device=dev)
        recv_e = torch.empty((S,), dtype=torch.int32, device=dev)
        _all_to_all(recv_x, send_x, rc, sc, self.group)
        _all_to_all(recv_e, send_e, rc, sc, self.group)
        dn_recv = self.backend.experts_q8(recv_x, recv_e) if S else torch.empty((0, self.E), device=dev)
        dn_sorted = torch.empty((T * self.K, self.E), dtype=torch.float32, device=dev)
        _all_to_all(dn_sorted, dn_recv.contiguous(), sc, rc, self.group)
        dn = torch.empty_like(dn_sorted)
        dn[order] = dn_sorted
        return self.backend.combine(dn, wts, resid)
