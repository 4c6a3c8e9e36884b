"""Expert parallelism (EP) for batched decode and prefill: the experts of a layer are split over
the ranks of a process group, tokens stay on the rank that owns them.

Rank r holds experts [r * X/N, (r+1) * X/N) as a shard layer (qms_cuda_moe_create_shard) and the
full router. One call of a layer, on every rank, with nothing read back to the host:

1. route its own tokens (replicated router, src/model.c:1043-1064): sel / wts [T][K];
2. pack (qms_cuda_ep_pack): every (token, slot) row, quantised once into Q8 blocks (the reference's
   QmsQ8, 44 bytes per 32 values, src/kernels.h:7-12), goes to the segment of the rank owning the
   slot's expert, at its index among that owner's slots in slot order. The send buffer holds N
   segments of `cap` entries whatever the routing; unused entries carry expert id -1;
3. two fixed-size all-to-alls (the rows and the ids): segment o goes to rank o;
4. the received rows run through the local experts (the grouped kernels; -1 entries are skipped)
   into their unweighted down rows;
5. one fixed-size all-to-all returns the down rows to the segments they came from;
6. combine each token's K down rows in selection order, read through the slot map, plus the
   residual (src/model.c:1152-1162; qms_cuda_ep_combine).

Segments have the same size on every rank, so no counts cross the host and the call can be captured
in a CUDA graph. cap = max_tokens * K can never overflow; a smaller cap moves fewer bytes, and a slot
past its segment's capacity is dropped, raises the overflow flag (`overflowed()`) and makes its
token's output NaN. Every per-slot computation is the same as in a single-GPU call, so the output is
bitwise equal to the unsharded layer's grouped path. Collectives go through torch.distributed (NCCL on
GPUs, gloo in the CPU tests); the compute steps come from a backend object so the dispatch logic can be
tested without a GPU.
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

    def new_flag(self, device):
        return torch.zeros((1,), dtype=torch.int32, device=device)

    def pack(self, xn, sel, n_expert, n_rank, cap, err):
        from . import ep_pack
        return ep_pack(xn, sel, n_expert, n_rank, cap, err=err)

    def experts_q8(self, xq, local_expert):
        return self.layer.experts_q8(xq, local_expert)

    def combine_slots(self, ret, slot, wts, resid):
        from . import ep_combine
        return ep_combine(ret, slot, wts, resid)


class ExpertParallelMoe:
    """One MoE layer sharded by expert over `group` (every rank calls forward with its own tokens,
    at most `max_tokens` of them; `cap` entries per destination rank, max_tokens * n_used by default)."""

    def __init__(self, backend, n_expert: int, n_used: int, n_embd: int, max_tokens: int, cap: int | None = None,
                 group=None):
        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_expert % self.world:
            raise ValueError(f"{n_expert} experts do not split evenly over {self.world} ranks")
        if max_tokens < 1:
            raise ValueError("max_tokens must be at least 1")
        self.n_expert, self.K, self.E = n_expert, n_used, n_embd
        self.max_tokens = max_tokens
        self.cap = cap if cap is not None else max_tokens * n_used
        self.err = None

    def forward(self, xn, resid=None):
        T = xn.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        if self.err is None:
            self.err = self.backend.new_flag(xn.device)
        sel, wts = self.backend.route(xn)                        # [T][K] global ids, weights
        send_x, send_e, slot = self.backend.pack(xn, sel, self.n_expert, self.world, self.cap, self.err)
        recv_x, recv_e = torch.empty_like(send_x), torch.empty_like(send_e)
        dist.all_to_all_single(recv_x, send_x, group=self.group)
        dist.all_to_all_single(recv_e, send_e, group=self.group)
        dn = self.backend.experts_q8(recv_x, recv_e)             # [world * cap][E], -1 entries untouched
        ret = torch.empty_like(dn)
        dist.all_to_all_single(ret, dn, group=self.group)
        return self.backend.combine_slots(ret, slot, wts, resid)

    def overflowed(self) -> bool:
        """True when a slot of some call so far did not fit its segment (reads the device flag)."""
        return self.err is not None and int(self.err.item()) != 0
