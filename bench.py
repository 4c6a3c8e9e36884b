"""Benchmarks of the Qwen3-MoE path on B200 (libqms_cuda through its C ABI).

Default (--mode model, BASELINE.json config 4 at batch 1): Qwen3-235B-A22B, the whole model on one
GPU - 94 layers, hidden 4096, 64 Q / 4 KV heads x 128, 128 experts top-8, moe_intermediate 1536,
Q4_0 weights and a Q6_K head drawn on the device with the configs' distributions (124 GiB resident),
fp32 KV cache of 4096 positions. A 1024-id random prompt is prefilled, then a step is 32 greedy
decode tokens: qms_cuda_decode_step captured once in a CUDA graph (argmax, position and next
embedding stay on the device). The metric is decode tokens/s; the roofline compares the bytes one
token must read (weights of the 8 selected experts in every layer, attention weights, the head, the
KV cache) with the measured HBM bandwidth.

--mode moe: the Qwen3-235B-A22B MoE layer operator at decode batch 1 —
hidden 4096, 128 experts, top-8, moe_intermediate 1536, Q4_0 experts, F32 router — on 1000
seeded tokens, each an independent T=1 call. Calls cycle through 8 resident layers with
independent seeded weights (8 x 1.36 GB), so consecutive calls share no weights and every
step's inputs are far larger than L2. A step is the 1000 calls; the metric is the MoE layer's
algorithmic HBM bytes (8 experts x 10,616,832 B + 2,097,152 B router = 87,031,808 B per
token-layer) divided by time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--mode model|moe|bs64|prefill]

N > 1 runs N independent replicas (one per GPU, launched by torch.distributed.run): batch-1
decode does not shard, so there is no collective on the data path (scaling "weak").

    python bench.py --mode bs64      # the same layer at T=64 tokens per call (config 4's bs64 operator)
    python bench.py --mode prefill   # T=4096 tokens per call (config 5's operator, per sequence)

The batched modes print their own JSON line: bs64 runs the expert-grouped GEMV (HBM roofline over
the distinct experts a call reads), prefill the expert-grouped tcgen05 GEMMs (int8 tensor roofline
over the block's integer ops). Under torch.distributed.run, `--ep` shards the experts over the
ranks (NCCL all-to-all of the slots' Q8 rows) instead of running replicas.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPE = "235b"
TOKENS = 1000
LAYERS = 8
METRIC = "Qwen3-235B Q4_0 MoE-layer HBM GB/s (decode bs1)"
WORKLOAD = ("Qwen3-235B-A22B MoE layer operator, decode bs1 (config 2): 1000 seeded tokens per step, "
            "each an independent T=1 call, cycling 8 resident layers of independent seeded weights")


def bytes_per_token_layer(E=4096, X=128, K=8, F=1536) -> int:
    expert = 3 * F * (E // 32) * 18          # gate + up + down, Q4_0 (18 bytes per 32 weights)
    return K * expert + X * E * 4            # + F32 router


def bytes_per_launch(E=4096, X=128, K=8, F=1536) -> int:
    """Bytes one batch-1 call of k_decode_bs1 must read: the F32 router and the gate, up and down
    weights of the K selected experts (the whole MoE block is one kernel)."""
    return bytes_per_token_layer(E, X, K, F)


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic() -> float | None:
    """DRAM bytes per k_decode_bs1 launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "k_decode_bs1_235b.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip())
    return None


# ---- clocks ------------------------------------------------------------------------------------

class ClockSampler:
    def __init__(self, gpu_index: int):
        self.path = Path(f"/tmp/qms_clocks_{os.getpid()}.csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-i", str(gpu_index), "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        load = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---- CPU: the reference's own moe() ------------------------------------------------------------

def cpu_reference_rate(seconds: float = 8.0, max_calls: int = 2000, layers: int = 2):
    """Time the reference build's moe() (oracle/_ref, compiled from its sources) on T=1 calls of
    the same workload, all host threads, `layers` resident 235B-shape layers in host RAM."""
    from oracle import Reference, host_threads
    from large_model_b200 import synth
    ref = Reference()
    threads = host_threads()
    ref.set_threads(threads)
    ls = [synth.make_moe_layer(SHAPE, seed=1000 + i) for i in range(layers)]
    xn = synth.make_hidden(ls[0].n_embd, 64, seed=2000)
    for t in range(4):                                    # warm-up (page in, thread pool)
        ref.moe(ls[t % layers], xn[t])
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (time.perf_counter() - t0 < seconds or n < 8):
        ref.moe(ls[n % layers], xn[n % len(xn)])
        n += 1
    dt = time.perf_counter() - t0
    gbs = n * bytes_per_token_layer() / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"{n} T=1 moe() calls over {layers} seeded 235B-shape layers in host RAM "
                      f"({dt:.1f} s, reference build {ref.variant}, {threads} OpenMP threads)"}, n, dt


def cpu_reference_batched(T: int, seconds: float = 10.0, layers: int = 2, zipf: float = 0.0):
    """The reference's moe() on T-token calls (moe() is sequence-agnostic), all host threads; with
    zipf > 0 the layers and tokens carry config 5's Zipf(zipf) skew."""
    from oracle import Reference, host_threads
    from large_model_b200 import synth
    ref = Reference()
    threads = host_threads()
    ref.set_threads(threads)
    ls = [synth.make_moe_layer(SHAPE, seed=1000 + i) for i in range(layers)]
    xn = synth.make_hidden(ls[0].n_embd, T, seed=2001)
    if zipf > 0:
        skewed = [synth.zipf_layer_and_hidden(l, T, s=zipf, seed=2002) for l in ls]
        ls, xn = [l for l, _ in skewed], skewed[0][1]
    ref.moe(ls[0], xn[: min(T, 8)])                       # warm-up (page in, thread pool)
    n, t0 = 0, time.perf_counter()
    while n < 1 or (time.perf_counter() - t0 < seconds and n < 64):
        ref.moe(ls[n % layers], xn)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n * T / dt, 1), "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"{n} T={T} moe() calls over {layers} seeded 235B-shape layers in host RAM "
                      f"({dt:.1f} s, reference build {ref.variant}, {threads} OpenMP threads)"}


def run_reference_arm(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import Reference, host_threads
    from large_model_b200 import synth
    ref = Reference()
    threads = host_threads()
    ref.set_threads(threads)
    ls = [synth.make_moe_layer(SHAPE, seed=1000 + i) for i in range(2)]
    xn = synth.make_hidden(ls[0].n_embd, 64, seed=2000)
    calls_per_step = 16
    k = 0
    for _ in range(a.warmup):
        for _ in range(calls_per_step):
            ref.moe(ls[k % 2], xn[k % 64])
            k += 1
    t0 = time.perf_counter()
    for _ in range(a.steps):
        for _ in range(calls_per_step):
            ref.moe(ls[k % 2], xn[k % 64])
            k += 1
    dt = time.perf_counter() - t0
    value = a.steps * calls_per_step * bytes_per_token_layer() / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt / a.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32",
            "data": "synthetic",
            "config": {"workload": WORKLOAD + f"; reference CPU arm: each step {calls_per_step} T=1 calls "
                                              f"over 2 resident layers", "tokens_per_step": calls_per_step},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": f"{calls_per_step} T=1 moe() calls per step, reference build {ref.variant}"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU ---------------------------------------------------------------------------------------

def zipf_direction(torch, E: int, X: int, s: float, seed: int, device, mu: float = 4.0):
    """Config 5's skew (large_model_b200.synth.zipf_layer_and_hidden, on the device): a unit vector u
    shared by every token's hidden state (x = z + mu u) and per-expert router offsets
    (b_e / mu) u with b_e = 0.02 sqrt(E) s log(1 / rank_e), so expert e is picked ~ rank_e^-s."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    u = torch.randn(E, generator=g, device=device, dtype=torch.float64)
    u /= u.norm()
    rank = torch.randperm(X, generator=g, device=device).to(torch.float64) + 1
    b = 0.02 * E ** 0.5 * s * -torch.log(rank)
    return u, b, mu


def device_layer(q, torch, seed: int, device, shard=None, zipf=None):
    """A 235B-shape layer drawn on the device with the config's distributions, then uploaded
    through qms_cuda_moe_create from device memory (GGUF layout, repacked by the library).
    shard = (expert_base, n_local): only those experts (an expert-parallel shard); zipf = the
    (u, b, mu) of zipf_direction: the router rows get config 5's skew."""
    from large_model_b200 import synth
    E, X, K, F = synth.MOE_SHAPES[SHAPE]
    XL = X if shard is None else shard[1]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    router = torch.randn((X, E), generator=g, device=device, dtype=torch.float32) * 0.02
    if zipf is not None:
        u, b, mu = zipf
        router = (router.double() + (b / mu)[:, None] * u[None, :]).float().contiguous()

    def q4_0(nblocks):
        blk = torch.empty((nblocks, 18), dtype=torch.uint8, device=device)
        d = (torch.rand(nblocks, generator=g, device=device) * 0.004 + 0.002).to(torch.float16)
        blk[:, 0:2] = d.view(torch.uint8).view(nblocks, 2)
        nib = torch.randint(-2 ** 31, 2 ** 31 - 1, (nblocks, 4), generator=g, device=device, dtype=torch.int32)
        blk[:, 2:] = nib.view(torch.uint8).view(nblocks, 16)
        return blk.view(-1)

    gate, up, down = q4_0(XL * F * E // 32), q4_0(XL * F * E // 32), q4_0(XL * E * F // 32)
    m = q.MoeLayer(E, X, K, F, router, gate, up, down, shard=shard)
    del router, gate, up, down
    return m


BATCH_T = {"bs64": 64, "prefill": 4096}


def run_batched(a):
    """T > 1 operator benchmark: alternating calls on 2 resident 235B-shape layers (2.7 GB > L2)."""
    import torch
    import large_model_b200 as q
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    q.init(local)
    dev = torch.device("cuda", local)
    T = BATCH_T[a.mode]
    E, X, K, F = 4096, 128, 8, 1536
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        cpu = cpu_reference_batched(T, seconds=10.0 if T <= 256 else 20.0, zipf=a.zipf)
    ep = a.ep and world > 1
    zipf = zipf_direction(torch, E, X, a.zipf, 31, dev) if a.zipf > 0 else None
    if ep:                                            # expert parallelism: X / world experts per rank
        from large_model_b200.ep import CudaBackend, ExpertParallelMoe
        per = X // world
        layers = [device_layer(q, torch, 500 + 17 * i, dev, shard=(rank * per, per), zipf=zipf) for i in range(2)]
        eps = [ExpertParallelMoe(CudaBackend(m), X, K, E, max_tokens=T) for m in layers]
    else:
        layers = [device_layer(q, torch, 500 + 17 * i, dev, zipf=zipf) for i in range(2)]
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)                          # every rank its own tokens
    xs = [torch.randn((T, E), generator=g, device=dev, dtype=torch.float32) for _ in range(2)]
    if zipf is not None:                              # the component every token shares
        xs = [(x + (zipf[2] * zipf[0]).float()[None, :]).contiguous() for x in xs]
    out = torch.empty((T, E), device=dev, dtype=torch.float32)
    for m in layers:
        m.reserve(T)
    calls = 8 if T <= 256 or a.zipf > 0 else 2      # config 5: 8 sequences x 4096 tokens per step
    stream = torch.cuda.Stream(device=dev)

    def step():
        for c in range(calls):
            if ep:
                eps[c % 2].forward(xs[(c // 2) % 2])
            else:
                layers[c % 2].forward(xs[(c // 2) % 2], out=out, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            step()
    torch.cuda.synchronize()
    # distinct experts per call (bytes a call must read)
    # (under EP: the union over all ranks' tokens - each expert is read once, by its owner)
    distinct = []
    for i in range(2):
        sel, _ = layers[i].route_only(xs[i])
        if ep:
            sels = [torch.empty_like(sel) for _ in range(world)]
            dist.all_gather(sels, sel)
            sel = torch.cat(sels)
        distinct.append(len(torch.unique(sel)))
        max_expert = int(torch.bincount(sel.reshape(-1).long(), minlength=X).max().item())
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(a.steps):
            step()
        ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    call_ms = ms / (a.steps * calls)
    tok_s = T * a.steps * calls * world / (ms / 1e3)
    # per-stage timing (router, gate/up + SwiGLU, down + combine) of single calls
    kev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ksum = [0.0, 0.0, 0.0]
    nk = 0 if ep else 4
    for c in range(nk):
        m = layers[c % 2]
        m.set_kernel_events(kev)
        with torch.cuda.stream(stream):
            m.forward(xs[c % 2], out=out, stream=stream)
        m.set_kernel_events(None)
        stream.synchronize()
        for i in range(3):
            ksum[i] += kev[2 * i].elapsed_time(kev[2 * i + 1]) / nk
    expert_bytes = 3 * F * (E // 32) * 18
    if ep:                                           # all ranks together, per call time
        call_bytes = world * X * E * 4 + statistics.mean(distinct) * expert_bytes
    else:
        call_bytes = world * (X * E * 4 + statistics.mean(distinct) * expert_bytes)
    ops = T * K * 6 * F * E                          # gate, up, down: 3 F E multiply-adds per slot
    # end to end through the host-buffer entry point
    xh = torch.empty((T, E), dtype=torch.float32, pin_memory=True)
    xh.copy_(xs[0].cpu())
    oh = torch.empty_like(xh, pin_memory=True)
    e2e_n = 4 if T <= 256 else 2
    e2e = None
    if not ep:
        layers[0].forward_host(xh.numpy(), out=oh.numpy())
        t0 = time.perf_counter()
        for i in range(e2e_n):
            layers[i % 2].forward_host(xh.numpy(), out=oh.numpy())
        e2e_s = time.perf_counter() - t0
        if dist:                                     # replicas: max over ranks, all ranks' tokens
            t = torch.tensor([e2e_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = {"value": round(T * world * e2e_n / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": T * E * 4,
               "d2h_bytes_per_step": T * E * 4, "note": "qms_cuda_moe_forward_host per call"}
    else:                                            # every rank: its tokens in from and out to pinned host memory
        def host_call(i):
            x = xh.to(dev, non_blocking=True)
            oh.copy_(eps[i % 2].forward(x), non_blocking=True)
            torch.cuda.current_stream().synchronize()
        host_call(0)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_n):
            host_call(i)
        t = torch.tensor([time.perf_counter() - t0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = {"value": round(T * world * e2e_n / float(t.item()), 1), "unit": "tok/s",
               "h2d_bytes_per_step": T * E * 4, "d2h_bytes_per_step": T * E * 4,
               "note": "per rank: its T tokens from pinned host memory, ExpertParallelMoe.forward, result to "
                       "pinned host memory; max over ranks"}
    # kernels of this library per call (the routing, grouping, expert and combine kernels of the path
    # the call takes; torch's own copies and all-to-alls under EP not counted)
    # (under EP the expert kernels see every segment entry: world * T * K slots over X / world experts)
    gemv = world * T * K <= 24 * (X // world) if ep else T * K <= 24 * X
    per_call = (11 if gemv else 12) if ep else (7 if gemv else 9)
    launches = per_call * calls * a.steps
    if rank == 0:
        if a.mode == "bs64":
            peak, peak_kind = peaks()
            gbs = call_bytes / (call_ms / 1e3) / 1e9
            roof = {"bound": "hbm", "kernel": "whole block (router, k_mma_group, k_gv_gate_up, k_gv_down, combine)",
                    "achieved": round(gbs, 1), "peak": peak * world, "unit": "GB/s",
                    "frac": round(gbs / (peak * world), 4),
                    "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                    "bytes_per_call": int(call_bytes), "distinct_experts_per_call": statistics.mean(distinct),
                    # DRAM bytes of k_gv_gate_up + k_gv_down for one call, one ncu capture
                    # (profiles/k_gv_235b_bs64.md), against ~1.32 GB algorithmic
                    "traffic": 1339233024 if world == 1 else None}
            metric, unit, value = "Qwen3-235B Q4_0 MoE-layer decode bs64 tokens/s (operator)", "tok/s", tok_s
        else:
            tops = world * ops / (call_ms / 1e3) / 1e12
            # The real bound: every 32-value block product's int32 sum is scaled in fp32 on the CUDA
            # cores (the reference's per-block arithmetic): at least ~2.5 instructions per block
            # product (int -> float, d_w * d_x, the FMA; profiles/k_mma_gemm_235b_bs64_prefill.md),
            # issued at 4 warp instructions per clock per SM.
            products = T * K * (2 * F * (E // 32) + E * (F // 32))
            sm_hz = (clocks.get("sm_mhz") or 1965.0) * 1e6
            floor_ms = products * 2.5 / (torch.cuda.get_device_properties(dev).multi_processor_count * 4 * 32 * sm_hz) * 1e3
            roof = {"bound": "tensor", "kernel": "whole block (router, k_mma_group, gathers, k_mma_gemm x2, combine)",
                    "achieved": round(tops, 1), "peak": 4500.0 * world, "unit": "TOP/s",
                    "frac": round(tops / (4500.0 * world), 4),
                    "peak_kind": "nominal dense int8 (no measured int8 peak on this pool)", "traffic": None,
                    "ops_per_call": ops,
                    "epilogue_bound": {"block_products_per_call": products, "instructions_per_product": 2.5,
                                       "floor_ms_per_call": round(floor_ms, 3),
                                       "frac": round(floor_ms / call_ms, 4),
                                       "note": "per-block fp32 scaling on the CUDA cores; the frac is that floor "
                                               "over the measured call time"}}
            metric, unit, value = "Qwen3-235B Q4_0 MoE-layer prefill tokens/s (operator, 4096-token calls)", "tok/s", tok_s
        line = {"metric": metric, "value": round(value, 1), "unit": unit, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
                "config": {"workload": f"Qwen3-235B-A22B MoE layer operator, T={T} tokens per call, {calls} calls "
                                       f"per step alternating 2 resident layers of seeded weights",
                           "tokens_per_call": T, "ms_per_call": round(call_ms, 4),
                           "stage_ms": {"router": round(ksum[0], 4), "gate_up_swiglu": round(ksum[1], 4),
                                        "down_combine": round(ksum[2], 4)},
                           "l2": "inputs larger than L2 (2 layers x 1.36 GB resident)",
                           "routing": (f"Zipf({a.zipf}) expert popularity (config 5): a shared hidden-state "
                                       f"component and per-expert router offsets; per call the busiest expert "
                                       f"takes {max_expert} of {T * K * (world if ep else 1)} slots"
                                       f"{' (all ranks: each rank its own T tokens)' if ep else ''}"
                                       if a.zipf > 0 else
                                       "seeded N(0,1) hidden states, N(0,0.02) router (near-uniform expert load)"),
                           "parallelism": (f"expert-parallel x{world} (device dispatch into fixed-capacity segments, "
                                           f"NCCL all-to-all)" if ep else f"replicas x{world}")},
                "roofline": roof, "cpu_baseline": cpu,
                "e2e": e2e,
                "gpu_launches": launches, "clocks": clocks}
        print(json.dumps(line), flush=True)
    for m in layers:
        m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---- the whole model (config 4, batch 1) ------------------------------------------------------------

MODEL_METRIC = "Qwen3-235B-A22B Q4_0 decode tok/s (bs1, whole model on one B200)"
MODEL_PROMPT = 1024
MODEL_CTX = 4096
TOKENS_PER_STEP = 32
BATCH_METRIC = "Qwen3-235B-A22B Q4_0 decode tok/s (bs64: 64 sequences, whole model on one B200)"
BATCH_SEQS = 64
BATCH_CTX = MODEL_PROMPT + 128                  # positions per sequence's KV cache
BATCH_OWN = 128                                 # prompt ids of each sequence's own (after a shared prefix)


def model_cfg(layers: int = 0):
    """Config 4 (Qwen3-235B-A22B); layers > 0 keeps that many layers (small cases for ncu captures;
    a bench line with fewer layers says so in its config)."""
    import dataclasses
    from large_model_b200 import synth
    cfg = synth.MODEL_CONFIGS["235b"]
    return dataclasses.replace(cfg, n_layer=layers) if layers > 0 else cfg


def model_bytes_per_token(cfg, pos: float, kv_es: int = 4) -> dict:
    """Algorithmic bytes one decode token at position `pos` must read, by part (GGUF sizes):
    per layer the router and 8 experts, the q/k/v/o projections, the fp32 K and V rows of every
    earlier position, the norms; plus the embedding row and the Q6_K head."""
    E, X, K, F, L = cfg.n_embd, cfg.n_expert, cfg.n_used, cfg.n_ff, cfg.n_layer
    QD, KD = cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
    moe = K * 3 * F * (E // 32) * 18 + X * E * 4
    attn = (QD + 2 * KD) * (E // 32) * 18 + E * (QD // 32) * 18
    kv = 2 * KD * kv_es * (pos + 1)
    norms = (2 * E + 2 * cfg.head_dim) * 4
    head = cfg.vocab * (E // 256) * 210
    parts = {"moe": L * moe, "attention_weights": L * attn, "kv_cache": L * kv, "norms": L * norms + E * 4,
             "head": head, "embedding_row": (E // 32) * 18}
    parts["total"] = sum(parts.values())
    return parts


def device_model(q, torch, cfg, seed: int, dev, ctx: int):
    """The 235B architecture drawn on the device with the configs' distributions (Q4_0 nibbles
    uniform 0..15 with fp16 scales U(0.002, 0.006), router N(0, 0.02), norms 1 + N(0, 0.01), a Q6_K
    head of uniform 6-bit values) and uploaded layer by layer from device memory (qms_cuda_model_*)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    E, D, H, Hk, X, F, V = cfg.n_embd, cfg.head_dim, cfg.n_head, cfg.n_head_kv, cfg.n_expert, cfg.n_ff, cfg.vocab

    def q4_0(n):
        nb = n // 32
        blk = torch.empty((nb, 18), dtype=torch.uint8, device=dev)
        blk[:, 0:2] = (torch.rand(nb, generator=g, device=dev) * 0.004 + 0.002).to(torch.float16).view(torch.uint8).view(nb, 2)
        blk[:, 2:] = torch.randint(-2 ** 31, 2 ** 31 - 1, (nb, 4), generator=g, device=dev, dtype=torch.int32).view(torch.uint8).view(nb, 16)
        return blk.view(-1)

    def q6_k(n):
        nb = n // 256
        blk = torch.empty((nb, 210), dtype=torch.uint8, device=dev)
        blk[:, :192] = torch.randint(-2 ** 31, 2 ** 31 - 1, (nb, 48), generator=g, device=dev, dtype=torch.int32).view(torch.uint8).view(nb, 192)
        blk[:, 192:208] = torch.randint(2, 9, (nb, 16), generator=g, device=dev, dtype=torch.uint8)
        blk[:, 208:210] = (torch.rand(nb, generator=g, device=dev) * 1.5e-4 + 1.5e-4).to(torch.float16).view(torch.uint8).view(nb, 2)
        return blk.view(-1)

    def norm(n):
        return 1.0 + 0.01 * torch.randn(n, generator=g, device=dev, dtype=torch.float32)

    trunk = {"token_embd.weight": q4_0(V * E), "output_norm.weight": norm(E), "output.weight": q6_k(V * E)}
    m = q.Model(cfg, trunk, ctx)
    del trunk
    QD, KD = H * D, Hk * D
    for l in range(cfg.n_layer):
        t = {"attn_norm": norm(E), "attn_q_norm": norm(D), "attn_k_norm": norm(D), "ffn_norm": norm(E),
             "attn_q": q4_0(QD * E), "attn_k": q4_0(KD * E), "attn_v": q4_0(KD * E), "attn_output": q4_0(E * QD),
             "ffn_gate_inp": torch.randn((X, E), generator=g, device=dev, dtype=torch.float32) * 0.02,
             "ffn_gate_exps": q4_0(X * F * E), "ffn_up_exps": q4_0(X * F * E), "ffn_down_exps": q4_0(X * E * F)}
        m.set_layer(l, t)
        del t
    torch.cuda.synchronize()
    return m


def host_model_tensors(cfg, seed: int) -> dict:
    """The same architecture as host arrays (numpy, seeded) for the reference's CPU forward."""
    from large_model_b200 import synth
    out = {}
    for i, (name, typ, ne) in enumerate(synth.model_tensors(cfg)):
        out[name] = np.ascontiguousarray(synth.tensor_data(cfg, seed, i))
    return out


def cpu_model_sample(layers=(2, 8), decode_tokens: int = 8, prompt: int = 256, seed: int = 77):
    """The reference's own qms_forward (oracle/_ref, compiled from its sources) on 235B-shape models
    of `layers` layers in host RAM (the full 94-layer model needs ~135 GB of host memory): each
    model prefills a random prompt, then the sizes decode `decode_tokens` tokens each, one call at a
    time and interleaved (both see the same host load). The time per token is linear in the layer count (t = fixed + L * per_layer: embedding and head, then
    identical layers), so two sizes give the 94-layer time. Returns (seconds per 94-layer token,
    description, threads)."""
    import dataclasses
    from oracle import Reference, host_threads
    ref = Reference()
    threads = host_threads()
    ref.set_threads(threads)
    base = model_cfg()
    attempts = 3
    models = {}
    try:
        for L in layers:
            cfg = dataclasses.replace(base, n_layer=L)
            t = host_model_tensors(cfg, seed)
            m = ref.model(cfg, t, prompt + 1 + attempts * decode_tokens + 4)
            ids = [int(v) for v in np.random.default_rng(seed).integers(0, cfg.vocab, prompt)]
            logits = m.forward(ids, 0)
            logits = m.forward([int(np.argmax(logits))], prompt)      # warm-up (thread pool, page-in)
            models[L] = [m, t, logits, prompt + 1]
        # the sizes' tokens interleaved, so both medians see the same host load; a slope that is
        # not positive (load that changed between the sizes anyway) is measured again
        for attempt in range(attempts):
            ts = {L: [] for L in layers}
            for _ in range(decode_tokens):
                for L in layers:
                    m, _, logits, pos = models[L]
                    t0 = time.perf_counter()
                    logits = m.forward([int(np.argmax(logits))], pos)
                    ts[L].append(time.perf_counter() - t0)
                    models[L][2], models[L][3] = logits, pos + 1
            per_tok = {L: statistics.median(ts[L]) for L in layers}
            if per_tok[layers[1]] > per_tok[layers[0]]:
                break
    finally:
        for m, *_ in models.values():
            m.close()
        models.clear()
    (l0, l1) = layers
    per_layer = (per_tok[l1] - per_tok[l0]) / (l1 - l0)
    note = ""
    if per_layer <= 0:             # unresolved: the larger model's time, all of it counted per layer
        per_layer = per_tok[l1] / l1
        note = f" (per-layer slope not resolved in {attempts} tries under host load: proportional estimate)"
    fixed = per_tok[l0] - l0 * per_layer if not note else 0.0
    t94 = fixed + base.n_layer * per_layer
    desc = (f"reference qms_forward ({ref.variant} build, {threads} OpenMP threads) on 235B-shape models of "
            f"{l0} and {l1} layers in host RAM, {prompt}-id prompt then {decode_tokens} decode tokens each (median): "
            f"{per_tok[l0] * 1e3:.1f} / {per_tok[l1] * 1e3:.1f} ms per token -> {per_layer * 1e3:.2f} ms per layer, "
            f"{fixed * 1e3:.1f} ms head + embedding; 94 layers: {t94 * 1e3:.1f} ms per token "
            f"(attention at position ~{prompt}, the device run decodes at ~{MODEL_PROMPT}){note}")
    return t94, desc, threads


def run_model_reference_arm(a):
    """--impl reference for the model metric: the reference's qms_forward on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    t94, desc, threads = cpu_model_sample(decode_tokens=max(8, a.steps))
    value = 1.0 / t94
    batch = a.mode == "model-bs64"
    if batch:     # one sequence at a time (src/model.h:116-118): B sequences take B x the bs1 time
        desc += f"; {a.batch} sequences served one after another: the same tok/s"
    line = {"impl": "reference", "metric": BATCH_METRIC if batch else MODEL_METRIC, "value": round(value, 4), "unit": "tok/s",
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t94 * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32",
            "data": "synthetic",
            "config": {"workload": f"Qwen3-235B-A22B decode, {'%d sequences' % a.batch if batch else 'batch 1'} "
                                   "(config 4); reference arm: each step one decode token on each sampled model",
                       "sample": desc,
                       "wall_s": round(time.perf_counter() - t0, 1)},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "reference",
                             "sample": desc},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_model(a):
    import torch
    import large_model_b200 as q
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    q.init(local)
    dev = torch.device("cuda", local)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:            # before the GPU model takes host time
        t94, desc, threads = cpu_model_sample()
        cpu = {"value": round(1.0 / t94, 4), "unit": "tok/s", "cores": threads, "kind": "reference", "sample": desc}
    cfg = model_cfg(a.model_layers)
    t_build = time.perf_counter()
    m = device_model(q, torch, cfg, 4242 + rank, dev, MODEL_CTX)
    if a.kv == "f16":
        m.set_kv_type(q.T_F16)
    t_build = time.perf_counter() - t_build
    rng = np.random.default_rng(99 + rank)
    prompt = [int(v) for v in rng.integers(0, cfg.vocab, MODEL_PROMPT)]
    t_pre = time.perf_counter()
    logits = m.forward(prompt, 0)
    t_pre = time.perf_counter() - t_pre
    room = MODEL_CTX - MODEL_PROMPT - 64                     # positions left for decode (the last 64 for the
    per_step = max(1, min(TOKENS_PER_STEP, room // (a.steps + a.warmup + 1)))   # section timers and e2e)
    stream = torch.cuda.Stream(device=dev)
    tok = torch.tensor([int(np.argmax(logits))], dtype=torch.int32, device=dev)
    pos = torch.tensor([MODEL_PROMPT], dtype=torch.int32, device=dev)
    lg = torch.empty(cfg.vocab, dtype=torch.float32, device=dev)
    with torch.cuda.stream(stream):
        m.decode_step(tok, pos, lg, stream=stream)            # outside capture: first-use setup
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(per_step):
                m.decode_step(tok, pos, lg, stream=stream)
        for _ in range(a.warmup):
            graph.replay()
    torch.cuda.synchronize()
    pos0 = int(pos.item())
    sampler = ClockSampler(local)
    time.sleep(0.5)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile_region = os.environ.get("QMS_PROFILE_REGION") == "1"   # ncu --profile-from-start off: the timed steps only
    if profile_region:
        torch.cuda.profiler.start()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(a.steps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if profile_region:
        torch.cuda.profiler.stop()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    pos1 = int(pos.item())
    m.status()
    ntok = a.steps * per_step
    tok_s = ntok * world / (ms / 1e3)
    bt = model_bytes_per_token(cfg, (pos0 + pos1) / 2, 2 if a.kv == "f16" else 4)
    step_gbs = bt["total"] * ntok / (ms / 1e3) / 1e9
    # section times per token (CUDA events around each section of a token step; they serialise the
    # programmatic overlap between kernels, so their sum is a little above the graph's time per token)
    m.profile(True)
    nprof = 8 if int(pos.item()) + 40 < MODEL_CTX else 1
    for k in range(nprof):
        lp = m.forward([int(tok.item())], int(pos.item()))
        tok.fill_(int(np.argmax(lp)))
        pos.add_(1)
    sec = [v / nprof for v in m.profile(False)]
    names = ["qkv", "attn", "o_proj", "router", "fetch", "moe", "output"]
    moe_us_layer = sec[5] * 1e3 / cfg.n_layer
    moe_gbs = bytes_per_token_layer() / (moe_us_layer / 1e6) / 1e9
    # end to end through the host-buffer entry point: ids in, every token's logits out (as
    # main.c's decode loop does: it reads the logits on the host, src/main.c:198-207)
    e2e_n = max(1, min(24, MODEL_CTX - int(pos.item()) - 2))
    lp = m.forward([int(tok.item())], int(pos.item()))
    p_e = int(pos.item()) + 1
    nxt = int(np.argmax(lp))
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(e2e_n):
        lp = m.forward([nxt], p_e + k)
        nxt = int(np.argmax(lp))
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    peak, peak_kind = peaks()
    if rank == 0:
        line = {
            "metric": MODEL_METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
            "config": {"workload": f"Qwen3-235B-A22B (config 4) decode batch 1: {cfg.n_layer} layers, 128 experts top-8, Q4_0 "
                                   "weights + Q6_K head drawn on the device (seeded torch RNG), fp32 KV ctx 4096, "
                                   f"{MODEL_PROMPT}-id random prompt prefilled; a step = {per_step} greedy "
                                   f"decode tokens (qms_cuda_decode_step x{per_step} in one CUDA graph)",
                       "tokens_per_step": per_step, "positions": [pos0, pos1],
                       "kv_cache": "fp16 (compacted)" if a.kv == "f16" else "fp32 (the reference's)",
                       "ms_per_token": round(ms / ntok, 4), "device_gb": round(m.device_bytes / 1e9, 2),
                       "build_s": round(t_build, 1), "prefill_s": round(t_pre, 2),
                       "bytes_per_token": {k: int(v) for k, v in bt.items()},
                       "section_ms_per_token": {n: round(v, 4) for n, v in zip(names, sec)},
                       "moe_layer": {"us": round(moe_us_layer, 2), "gbs": round(moe_gbs, 1),
                                     "note": "ffn RMSNorm + k_decode_bs1 per layer, from the section timers"},
                       "l2": "inputs far larger than L2 (124 GiB of weights)",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (embedding, per layer QKV / RoPE+KV / attention "
                                                   "/ O / RMSNorm / MoE, head + argmax)",
                         "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(step_gbs / peak, 4),
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": None,
                         "dominant_kernel": {"name": "k_decode_bs1 (MoE block)", "us_per_launch": round(moe_us_layer, 2),
                                             "achieved": round(moe_gbs, 1), "frac": round(moe_gbs / peak, 4),
                                             "bytes_per_launch": bytes_per_token_layer(),
                                             "share_of_step": round(sec[5] / max(1e-9, sum(sec)), 3)}},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_n * world / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": cfg.vocab * 4,
                    "note": "qms_cuda_forward per token (host id in, the token's 151936 logits to host memory, "
                            "argmax on the host), per token; h2d/d2h bytes are per token"},
            # per token: the embedding gather, per layer QKV / attention / merge / O / MoE, the head
            "gpu_launches": ntok * (2 + 5 * cfg.n_layer),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del graph
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def batch_bytes_per_step(cfg, B: int, pos: float, kv_es: int = 4) -> dict:
    """Algorithmic bytes of one batched decode step: each expert the step selects once (its expected
    count for B tokens x top-8 of 128 under uniform routing), router, attention weights, each
    sequence's KV rows, norms, the head and B embedding rows."""
    ex = cfg.n_expert * (1.0 - (1.0 - cfg.n_used / cfg.n_expert) ** B)
    per = model_bytes_per_token(cfg, pos, kv_es)
    moe = cfg.n_layer * (ex * 3 * cfg.n_ff * cfg.n_embd * 18 // 32 + cfg.n_expert * cfg.n_embd * 4)
    d = {"moe": moe, "attention_weights": per["attention_weights"], "kv_cache": B * per["kv_cache"],
         "norms": per["norms"], "head": per["head"], "embedding_rows": B * per["embedding_row"]}
    d["total"] = sum(d.values())
    d["distinct_experts_per_layer"] = ex
    return d


def run_model_batch(a):
    """--mode model-bs64: B sequences decoded together, one token each per step (qms_cuda_decode_batch
    in a CUDA graph). Each sequence's 1024-id prompt is a shared 896-id prefix (prefilled once and
    copied into every sequence's cache) followed by 128 ids of its own (prefilled per sequence), so
    the sequences' hidden states, and their experts, differ as independent prompts' do."""
    import torch
    import large_model_b200 as q
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    q.init(local)
    dev = torch.device("cuda", local)
    B = a.batch
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        t94, desc, threads = cpu_model_sample()
        cpu = {"value": round(1.0 / t94, 4), "unit": "tok/s", "cores": threads, "kind": "reference",
               "sample": desc + "; the reference serves one sequence at a time (src/model.h:116-118), so B "
                                "sequences take B x its bs1 time: the same tok/s"}
    cfg = model_cfg(a.model_layers)
    assert a.steps + a.warmup + 8 < BATCH_CTX - MODEL_PROMPT, "steps beyond the sequences' context"
    t_build = time.perf_counter()
    m = device_model(q, torch, cfg, 4242 + rank, dev, BATCH_CTX)
    if a.kv == "f16":
        m.set_kv_type(q.T_F16)
    m.set_sequences(B)
    t_build = time.perf_counter() - t_build
    rng = np.random.default_rng(99 + rank)
    shared = MODEL_PROMPT - BATCH_OWN
    prefix = [int(v) for v in rng.integers(0, cfg.vocab, shared)]
    t_pre = time.perf_counter()
    m.forward(prefix, 0, seq=0)
    first = []
    for b in range(B):
        if b:
            m.copy_sequence(0, b, shared)
        own = [int(v) for v in rng.integers(0, cfg.vocab, BATCH_OWN)]
        first.append(int(np.argmax(m.forward(own, shared, seq=b))))
    t_pre = time.perf_counter() - t_pre
    stream = torch.cuda.Stream(device=dev)
    tok = torch.tensor(first, dtype=torch.int32, device=dev)
    pos = torch.full((B,), MODEL_PROMPT, dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        m.decode_batch(tok, pos, stream=stream)              # outside capture: first-use setup
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            m.decode_batch(tok, pos, stream=stream)
        for _ in range(a.warmup):
            graph.replay()
    torch.cuda.synchronize()
    pos0 = int(pos[0].item())
    sampler = ClockSampler(local)
    time.sleep(0.5)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile_region = os.environ.get("QMS_PROFILE_REGION") == "1"   # ncu --profile-from-start off: the timed steps only
    if profile_region:
        torch.cuda.profiler.start()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(a.steps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if profile_region:
        torch.cuda.profiler.stop()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    pos1 = int(pos[0].item())
    m.status()
    distinct = len(set(tok.tolist()))
    tok_s = B * a.steps * world / (ms / 1e3)
    # section times of one step (CUDA events between sections, which serialise the overlap)
    m.profile(True)
    m.forward_batch(tok.cpu().numpy(), pos.cpu().numpy())
    sec = m.profile(False)
    names = ["qkv", "attn", "o_proj", "router", "fetch", "moe", "output"]
    bt = batch_bytes_per_step(cfg, B, (pos0 + pos1) / 2, 2 if a.kv == "f16" else 4)
    step_gbs = bt["total"] * a.steps / (ms / 1e3) / 1e9
    # end to end through the host-buffer entry point: B ids and positions in, B rows of logits out,
    # the argmax of each row on the host
    e2e_n = 3
    ids = tok.cpu().numpy()
    p_e = pos.cpu().numpy()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(e2e_n):
        lg = m.forward_batch(ids, p_e)
        ids = lg.argmax(axis=1).astype(np.int32)
        p_e = p_e + 1
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    peak, peak_kind = peaks()
    if rank == 0:
        line = {
            "metric": BATCH_METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
            "config": {"workload": f"Qwen3-235B-A22B (config 4) decode, {B} sequences: {cfg.n_layer} layers, Q4_0 weights + "
                                   "Q6_K head drawn on the device (seeded torch RNG), fp32 KV caches of "
                                   f"{BATCH_CTX} positions each; a {MODEL_PROMPT}-id random prompt prefilled "
                                   f"once and copied to every sequence, {B} random next tokens; a step = one "
                                   f"token for each sequence (qms_cuda_decode_batch in one CUDA graph)",
                       "sequences": B, "positions": [pos0, pos1], "distinct_tokens_last_step": distinct,
                       "kv_cache": "fp16 (compacted)" if a.kv == "f16" else "fp32 (the reference's)",
                       "ms_per_token_per_sequence": round(ms / a.steps, 3), "device_gb": round(m.device_bytes / 1e9, 2),
                       "build_s": round(t_build, 1), "prefill_and_copy_s": round(t_pre, 2),
                       "section_ms_per_step": {n: round(v, 3) for n, v in zip(names, sec)},
                       "bytes_per_step": {k: (round(v, 1) if isinstance(v, float) else int(v)) for k, v in bt.items()},
                       "l2": "inputs far larger than L2 (124 GiB of weights)",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "kernel": "whole batched decode step (per layer RMSNorm / QKV / RoPE+KV / "
                                                   "attention / O / MoE grouped GEMV, head + per-row argmax)",
                         "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(step_gbs / peak, 4),
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "traffic": None},
            "cpu_baseline": cpu,
            "e2e": {"value": round(B * e2e_n * world / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8 * B,
                    "d2h_bytes_per_step": B * cfg.vocab * 4,
                    "note": "qms_cuda_forward_batch per step (host ids and positions in, every sequence's 151936 "
                            "logits to host memory, argmax per row on the host)"},
            # per step: the embedding; per layer RMSNorm, QKV, attention, merge (Q8 out), O, RMSNorm
            # and the 7 kernels of the batched MoE block (router, top-k, Q8 rows, grouping, gate/up,
            # down, combine); the head's RMSNorm, the head and the per-row argmax (the launch list in
            # profiles/launches_decode_step_235b_bs64.md counts the same 1226)
            "gpu_launches": a.steps * (1 + 13 * cfg.n_layer + 3),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del graph
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--mode", default="model", choices=["model", "model-bs64", "moe", "bs64", "prefill"])
    ap.add_argument("--batch", type=int, default=BATCH_SEQS, help="sequences in --mode model-bs64")
    ap.add_argument("--model-layers", type=int, default=0,
                    help="model modes: keep only this many layers (small cases for profiling; not a bench line)")
    ap.add_argument("--kv", default="f32", choices=["f32", "f16"],
                    help="model modes: KV cache elements (f16: the compacted cache, not the reference's arithmetic)")
    ap.add_argument("--ep", action="store_true", help="batched modes under torchrun: shard the experts over the ranks")
    ap.add_argument("--zipf", type=float, default=0.0,
                    help="batched modes: Zipf(s) expert popularity (config 5: --mode prefill --zipf 1.1)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    if a.impl == "reference":
        return run_model_reference_arm(a) if a.mode in ("model", "model-bs64") else run_reference_arm(a)
    if a.mode == "model":
        return run_model(a)
    if a.mode == "model-bs64":
        return run_model_batch(a)
    if a.mode != "moe":
        return run_batched(a)

    import torch
    import large_model_b200 as q

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    q.init(local)
    dev = torch.device("cuda", local)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        cpu, _, _ = cpu_reference_rate()

    layers = [device_layer(q, torch, 100 + 17 * i, dev) for i in range(a.layers)]
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    E = layers[0].n_embd
    xn = torch.randn((a.tokens, E), generator=g, device=dev, dtype=torch.float32)
    out = torch.empty_like(xn)
    for m in layers:
        m.reserve(1)
    stream = torch.cuda.Stream(device=dev)

    def step():
        for t in range(a.tokens):
            layers[t % a.layers].forward(xn[t:t + 1], out=out[t:t + 1], stream=stream)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    graph = None
    if not a.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step

    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            run()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    time.sleep(0.6)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(a.steps):
            run()
        ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens_total = a.steps * a.tokens * world
    value = tokens_total * bytes_per_token_layer() / (ms / 1e3) / 1e9

    # per-kernel timing pass (CUDA events around each kernel on the launch stream)
    kev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ksum = [0.0, 0.0, 0.0]
    nk = min(200, a.tokens)
    for t in range(nk):
        m = layers[t % a.layers]
        m.set_kernel_events(kev)
        with torch.cuda.stream(stream):
            m.forward(xn[t:t + 1], out=out[t:t + 1], stream=stream)
        m.set_kernel_events(None)
        stream.synchronize()
        for i in range(3):
            ksum[i] += kev[2 * i].elapsed_time(kev[2 * i + 1])
    kms = [s / nk for s in ksum]
    peak, peak_kind = peaks()
    kern_gbs = bytes_per_launch() / (kms[1] / 1e3) / 1e9

    # end to end through the host-buffer entry point (pinned host memory, copies in the timed region)
    xh = torch.empty((a.tokens, E), dtype=torch.float32, pin_memory=True)
    xh.copy_(xn.cpu())
    oh = torch.empty_like(xh, pin_memory=True)
    xh_np, oh_np = xh.numpy(), oh.numpy()
    e2e_steps = max(1, min(a.steps, 3))
    for t in range(min(50, a.tokens)):
        layers[t % a.layers].forward_host(xh_np[t:t + 1], out=oh_np[t:t + 1])
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for t in range(a.tokens):
            layers[t % a.layers].forward_host(xh_np[t:t + 1], out=oh_np[t:t + 1])
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = e2e_steps * a.tokens * world * bytes_per_token_layer() / e2e_s / 1e9

    if rank == 0:
        traffic = profile_traffic()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens_per_step": a.tokens, "layers": a.layers,
                       "bytes_per_token_layer": bytes_per_token_layer(),
                       "token_layers_per_s": round(tokens_total / (ms / 1e3), 1),
                       "moe_only_decode_tok_s_94_layers": round(tokens_total / (ms / 1e3) / 94, 2),
                       "us_per_token_layer": round(ms * 1e3 / (a.steps * a.tokens), 3),
                       "l2": f"inputs larger than L2 ({a.layers} layers x 1.36 GB resident)",
                       "graph": graph is not None, "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "kernel": "k_decode_bs1", "achieved": round(kern_gbs, 1), "peak": peak,
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback", "unit": "GB/s", "frac": round(kern_gbs / peak, 4),
                         "traffic": traffic, "bytes_per_launch": bytes_per_launch(),
                         "kernel_us": {"k_decode_bs1": round(kms[1] * 1e3, 2)},
                         "timing": "launch alone, CUDA events on its stream (no overlap with the previous call)",
                         "op_frac": round(value / world / peak, 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": a.tokens * E * 4,
                    "d2h_bytes_per_step": a.tokens * E * 4,
                    "note": "qms_cuda_moe_forward_host per token: copy in, 1 kernel, copy out, wait"},
            "gpu_launches": a.tokens * a.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del graph
    for m in layers:
        m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
