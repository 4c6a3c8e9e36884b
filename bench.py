"""Benchmark of the Qwen3-MoE feed-forward hot path on B200 (libqms_cuda through its C ABI).

Workload: the Qwen3-235B-A22B MoE layer operator at decode batch 1 —
hidden 4096, 128 experts, top-8, moe_intermediate 1536, Q4_0 experts, F32 router — on 1000
seeded tokens, each an independent T=1 call. Calls cycle through 8 resident layers with
independent seeded weights (8 x 1.36 GB), so consecutive calls share no weights and every
step's inputs are far larger than L2. A step is the 1000 calls; the metric is the MoE layer's
algorithmic HBM bytes (8 experts x 10,616,832 B + 2,097,152 B router = 87,031,808 B per
token-layer) divided by time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

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


def cpu_reference_batched(T: int, seconds: float = 10.0, layers: int = 2):
    """The reference's moe() on T-token calls (moe() is sequence-agnostic), all host threads."""
    from oracle import Reference, host_threads
    from large_model_b200 import synth
    ref = Reference()
    threads = host_threads()
    ref.set_threads(threads)
    ls = [synth.make_moe_layer(SHAPE, seed=1000 + i) for i in range(layers)]
    xn = synth.make_hidden(ls[0].n_embd, T, seed=2001)
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

def device_layer(q, torch, seed: int, device, shard=None):
    """A 235B-shape layer drawn on the device with the config's distributions, then uploaded
    through qms_cuda_moe_create from device memory (GGUF layout, repacked by the library).
    shard = (expert_base, n_local): only those experts (an expert-parallel shard)."""
    from large_model_b200 import synth
    E, X, K, F = synth.MOE_SHAPES[SHAPE]
    XL = X if shard is None else shard[1]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    router = torch.randn((X, E), generator=g, device=device, dtype=torch.float32) * 0.02

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
        cpu = cpu_reference_batched(T, seconds=10.0 if T <= 256 else 20.0)
    ep = a.ep and world > 1
    if ep:                                            # expert parallelism: X / world experts per rank
        from large_model_b200.ep import CudaBackend, ExpertParallelMoe
        per = X // world
        layers = [device_layer(q, torch, 500 + 17 * i, dev, shard=(rank * per, per)) for i in range(2)]
        eps = [ExpertParallelMoe(CudaBackend(m), X, K, E) for m in layers]
    else:
        layers = [device_layer(q, torch, 500 + 17 * i, dev) for i in range(2)]
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)                          # every rank its own tokens
    xs = [torch.randn((T, E), generator=g, device=dev, dtype=torch.float32) for _ in range(2)]
    out = torch.empty((T, E), device=dev, dtype=torch.float32)
    for m in layers:
        m.reserve(T)
    calls = 8 if T <= 256 else 2
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
    gemv = T * K <= 24 * (X // world if ep else X)
    per_call = (10 if gemv else 11) if ep else (7 if gemv else 9)
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
            roof = {"bound": "tensor", "kernel": "whole block (router, k_mma_group, gathers, k_mma_gemm x2, combine)",
                    "achieved": round(tops, 1), "peak": 4500.0 * world, "unit": "TOP/s",
                    "frac": round(tops / (4500.0 * world), 4),
                    "peak_kind": "nominal dense int8 (no measured int8 peak on this pool)", "traffic": None,
                    "ops_per_call": ops}
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
                           "routing": "seeded N(0,1) hidden states, N(0,0.02) router (near-uniform expert load)",
                           "parallelism": f"expert-parallel x{world} (NCCL all-to-all)" if ep else f"replicas x{world}"},
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
    ap.add_argument("--mode", default="decode", choices=["decode", "bs64", "prefill"])
    ap.add_argument("--ep", action="store_true", help="batched modes under torchrun: shard the experts over the ranks")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    if a.impl == "reference":
        return run_reference_arm(a)
    if a.mode != "decode":
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
