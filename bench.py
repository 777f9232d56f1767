"""Benchmark: mixed-tier paged decode attention, KV tokens/s and HBM GB/s against the roofline.

Workload (one decode step = one attention pass over the whole cache of one layer):
Llama-3-8B-shaped layer, batch 8 per GPU, 32 query heads, 8 KV heads, head_dim 128, context
32,768 tokens in 16-token pages, tiers by age (newest to oldest): FP16 1024 tokens, simulated-FP8
3072, INT8 4096, INT4 8192, INT2 8192, 1-bit 8192.  K/V are seeded N(0,1) fp16 quantized by the
tier codecs; queries N(0,1)/sqrt(128); softmax scale 1/sqrt(128).  The compressed cache is
280.8 MB per GPU, larger than the 126 MB L2, so every step streams it from HBM.

Multi-GPU: one process per GPU (torchrun), the layer sharded by KV head.  The batch grows with the
ranks (8 x N sequences) and rank r holds KV heads [8r/N, 8(r+1)/N) of every sequence and page, so
each GPU streams the same 280.8 MB per step ("weak" scaling); a step is the attention over the
rank's heads with the all-gather of the per-head outputs into [8N, 32, 1, 128] fused in
(sharding.FusedHeadShardedDecode: the kernel writes its output rows straight into every rank's
output buffer in peer memory, and a one-thread wait kernel completes the step).  The NCCL path
(kernel, all_gather_into_tensor, head-order copy; sharding.HeadShardedDecode) is timed beside it.
`value` is the whole-job KV tokens/s (8N x 32768 / max-over-ranks step time).  At N = 1 there is
nothing to gather and the step is the kernel alone.

Timing: W untimed steps, then windows of exactly K steps (CUDA events on the launching stream,
barrier + synchronize around each) repeated until at least one second of device time has passed,
so the clock sampler sees the kernel under load; the reported step time is the median window.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Further workloads (not the headline line) are measured by the same script:

    python bench.py --workload jl-archive          # attention over the JL archive: B 4, H_q 32,
                                                   # H_kv 8, D 128, 64 blocks of 1024 tokens -> 128 rows
    torchrun --nproc-per-node N bench.py --workload llama3-70b --gpus N   (or N = 1 without torchrun)
                                                   # Llama-3-70B layer: B 64, H_q 64, H_kv 8, context
                                                   # 131072 (the 8B tier ratios x4), KV-head sharded over
                                                   # N GPUs; each rank's 1-bit share (oldest 25%) in
                                                   # pinned host memory, streamed under the resident tiers
    python bench.py --workload tinyllama-sidecars  # TinyLlama-shaped layer: H_q 32, H_kv 4, D 64, 4096
                                                   # tokens, 3840 in INT8 pages with outlier sidecars
    python bench.py --workload llama3-8b-sidecars  # the Llama-3-8B layer with sigma-3 outlier sidecars on
                                                   # every quantized page, with and without the corrections
    python bench.py --workload cascade             # pack/unpack of every tier, 1M tokens x 8 heads x 128

--impl reference times the CPU restatement of the reference's path (dequantize every page, then
softmax attention over the reconstructed K/V; argus_cache core/memory_manager.py:1157-1315 +
1424-1430) on the host cores, on a bounded sample (as many of the sequences as fit about 2.5 minutes, all KV
heads, full context).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "argus-anchored-random-geometric-unbiased-storage_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode-attn KV tokens/s/GPU & HBM GB/s vs roofline (mixed tiers), 1/2/4/8 B200"
UNIT = "KV tokens/s"
B, HQ, HKV, D, P = 8, 32, 8, 128, 16
L = 32768
SPLIT = [("one_bit", 8192), ("int2", 8192), ("int4", 8192), ("int8", 4096), ("fp8", 3072), ("fp16", 1024)]
WORKLOAD = "llama3-8b-layer-mixed-tier-decode"


def config(world):
    par = "single GPU" if world == 1 else f"kv-head sharded x{world} ({HKV // world} KV heads per GPU), NCCL all-gather of outputs"
    return {"workload": WORKLOAD, "global_batch": B * world, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
            "context": L, "page_size": P, "tiers_oldest_first": dict(SPLIT),
            "bytes_per_gpu": "280.8 MB compressed (8 sequences x 8 KV heads' worth)",
            "l2": "inputs larger than L2 (280.8 MB compressed per GPU vs 126 MB L2), no flush",
            "parallelism": par}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_from_profile():
    """DRAM bytes per launch of the decode kernel from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "decode_attention_llama8b.json")
    try:
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


# ------------------------------------------------------------------------------ workload
def build_cache(device, seed, batch=None, heads_kv=None, sample=None):
    """The tiered cache of `batch` sequences x `heads_kv` KV heads (default: the module's B, HKV),
    quantized on the device by the tier codecs, its AttentionPlan, and N(0,1)/sqrt(D) queries for
    the group of query heads of those KV heads.  With `sample` (a list of (b, h) pairs) also returns
    host copies of those pairs' fp16 K/V before quantization: {tier: (k, v)} of [pages, P, D] each."""
    import torch

    from argus_b200 import attention as A
    from argus_b200.core import quantization as Q

    Bc = B if batch is None else batch
    Hc = HKV if heads_kv is None else heads_kv
    g = torch.Generator(device=device).manual_seed(seed)
    arenas, pages, src = [], [], {}
    for tier, ntok in SPLIT:
        n = ntok // P
        k = torch.randn(n, Bc, Hc, P, D, device=device, generator=g).half()
        v = torch.randn(n, Bc, Hc, P, D, device=device, generator=g).half()
        if sample is not None:
            src[tier] = {bh: (k[:, bh[0], bh[1]].cpu().numpy(), v[:, bh[0], bh[1]].cpu().numpy()) for bh in sample}
        a = A.KVArena.allocate(A.TIER_NAMES[tier], Bc, Hc, n, P, D, device)
        if tier == "fp16":
            a.write_pages(0, k, v)
        elif tier in ("int8", "fp8", "e4m3"):
            f = {"int8": Q.quantize_to_int8, "fp8": Q.quantize_to_fp8_simulated, "e4m3": Q.quantize_to_e4m3}[tier]
            (kq, ks), (vq, vs) = f(k), f(v)
            a.write_pages(0, kq, vq, ks, vs)
        elif tier in ("int4", "int2"):
            f = Q.quantize_to_int4_packed if tier == "int4" else Q.quantize_to_int2_packed
            (kp, ks, km), (vp, vs, vm) = f(k), f(v)
            a.write_pages(0, kp, vp, ks, vs, km, vm)
        else:
            (kp, ks), (vp, vs) = Q.quantize_to_1bit_packed(k), Q.quantize_to_1bit_packed(v)
            a.write_pages(0, kp, vp, ks, vs)
        del k, v
        ai = len(arenas)
        arenas.append(a)
        pages += [(ai, j, P) for j in range(n)]
    torch.cuda.synchronize(device)
    plan = A.AttentionPlan(arenas, pages, batch=Bc, heads_kv=Hc, group=HQ // HKV, head_dim=D)
    q = (torch.randn(Bc, Hc * (HQ // HKV), 1, D, device=device, generator=g) / math.sqrt(D)).half()
    return (plan, q, src) if sample is not None else (plan, q)


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.25)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) > 8 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


# ----------------------------------------------------------------------- CPU reference arm
def cpu_reference_step(pages_np, q_np, threads):
    """One sequence of the workload through the CPU restatement of the reference's path: every
    page dequantized (oracle, bit-exact with the reference's codecs), then softmax attention over
    the reconstructed K/V per GQA group."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np
    import torch

    import oracle

    def deq(item):
        tier, pg = item
        return oracle.page_kv(tier, pg)

    with ThreadPoolExecutor(max_workers=threads) as ex:
        kv = list(ex.map(deq, pages_np))
    K = torch.from_numpy(np.concatenate([k for k, _ in kv], axis=2)).float()
    V = torch.from_numpy(np.concatenate([v for _, v in kv], axis=2)).float()
    q = torch.from_numpy(q_np).float()  # [1, HQ, 1, D]
    g = HQ // HKV
    qg = q.view(1, HKV, g, D)
    w = torch.matmul(qg, K.transpose(-1, -2)) / math.sqrt(D)
    p = torch.softmax(w, dim=-1)
    return torch.matmul(p, V)


def cpu_sample(seed=0):
    """Host copies of one sequence's pages (b = 0, all KV heads, full context)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(seed)
    pages = []
    for tier, ntok in SPLIT:
        for _ in range(ntok // P):
            k = rng.standard_normal((1, HKV, P, D), dtype=np.float32).astype(np.float16)
            v = rng.standard_normal((1, HKV, P, D), dtype=np.float32).astype(np.float16)
            if tier == "fp16":
                pg = {"key": k, "value": v}
            elif tier in ("fp8", "int8"):
                f = oracle.quantize_to_int8 if tier == "int8" else oracle.quantize_to_fp8_simulated
                pg = dict(zip(("key_q", "key_scales"), f(k)))
                pg.update(zip(("value_q", "value_scales"), f(v)))
            elif tier in ("int4", "int2"):
                f = oracle.quantize_to_int4_packed if tier == "int4" else oracle.quantize_to_int2_packed
                pg = dict(zip(("key_packed", "key_scales", "key_min"), f(k)))
                pg.update(zip(("value_packed", "value_scales", "value_min"), f(v)))
            else:
                pg = dict(zip(("key_packed", "key_scales"), oracle.quantize_to_1bit_packed(k)))
                pg.update(zip(("value_packed", "value_scales"), oracle.quantize_to_1bit_packed(v)))
            pages.append((tier, pg))
    q = (rng.standard_normal((1, HQ, 1, D)) / math.sqrt(D)).astype(np.float16)
    return pages, q


CPU_PORT_SCOPE = ("the oracle port of the reference's reconstruct-then-attend path: every page dequantized with the "
                  "reference's codecs bit for bit (C), concatenated, then fp32 torch softmax attention per GQA group; "
                  "it leaves out the reference's per-page Python dict walk, prefetch-cache lookups, per-page .item() "
                  "syncs and importance/resurrection bookkeeping, so the reference itself is slower")


def time_cpu(steps, warmup, threads, min_seconds=0.0, nseq=1):
    """Seconds per step of the CPU path over `nseq` distinct sequences per step; runs at least
    `steps` steps and at least `min_seconds`.  Returns (KV tokens/s, seconds per step, steps run)."""
    import torch

    torch.set_num_threads(threads)
    samples = [cpu_sample(seed) for seed in range(nseq)]

    def step():
        for pages, q in samples:
            cpu_reference_step(pages, q, threads)

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    n = 0
    while n < steps or time.perf_counter() - t0 < min_seconds:
        step()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return nseq * L / dt, dt, n


def cpu_baselines(min_seconds=10.0):
    """The cpu_baseline object: the oracle port on all host threads (one sequence per step for at
    least min_seconds) and on one thread (at least one step)."""
    threads = os.cpu_count() or 1
    value, dt, n = time_cpu(3, 1, threads, min_seconds=min_seconds)
    v1, dt1, n1 = time_cpu(1, 0, 1, min_seconds=min_seconds / 2)
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"1 sequence x {HKV} KV heads x {L} tokens per step (one of the {B} sequences of a GPU's share), "
                      f"{n} timed steps ({n * dt:.1f} s of CPU work) on {threads} threads",
            "one_thread": {"value": v1, "unit": UNIT, "cores": 1, "steps": n1, "seconds": round(n1 * dt1, 1)},
            "scope": CPU_PORT_SCOPE}


def run_reference(args, rank):
    """The reference arm: the CPU path on all host threads, rank 0 only.  Each step attends as many
    of the workload's 8 sequences (all KV heads, full context) as keep the whole run within about
    two and a half minutes."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    _, t_seq, _ = time_cpu(1, 0, threads)
    nseq = int(max(1, min(B, 150.0 / max(1e-3, (args.steps + args.warmup) * t_seq))))
    value, dt, _ = time_cpu(args.steps, args.warmup, threads, nseq=nseq)
    sample = (f"{nseq} of the {B} sequences of the workload x {HKV} KV heads x {L} tokens per step, "
              f"{threads} host threads")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": config(args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                             "scope": CPU_PORT_SCOPE},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- our arm
def _windows(fn, steps, world, device, min_seconds=1.0, max_windows=4000):
    """Device milliseconds per step of windows of exactly `steps` calls of fn, each window bracketed
    by a barrier and a synchronize on both sides and timed with CUDA events on the current stream,
    repeated until min_seconds of device time (every rank runs the same number of windows).
    Returns the per-window times, each the max over ranks."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier()

    def window():
        torch.cuda.synchronize(device)
        barrier()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        return e0.elapsed_time(e1) / steps

    first = window()
    t = torch.tensor([first], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    n = int(min(max_windows, max(1, math.ceil(min_seconds * 1e3 / max(1e-6, float(t.item()) * steps)))))
    ms = [first] + [window() for _ in range(n - 1)]
    t = torch.tensor(ms, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from argus_b200 import sharding

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if HKV % world:
        raise SystemExit(f"{HKV} KV heads do not split over {world} ranks")
    hl = HKV // world
    Bg = B * world  # global batch: every GPU holds B x HKV (batch, kv_head) pairs' worth of pages
    plan, _ = build_cache(device, seed=1234 + rank, batch=Bg, heads_kv=hl)
    gq = torch.Generator(device=device).manual_seed(99)  # the same queries on every rank
    q_full = (torch.randn(Bg, HQ, 1, D, device=device, generator=gq) / math.sqrt(D)).half()
    stream = torch.cuda.current_stream(device)
    if world > 1:
        # the product path: the all-gather runs inside the attention kernel (peer stores + arrival
        # counters); the NCCL path is timed beside it for comparison
        fused = sharding.FusedHeadShardedDecode(plan, HKV)
        step = lambda: fused(q_full)  # noqa: E731
        step_api = sharding.HeadShardedDecode(plan, HKV)
    else:
        step = lambda: plan.run(q_full)  # noqa: E731

    for _ in range(args.warmup):
        step()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    smi_index = vis.split(",")[local_rank] if vis else str(local_rank)
    with ClockSampler(smi_index) as clk:
        wins = _windows(step, args.steps, world, device, min_seconds=args.min_seconds)
    ms = statistics.median(wins)

    # per-step breakdown at N > 1: the plain kernel on this rank's heads (no gather) for the roofline,
    # the fused step's wait for the peers' rows, and the NCCL path (kernel, then all-gather and
    # head-order copy) for comparison, each from events in one window of K steps
    kernel_ms, gather_ms, nccl = ms, 0.0, None
    if world > 1:
        q_local = sharding.shard_queries(q_full, HKV, world, rank)
        kernel_ms = statistics.median(_windows(lambda: plan.run(q_local), args.steps, world, device,
                                               min_seconds=0.2))
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        torch.cuda.synchronize(device)
        dist.barrier()
        for e in evs:
            e[0].record(stream)
            fused.local(q_full)
            e[1].record(stream)
            fused.wait()
            e[2].record(stream)
        torch.cuda.synchronize(device)
        for _ in range(args.warmup):
            step_api(q_full)
        nccl_ms = statistics.median(_windows(lambda: step_api(q_full), args.steps, world, device, min_seconds=0.2))
        kg = torch.tensor([statistics.median([e[0].elapsed_time(e[1]) for e in evs]),
                           statistics.median([e[1].elapsed_time(e[2]) for e in evs]), nccl_ms], device=device)
        dist.all_reduce(kg, op=dist.ReduceOp.MAX)
        fused_kernel_ms, gather_ms, nccl_ms = kg.tolist()
        nccl = {"ms_per_step": nccl_ms, "value": Bg * L / (nccl_ms * 1e-3),
                "path": "HeadShardedDecode: kernel, NCCL all_gather_into_tensor in place, head-order copy"}

    # end-to-end through the public API: the full query batch from pinned host memory, the step,
    # the (gathered) output back to host, every step
    q_host = q_full.cpu().pin_memory()
    o_host = torch.empty_like(q_host).pin_memory()
    if world > 1:
        q_dev = torch.empty_like(q_full)

        def e2e_step():
            q_dev.copy_(q_host, non_blocking=True)
            o_host.copy_(fused(q_dev), non_blocking=True)
        e2e_path = ("FusedHeadShardedDecode: pinned host q in, attention with the all-gather fused in (peer "
                    "stores), gathered output out, every step")
    else:
        e2e_step = lambda: plan.run_host(q_host, o_host)  # noqa: E731
        e2e_path = "AttentionPlan.run_host: pinned host q in, fused kernel, output out, one CUDA graph per step"
    for _ in range(args.warmup):
        e2e_step()
    e2e_wins = _windows(e2e_step, args.steps, world, device, min_seconds=args.min_seconds / 4)
    e2e_ms = statistics.median(e2e_wins)
    if world > 1:
        fused.close()  # every rank: unmaps the peers' buffers (barriers inside)
    if rank != 0:
        return
    tokens = Bg * L
    hbm, peak_kind = peaks()
    achieved = plan.compressed_bytes / (kernel_ms * 1e-3) / 1e9
    line = {"metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic", "config": config(world),
            "timing": {"windows": len(wins), "steps_per_window": args.steps, "statistic": "median window",
                       "window_ms_per_step_min_max": [min(wins), max(wins)],
                       "timed_device_seconds": round(sum(wins) * args.steps / 1e3, 3)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_kind": peak_kind, "traffic": traffic_from_profile(),
                         "algorithmic_bytes_per_launch": plan.compressed_bytes,
                         "timed": "decode kernel (split-K combine fused), CUDA events"},
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": q_full.numel() * 2,
                    "d2h_bytes_per_step": q_full.numel() * 2, "path": e2e_path},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "splits": plan.n_splits}
    if world > 1:
        line["step_breakdown_ms"] = {"kernel_alone": kernel_ms, "fused_kernel": fused_kernel_ms,
                                     "wait_for_peers": gather_ms,
                                     "gather_bytes_per_rank": q_full.numel() * 2 // world,
                                     "limiting": "kernel" if kernel_ms >= 0.5 * ms else "gather"}
        line["nccl_all_gather_path"] = nccl
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baselines()
    print(json.dumps(line), flush=True)


def _timed(fn, steps, warmup):
    """Device time per call (ms) of `steps` back-to-back calls; a device-side sleep queued first keeps
    host launch overhead out of the measured span."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    torch.cuda._sleep(5_000_000)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_jl_archive(args):
    import torch

    from argus_b200.core import jl

    dev = torch.device("cuda", 0)
    Bj, HQj, HKVj, Dj, N, ratio, NB = 4, 32, 8, 128, 1024, 8, 64
    MJ = N // ratio
    g = torch.Generator(device=dev).manual_seed(4321)
    W = jl.projection_matrix(N, dtype=torch.float16, device="cpu", ratio=ratio)
    R = jl.reconstruction_operator_solve(W).half().to(dev)
    att = jl.JLAttention(R)
    yk = torch.randn(Bj, HKVj, NB, MJ, Dj, device=dev, generator=g).half()
    yv = torch.randn(Bj, HKVj, NB, MJ, Dj, device=dev, generator=g).half()
    q = (torch.randn(Bj, HQj, 1, Dj, device=dev, generator=g) / math.sqrt(Dj)).half()
    out = torch.empty_like(q)
    lse = torch.empty(Bj, HQj, 1, device=dev)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    with ClockSampler(vis.split(",")[0] if vis else "0") as clk:
        ms = _timed(lambda: att.run(q, yk, yv, out=out, lse=lse), args.steps, args.warmup)
    hbm, peak_kind = peaks()
    ybytes = 2 * yk.numel() * 2
    tokens = Bj * NB * N
    extra = {"clocks": clk.summary()}
    if not args.no_cpu_baseline:
        extra["cpu_baseline"] = _jl_cpu(R.cpu().numpy(), yk, yv, q, HQj // HKVj)
    print(json.dumps({"metric": "JL-archive decode attention, archived KV tokens/s", "value": tokens / (ms * 1e-3),
                      "unit": "KV tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": ms, "higher_is_better": True, "dtype": "fp16", "data": "synthetic",
                      "config": {"workload": "jl-archive", "batch": Bj, "q_heads": HQj, "kv_heads": HKVj,
                                 "head_dim": Dj, "blocks": NB, "block_tokens": N, "block_rows": MJ},
                      "roofline": {"bound": "hbm", "achieved": ybytes / (ms * 1e-3) / 1e9, "peak": hbm,
                                   "unit": "GB/s", "frac": ybytes / (ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind,
                                   "algorithmic_bytes_per_launch": ybytes}, **extra}), flush=True)


def _jl_cpu(R, yk, yv, q, G, min_seconds=10.0):
    """The reference's path for archived blocks on the host: every block rebuilt as K = R Yk,
    V = R Yv (the oracle's float64 product rounded to fp16), then softmax attention of the (b, kv
    head)'s G queries over all its rebuilt tokens; (b, kv head) pairs in turn until min_seconds."""
    import numpy as np

    import oracle

    Bj, Hk, NB, MJ, Dj = yk.shape
    N = R.shape[0]
    qn = q.float().cpu().numpy()
    scale = 1.0 / math.sqrt(Dj)
    pairs, t0 = 0, time.perf_counter()
    while True:
        b, h = divmod(pairs % (Bj * Hk), Hk)
        ykh = yk[b, h].cpu().numpy()
        yvh = yv[b, h].cpu().numpy()
        kv = [oracle.page_kv("jl", {"key_proj": ykh[j], "value_proj": yvh[j]}, R) for j in range(NB)]
        K = np.concatenate([k for k, _ in kv])
        V = np.concatenate([v for _, v in kv])
        oracle.sdpa_f64(qn[b:b + 1, h * G:(h + 1) * G], K[None, None], V[None, None], scale)
        pairs += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    tokens = pairs * NB * N / Hk  # a KV token covers all of a sequence's KV heads
    return {"value": tokens / dt, "unit": "KV tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{pairs} (batch, kv head) pairs of {NB} blocks x {N} tokens rebuilt and attended "
                      f"({dt:.1f} s)"}


def _tinyllama_pages(device, seed=0):
    """The TinyLlama-shaped layer: B 1, H_kv 4, D 64, 4096 tokens of N(0,1) K/V with 4 outlier
    channels per head scaled x8; the oldest 3840 tokens as 240 INT8 pages of 16 tokens whose
    outliers (sigma 3) are isolated into COO sidecars first, the newest 256 as FP16 pages."""
    import torch

    from argus_b200 import attention as A
    from argus_b200 import paged
    from argus_b200.core import quantization as Q
    from argus_b200.core.memory_manager import isolate_outliers

    Bt, HKVt, Dt, Pt, Lt, HOT = 1, 4, 64, 16, 4096, 256
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(Bt, HKVt, Lt, Dt, generator=g)
    v = torch.randn(Bt, HKVt, Lt, Dt, generator=g)
    for h in range(HKVt):
        ch = torch.randperm(Dt, generator=g)[:4]
        k[:, h, :, ch] *= 8.0
        v[:, h, :, ch] *= 8.0
    k_cpu, v_cpu = k.half(), v.half()
    k, v = k_cpu.to(device), v_cpu.to(device)
    ncold = (Lt - HOT) // Pt
    cold = A.KVArena.allocate(A.TIER_INT8, Bt, HKVt, ncold, Pt, Dt, device)
    hot = A.KVArena.allocate(A.TIER_FP16, Bt, HKVt, HOT // Pt, Pt, Dt, device)
    side = []
    entries = 0
    for j in range(ncold):
        kp, vp = k[:, :, j * Pt:(j + 1) * Pt], v[:, :, j * Pt:(j + 1) * Pt]
        kn, ko, km = isolate_outliers(kp, 3.0)
        vn, vo, vm = isolate_outliers(vp, 3.0)
        (kq, ks), (vq, vs) = Q.quantize_to_int8(kn), Q.quantize_to_int8(vn)
        cold.write_pages(j, kq[None], vq[None], ks[None], vs[None])
        ki, kv_ = paged.outliers_to_coo(km, ko)
        vi, vv_ = paged.outliers_to_coo(vm, vo)
        side.append((ki, kv_, vi, vv_))
        entries += ki.shape[0] + vi.shape[0]
    for j in range(HOT // Pt):
        t0 = Lt - HOT + j * Pt
        hot.write_pages(j, k[None, :, :, t0:t0 + Pt], v[None, :, :, t0:t0 + Pt])
    return cold, hot, side, entries, (Bt, HKVt, Dt, Pt, Lt), (k_cpu.numpy(), v_cpu.numpy())


def run_tinyllama_sidecars(args):
    import torch

    from argus_b200 import attention as A
    from argus_b200 import paged

    dev = torch.device("cuda", 0)
    cold, hot, side, entries, (Bt, HKVt, Dt, Pt, Lt), (k_np, v_np) = _tinyllama_pages(dev)
    HQt = 32
    blocks_bytes = 0
    for j, (ki, kv_, vi, vv_) in enumerate(side):
        paged.attach_outliers(cold, j, ki, kv_, vi, vv_)
        blocks_bytes += cold._outlier_blocks[j].numel()
    pages = [(0, j, Pt) for j in range(cold.slots)] + [(1, j, Pt) for j in range(hot.slots)]
    plan = A.AttentionPlan([cold, hot], pages, batch=Bt, heads_kv=HKVt, group=HQt // HKVt, head_dim=Dt)
    g = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(Bt, HQt, 1, Dt, device=dev, generator=g).half()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed_cold(fn, steps):
        """Median device time per call (ms) with L2 flushed before each call (the whole cache is
        2.4 MB, far below the 126 MB L2)."""
        ts = []
        for i in range(steps + args.warmup):
            flush.fill_(i & 0xff)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    ms = timed_cold(lambda: plan.run(q), args.steps)
    # the same pages without their corrections: the cost of the sidecars
    bare_cold = A.KVArena(cold.tier, cold.layout, cold.k, None, bh_stride=cold.bh_stride, record_bytes=cold.record_bytes,
                          page_tokens=Pt, head_dim=Dt, batch=Bt, heads=HKVt, slots=cold.slots)
    bare = A.AttentionPlan([bare_cold, hot], pages, batch=Bt, heads_kv=HKVt, group=HQt // HKVt, head_dim=Dt)
    ms_bare = timed_cold(lambda: bare.run(q), args.steps)
    hbm, peak_kind = peaks()
    nbytes = plan.compressed_bytes + blocks_bytes
    cpu = None
    if not args.no_cpu_baseline:
        cpu = _tinyllama_cpu(k_np, v_np, q.cpu().numpy(), Pt, HQt)
    print(json.dumps({"metric": "TinyLlama-shaped GQA decode attention, INT8 pages with outlier sidecars, KV tokens/s",
                      "value": Bt * Lt / (ms * 1e-3), "unit": "KV tokens/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "fp16",
                      "data": "synthetic",
                      "config": {"workload": "tinyllama-sidecars", "batch": Bt, "q_heads": HQt, "kv_heads": HKVt,
                                 "head_dim": Dt, "context": Lt, "page_size": Pt,
                                 "tiers_oldest_first": {"int8 (sidecars, sigma 3)": Lt - 256, "fp16": 256},
                                 "outlier_entries": entries, "l2": "flushed before every timed launch"},
                      "without_sidecars_ms": ms_bare,
                      "roofline": {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9, "peak": hbm,
                                   "unit": "GB/s", "frac": nbytes / (ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind,
                                   "algorithmic_bytes_per_launch": nbytes,
                                   "note": "2.4 MB per launch: latency-bound, far from any bandwidth roof"},
                      "cpu_baseline": cpu}),
          flush=True)


def _tinyllama_cpu(k, v, q, Pt, HQt, min_seconds=10.0):
    """The reference's path for the same layer on the host cores (oracle port, bit-exact codecs):
    every INT8 page dequantized and its sidecars scattered back, then softmax attention over the
    rebuilt K/V.  Pages are built once; each timed step rebuilds and attends."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np
    import torch

    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    Lt, HOT = k.shape[2], 256
    pages = []
    for j in range((Lt - HOT) // Pt):
        kp, vp = k[:, :, j * Pt:(j + 1) * Pt], v[:, :, j * Pt:(j + 1) * Pt]
        kn, ko, km = oracle.isolate_outliers(kp, 3.0)
        vn, vo, vm = oracle.isolate_outliers(vp, 3.0)
        pg = dict(zip(("key_q", "key_scales"), oracle.quantize_to_int8(kn)))
        pg.update(zip(("value_q", "value_scales"), oracle.quantize_to_int8(vn)))
        pg["key_out_indices"], pg["key_out_values"] = oracle.sidecar(km, ko)
        pg["value_out_indices"], pg["value_out_values"] = oracle.sidecar(vm, vo)
        pages.append(("int8", pg))
    for j in range(HOT // Pt):
        t0 = Lt - HOT + j * Pt
        pages.append(("fp16", {"key": k[:, :, t0:t0 + Pt], "value": v[:, :, t0:t0 + Pt]}))
    Hkv, D = k.shape[1], k.shape[3]

    def step():
        with ThreadPoolExecutor(max_workers=threads) as ex:
            kv = list(ex.map(lambda item: oracle.page_kv(*item), pages))
        K = torch.from_numpy(np.concatenate([a for a, _ in kv], axis=2)).float()
        V = torch.from_numpy(np.concatenate([b for _, b in kv], axis=2)).float()
        qg = torch.from_numpy(q).float().view(1, Hkv, HQt // Hkv, D)
        p = torch.softmax(torch.matmul(qg, K.transpose(-1, -2)) / math.sqrt(D), dim=-1)
        return torch.matmul(p, V)

    step()
    t0 = time.perf_counter()
    n = 0
    while n < 3 or time.perf_counter() - t0 < min_seconds:
        step()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": Lt / dt, "unit": "KV tokens/s", "cores": threads, "kind": "port",
            "sample": f"the whole layer per step (1 x {Hkv} KV heads x {Lt} tokens), {n} timed steps "
                      f"({n * dt:.1f} s of CPU work)"}


def run_tier_sweep(args):
    """The Llama-3-8B layer (B 8, 32 q / 8 KV heads, D 128) with every token in one tier, for each
    tier: 32K tokens (16K for fp16, which would not be a compressed layer), the fused kernel timed
    alone (no CPU leg); one JSON line per tier with its share of the HBM roof."""
    import torch

    global SPLIT
    dev = torch.device("cuda", 0)
    hbm, peak_kind = peaks()
    saved = SPLIT
    try:
        for tier in ("fp16", "fp8", "int8", "int4", "int2", "one_bit", "e4m3"):
            SPLIT = [(tier, 16384 if tier == "fp16" else 32768)]
            plan, q = build_cache(dev, seed=1234)
            for _ in range(args.warmup):
                plan.run(q)
            ms = statistics.median(_windows(lambda: plan.run(q), args.steps, 1, dev, min_seconds=args.min_seconds))
            tokens = B * HKV * SPLIT[0][1]
            gbs = plan.compressed_bytes / (ms * 1e-3) / 1e9
            print(json.dumps({"metric": "decode-attn KV tokens/s, one tier", "value": tokens / (ms * 1e-3),
                              "unit": "KV tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": ms, "higher_is_better": True, "dtype": "fp16", "data": "synthetic",
                              "config": {"workload": "tier-sweep", "tier": tier, "batch": B, "q_heads": HQ,
                                         "kv_heads": HKV, "head_dim": D, "context": SPLIT[0][1], "page_size": P},
                              "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                           "frac": gbs / hbm, "peak_kind": peak_kind,
                                           "algorithmic_bytes_per_launch": plan.compressed_bytes}}), flush=True)
            del plan, q
            torch.cuda.empty_cache()
    finally:
        SPLIT = saved


def run_8b_sidecars(args):
    """The Llama-3-8B mixed-tier layer (B 8, 32 q / 8 KV heads, D 128, 32K context, every tier) with
    the reference's outlier isolation (sigma 3, core/memory_manager.py:89-113) applied to every
    quantized page before it is quantized, its COO sidecars attached as correction blocks that the
    fused kernel applies while reading the pages compressed.  Timed with and without the
    corrections; bytes = compressed pages + correction blocks."""
    import torch

    from argus_b200 import attention as A
    from argus_b200 import paged
    from argus_b200.core.memory_manager import isolate_outliers

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1234)
    arenas, pages, entries, block_bytes = [], [], 0, 0
    for tier, ntok in SPLIT:
        n = ntok // P
        k = torch.randn(n, B, HKV, P, D, device=dev, generator=g).half()
        v = torch.randn(n, B, HKV, P, D, device=dev, generator=g).half()
        a = A.KVArena.allocate(A.TIER_NAMES[tier], B, HKV, n, P, D, dev)
        if tier == "fp16":
            a.write_pages(0, k, v)
        else:
            for j in range(n):
                kn, ko, km = isolate_outliers(k[j], 3.0)
                vn, vo, vm = isolate_outliers(v[j], 3.0)
                paged.quantize_page(a, j, kn, vn)
                ki, kv_ = paged.outliers_to_coo(km, ko)
                vi, vv_ = paged.outliers_to_coo(vm, vo)
                paged.attach_outliers(a, j, ki, kv_, vi, vv_)
                entries += ki.shape[0] + vi.shape[0]
                block_bytes += a._outlier_blocks[j].numel()
        del k, v
        arenas.append(a)
        pages += [(len(arenas) - 1, j, P) for j in range(n)]
    torch.cuda.synchronize()
    plan = A.AttentionPlan(arenas, pages, batch=B, heads_kv=HKV, group=HQ // HKV, head_dim=D)
    bare_arenas = [A.KVArena(a.tier, a.layout, a.k, a.v, bh_stride=a.bh_stride, record_bytes=a.record_bytes,
                             page_tokens=P, head_dim=D, batch=B, heads=HKV, slots=a.slots) for a in arenas]
    bare = A.AttentionPlan(bare_arenas, pages, batch=B, heads_kv=HKV, group=HQ // HKV, head_dim=D)
    q = (torch.randn(B, HQ, 1, D, device=dev, generator=g) / math.sqrt(D)).half()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    with ClockSampler(vis.split(",")[0] if vis else "0") as clk:
        ms = statistics.median(_windows(lambda: plan.run(q), args.steps, 1, dev, min_seconds=args.min_seconds))
        ms_bare = statistics.median(_windows(lambda: bare.run(q), args.steps, 1, dev, min_seconds=0.3))
    hbm, peak_kind = peaks()
    nbytes = plan.compressed_bytes + block_bytes
    values = sum(2 * B * HKV * n * D for t, n in SPLIT if t != "fp16")
    print(json.dumps({"metric": "Llama-3-8B layer decode with outlier sidecars (sigma 3) on every quantized page, "
                                "KV tokens/s", "value": B * L / (ms * 1e-3), "unit": "KV tokens/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "dtype": "fp16", "data": "synthetic",
                      "config": {"workload": "llama3-8b-sidecars", "batch": B, "q_heads": HQ, "kv_heads": HKV,
                                 "head_dim": D, "context": L, "page_size": P, "tiers_oldest_first": dict(SPLIT),
                                 "sigma": 3.0, "outlier_entries": entries,
                                 "outlier_density": entries / max(1, values), "correction_block_bytes": block_bytes},
                      "without_sidecars_ms": ms_bare, "sidecar_cost": ms / ms_bare,
                      "fp16_rebuild_equivalent_ms": 2 * B * HKV * L * D * 2 / (hbm * 1e9) * 1e3,
                      "roofline": {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9, "peak": hbm,
                                   "unit": "GB/s", "frac": nbytes / (ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind,
                                   "algorithmic_bytes_per_launch": nbytes},
                      "clocks": clk.summary()}), flush=True)


def run_70b(args, rank, world, local_rank):
    """Llama-3-70B layer: B 64, H_q 64, H_kv 8, D 128, context 131072 with the 8B tier ratios x4
    (8.98 GB compressed).  Sharded by KV head over the ranks (rank r holds heads [8r/N, 8(r+1)/N) of
    every page: the layer's bytes split N ways, "strong" scaling).  Each rank's share of the oldest
    25% of the pages (its slice of the 1-bit tier) lives in pinned host memory allocated from a
    thread pinned to the GPU's NUMA node, and is streamed in runs of 512 slots on a side stream while
    the resident tiers are attended (spill.SpilledLayerDecode); the two results are joined by LSE and
    the per-head outputs all-gathered (NCCL).  value = B x L / max-over-ranks step time; also the
    resident tiers' kernel against the HBM roof and the host link's GB/s per rank."""
    import torch
    import torch.distributed as dist

    from argus_b200 import attention as A
    from argus_b200 import sharding, spill

    global B, HQ, L, SPLIT
    B, HQ, L = 64, 64, 131072
    SPLIT = [(t, 4 * n) for t, n in SPLIT]
    if HKV % world:
        raise SystemExit(f"{HKV} KV heads do not split over {world} ranks")
    hl = HKV // world
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    cpus = spill.numa_local_cpus(device)
    if cpus:
        os.sched_setaffinity(0, cpus)
    plan_all, _ = build_cache(device, seed=4242 + rank, batch=B, heads_kv=hl)
    gq = torch.Generator(device=device).manual_seed(99)
    q_full = (torch.randn(B, HQ, 1, D, device=device, generator=gq) / math.sqrt(D)).half()
    q_local = sharding.shard_queries(q_full, HKV, world, rank)
    res = plan_all.arenas[1:]  # SPLIT starts with the 1-bit tier: it is the spilled one
    plan_res = A.AttentionPlan(res, [(ai, j, P) for ai, a in enumerate(res) for j in range(a.slots)], batch=B,
                               heads_kv=hl, group=HQ // HKV, head_dim=D)
    host = spill.arenas_to_host([plan_all.arenas[0]])[0]
    layer = spill.SpilledLayerDecode(plan_res, host, chunk_slots=512)
    if world > 1:
        gather = sharding.HeadShardedDecode(plan_res, HKV)
        buf, out_full = gather._buffers(q_local.shape, q_local.dtype, device)

        def step():
            layer(q_local, out=buf[rank])
            gather.all_gather(buf)
            gather.to_head_order(buf, out_full)
    else:
        step = lambda: layer(q_local)  # noqa: E731
    for _ in range(args.warmup):
        step()
    lse_r = torch.empty(B, hl * (HQ // HKV), 1, device=device)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    with ClockSampler(vis.split(",")[local_rank] if vis else str(local_rank)) as clk:
        wins = _windows(step, args.steps, world, device, min_seconds=args.min_seconds)
        res_ms = statistics.median(_windows(lambda: plan_res.run(q_local, lse=lse_r), args.steps, world, device,
                                            min_seconds=0.2))
        all_ms = statistics.median(_windows(lambda: plan_all.run(q_local), args.steps, world, device,
                                            min_seconds=0.2))
    ms = statistics.median(wins)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        value, dt, cpu_steps = time_cpu(1, 0, os.cpu_count() or 1, min_seconds=10.0)
        cpu = {"value": value, "unit": "KV tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"1 sequence x {HKV} KV heads x {L} tokens per step (every tier resident), "
                         f"{cpu_steps} timed steps ({cpu_steps * dt:.1f} s of CPU work)", "scope": CPU_PORT_SCOPE}
    if rank != 0:
        return
    hbm, peak_kind = peaks()
    spilled = host.k.numel()
    print(json.dumps({"metric": "Llama-3-70B layer decode, KV-head sharded, oldest 25% spilled to host, KV tokens/s",
                      "value": B * L / (ms * 1e-3), "unit": "KV tokens/s", "n_gpus": world, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                      "dtype": "fp16", "data": "synthetic",
                      "config": {"workload": "llama3-70b", "batch": B, "q_heads": HQ, "kv_heads": HKV,
                                 "head_dim": D, "context": L, "tiers_oldest_first": dict(SPLIT),
                                 "spilled": "one_bit (25% of the tokens): pinned host memory of the GPU's NUMA node, "
                                            "streamed in runs of 512 slots",
                                 "parallelism": f"kv-head sharded x{world} ({hl} KV heads per GPU)" +
                                                (", NCCL all-gather of outputs" if world > 1 else "")},
                      "timing": {"windows": len(wins), "steps_per_window": args.steps, "statistic": "median window"},
                      "per_rank": {"compressed_bytes": plan_all.compressed_bytes, "spilled_bytes": spilled,
                                   "host_link_GBs": spilled / (ms * 1e-3) / 1e9,
                                   "resident_tiers_ms": res_ms,
                                   "resident_tiers_frac_of_hbm": plan_res.compressed_bytes / (res_ms * 1e-3) / 1e9 / hbm,
                                   "all_resident_ms": all_ms,
                                   "all_resident_frac_of_hbm": plan_all.compressed_bytes / (all_ms * 1e-3) / 1e9 / hbm,
                                   "peak_kind": peak_kind, "numa_local_cpus": len(cpus) if cpus else None},
                      "limiting": "host link (the spilled tier's copies)" if ms > 1.5 * res_ms else
                                  "HBM (the resident tiers' kernel)",
                      "clocks": clk.summary(), "cpu_baseline": cpu}), flush=True)


def run_cascade(args):
    """Quantize/pack cascade microbench: 1,048,576 tokens x 8 KV heads x 128 fp16 (2 GiB, N(0,1)
    with 1% of the values from Laplace(0,4)) packed into every tier and unpacked again through the
    public codec API; bytes = input read + payload and metadata written (unpack: the mirror)."""
    import torch

    from argus_b200.core import quantization as Q

    dev = torch.device("cuda", 0)
    Bc, Hc, Tc, Dc = 1, 8, 1048576, 128
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(Bc, Hc, Tc, Dc, device=dev, generator=g, dtype=torch.float16)
    u = torch.rand(Bc, Hc, Tc, Dc, device=dev, generator=g) - 0.5
    lap = (-4.0 * torch.sign(u) * torch.log1p(-2.0 * u.abs())).half()
    x = torch.where(torch.rand(Bc, Hc, Tc, Dc, device=dev, generator=g) < 0.01, lap, x)
    del u, lap
    torch.cuda.synchronize()
    tiers = [("fp8_sim", Q.quantize_to_fp8_simulated, Q.dequantize_from_fp8_simulated),
             ("int8", Q.quantize_to_int8, Q.dequantize_from_int8),
             ("int4", Q.quantize_to_int4_packed, Q.dequantize_from_int4_packed),
             ("int2", Q.quantize_to_int2_packed, Q.dequantize_from_int2_packed),
             ("1bit", Q.quantize_to_1bit_packed, Q.dequantize_from_1bit_packed)]
    hbm, peak_kind = peaks()
    xbytes = x.numel() * 2
    per_tier, tot_bytes, tot_ms = {}, 0, 0.0
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    with ClockSampler(vis.split(",")[0] if vis else "0") as clk:
        for name, qf, df in tiers:
            coded = qf(x)
            cbytes = sum(t.numel() * t.element_size() for t in coded)
            ms_p = _timed(lambda: qf(x), args.steps, args.warmup)
            ms_u = _timed(lambda: df(*coded), args.steps, args.warmup)
            nb = xbytes + cbytes
            per_tier[name] = {"pack_ms": ms_p, "unpack_ms": ms_u, "pack_GBs": nb / ms_p / 1e6,
                              "unpack_GBs": nb / ms_u / 1e6, "pack_frac": nb / ms_p / 1e6 / hbm,
                              "unpack_frac": nb / ms_u / 1e6 / hbm, "coded_bytes": cbytes}
            tot_bytes += 2 * nb
            tot_ms += ms_p + ms_u
            del coded
            torch.cuda.empty_cache()
    value = tot_bytes / tot_ms / 1e6
    line = {"metric": "quantize/pack cascade microbench, pack+unpack GB/s over all tiers", "value": value,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot_ms,
            "higher_is_better": True, "dtype": "fp16->u8/i8", "data": "synthetic",
            "config": {"workload": "cascade-microbench", "tokens": Tc, "kv_heads": Hc, "head_dim": Dc,
                       "outliers": "1% Laplace(0,4)", "l2": "inputs larger than L2 (2 GiB), no flush"},
            "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s", "frac": value / hbm,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_step": tot_bytes},
            "tiers": per_tier, "clocks": clk.summary()}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = _cascade_cpu()
    print(json.dumps(line), flush=True)


def _cascade_cpu(min_seconds=10.0):
    """The reference's CPU codecs (oracle port, bit-exact) on a bounded sample of the same tensor
    shape: pack+unpack of every tier over 8 heads x 16384 tokens, GB/s by the same byte count."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 8, 16384, 128), dtype=np.float32)
    m = rng.random(x.shape) < 0.01
    x[m] = rng.laplace(0, 4, m.sum())
    x = x.astype(np.float16)
    fns = [(oracle.quantize_to_fp8_simulated, oracle.dequantize_from_int8),
           (oracle.quantize_to_int8, oracle.dequantize_from_int8),
           (oracle.quantize_to_int4_packed, oracle.dequantize_from_int4_packed),
           (oracle.quantize_to_int2_packed, oracle.dequantize_from_int2_packed),
           (oracle.quantize_to_1bit_packed, oracle.dequantize_from_1bit_packed)]
    t0 = time.perf_counter()
    nbytes, n = 0, 0
    while n < 1 or time.perf_counter() - t0 < min_seconds:
        for qf, df in fns:
            coded = qf(x)
            df(*coded)
            nbytes += 2 * (x.nbytes + sum(c.nbytes for c in coded))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"1 x 8 heads x 16384 tokens x 128, every tier packed and unpacked, {n} rounds ({dt:.1f} s)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--min-seconds", type=float, default=1.0,
                    help="repeat the K-step timed window until this much device time has passed")
    ap.add_argument("--workload", choices=("llama3-8b-layer", "jl-archive", "llama3-70b", "tinyllama-sidecars",
                                           "llama3-8b-sidecars", "cascade", "tier-sweep"), default="llama3-8b-layer")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "jl-archive":
        run_jl_archive(args)
        return
    if args.workload == "tinyllama-sidecars":
        run_tinyllama_sidecars(args)
        return
    if args.workload == "llama3-8b-sidecars":
        run_8b_sidecars(args)
        return
    if args.workload == "cascade":
        run_cascade(args)
        return
    if args.workload == "tier-sweep":
        run_tier_sweep(args)
        return
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "llama3-70b" and world == 1:
        run_70b(args, 0, 1, local_rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        if args.workload == "llama3-70b":
            run_70b(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
