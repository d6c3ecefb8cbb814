"""Benchmark: Page16 decode KV-read bandwidth and tokens/s (BP-KV hot path).

Workload (config 2 of the benchmark plan): Llama-3.1-8B-shaped decode step,
bf16, 32 layers, 32 query / 8 KV heads, head_dim 128, 32 requests per GPU with
context lengths uniform in [4096, 32768], KV scattered in 16-token pages over a
pool sized to 90% of HBM with seeded random block tables, q/k/v ~ 0.5 N(0,1).
One step = one decode step over all 32 layers (one Page16 call per layer on
that layer's pool view).  Requests are sharded across GPUs with no collective
(weak scaling: 32 requests per GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference's CPU path (the gather-then-attention
restatement in oracle/, fp32) on the host cores on a bounded sample of the
same workload; only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS, HQ, HKV, D = 32, 32, 8, 128
BATCH = 32
CTX_LO, CTX_HI = 4096, 32768
POOL_FRAC = 0.90
KV_BYTES_PER_TOKEN = 2 * HKV * D * 2  # K+V, bf16, one layer
METRIC = "decode KV-read HBM GB/s & % peak and tokens/s at 32K ctx, 1/2/4/8 B200"
WORKLOAD = ("llama3.1-8b-shaped page16 decode: 32 layers, 32q/8kv heads, d128, 32 requests/GPU, "
            "ctx U[4096,32768], 16-token pages in a pool of 90% HBM, random block tables")


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def make_requests(seed: int):
    rng = np.random.default_rng(seed)
    lens = rng.integers(CTX_LO, CTX_HI + 1, size=BATCH).astype(np.int32)
    return rng, lens


def algorithmic_bytes(lens) -> int:
    """Bytes one layer's decode must move: KV of every token, q, out, table, lens."""
    kv = int(np.sum(lens)) * KV_BYTES_PER_TOKEN
    pages = int(np.sum((lens + 15) // 16))
    return kv + 2 * BATCH * HQ * D * 2 + 4 * pages + 4 * BATCH


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU side: the reference's gather-then-attention path (oracle/page16.py), fp32
# ---------------------------------------------------------------------------
CPU_SAMPLE_REQUESTS = 8


def cpu_sample(seed: int = 1234):
    """Host-resident synthetic sample: one layer x 8 of the 32 requests (same
    length distribution, pages, scale as the GPU workload), fp32."""
    rng, lens = make_requests(seed)
    lens = lens[:CPU_SAMPLE_REQUESTS]
    need = (lens + 15) // 16
    n_pages = int(need.sum())
    k = (rng.standard_normal((n_pages, 16, HKV, D), dtype=np.float32) * 0.5)
    v = (rng.standard_normal((n_pages, 16, HKV, D), dtype=np.float32) * 0.5)
    q = (rng.standard_normal((len(lens), HQ, D), dtype=np.float32) * 0.5)
    perm = rng.permutation(n_pages).astype(np.int32)
    bt = np.zeros((len(lens), int(need.max())), np.int32)
    off = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[off:off + n]
        off += int(n)
    return q, k, v, bt, lens


def time_cpu_step(sample) -> float:
    from oracle.page16 import page16_decode_reference
    q, k, v, bt, lens = sample
    t0 = time.perf_counter()
    page16_decode_reference(q, k, v, bt, lens, D ** -0.5, HQ // HKV, compute_dtype=np.float32)
    return time.perf_counter() - t0


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline_block(sample, reps: int = 2):
    import torch
    torch.set_num_threads(cpu_cores())
    time_cpu_step(sample)  # warm
    dt = min(time_cpu_step(sample) for _ in range(reps))
    lens = sample[4]
    gbs = algorithmic_bytes_sample(lens) / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu_cores(), "kind": "port",
            "sample": f"1 of 32 layers x {len(lens)} of 32 requests of the same workload, fp32 numpy "
                      f"(BLAS threads = host cores), {dt * 1e3:.0f} ms per call",
            "tokens_per_s_extrapolated": round(len(lens) / (dt * LAYERS), 3)}


def algorithmic_bytes_sample(lens) -> int:
    return int(np.sum(lens)) * KV_BYTES_PER_TOKEN + 2 * len(lens) * HQ * D * 2


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    sample = cpu_sample()
    for _ in range(args.warmup):
        time_cpu_step(sample)
    times = [time_cpu_step(sample) for _ in range(args.steps)]
    dt = float(np.mean(times))
    lens = sample[4]
    gbs = algorithmic_bytes_sample(lens) / dt / 1e9
    cb = {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu_cores(), "kind": "port",
          "sample": f"1 of 32 layers x {len(lens)} of 32 requests, fp32 numpy restatement of the reference "
                    f"gather-then-attention path (core/engine.py:4060-4100)"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": cb["sample"]},
        "tokens_per_s_extrapolated": round(len(lens) / (dt * LAYERS), 3),
        "cpu_baseline": cb,
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def setup_rank(rank: int, device, seed_base: int = 2024, small: bool = False):
    import torch
    global LAYERS
    rng, lens = make_requests(seed_base + rank)
    need = (lens + 15) // 16
    if small:  # profiling case: one layer, pool of just the needed pages (~2.5 GB)
        LAYERS = 1
        n_pages = int(need.sum()) + 64
    else:
        total = torch.cuda.get_device_properties(device).total_memory
        page_bytes = 2 * LAYERS * 16 * HKV * D * 2  # K and V pages of all layers
        n_pages = int(POOL_FRAC * total) // page_bytes
    assert int(need.sum()) <= n_pages
    k_pool = torch.empty((LAYERS, n_pages, 16, HKV, D), dtype=torch.bfloat16, device=device)
    v_pool = torch.empty_like(k_pool)
    g = torch.Generator(device=device).manual_seed(seed_base + rank)
    for l in range(LAYERS):  # q/k/v ~ 0.5 N(0,1) over the whole pool
        k_pool[l].normal_(0.0, 0.5, generator=g)
        v_pool[l].normal_(0.0, 0.5, generator=g)
    perm = rng.permutation(n_pages).astype(np.int32)
    bt = np.zeros((BATCH, int(need.max())), np.int32)
    off = 0
    for b, n in enumerate(need):  # all layers share block ids (core/scheduler.py:1141)
        bt[b, :n] = perm[off:off + n]
        off += int(n)
    qs = [(torch.randn((BATCH, HQ, D), generator=g, device=device) * 0.5).to(torch.bfloat16) for _ in range(LAYERS)]
    return dict(k_pool=k_pool, v_pool=v_pool, bt=bt, lens=lens, qs=qs, n_pages=n_pages)


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist
    from unifiedkv_b200.page16_native import page16_decode_attention

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    st = setup_rank(rank, device, small=args.profile_small)
    k_pool, v_pool, qs = st["k_pool"], st["v_pool"], st["qs"]
    bt_d = torch.from_numpy(st["bt"]).to(device)
    lens_d = torch.from_numpy(st["lens"]).to(device)
    scale = D ** -0.5
    outs = [None] * LAYERS
    stream = torch.cuda.current_stream(device)

    def step(events=None):
        for l in range(LAYERS):
            if events is not None:
                events[l][0].record(stream)
            outs[l] = page16_decode_attention(qs[l], k_pool[l], v_pool[l], bt_d, lens_d, softmax_scale=scale,
                                              n_rep=HQ // HKV)
            if events is not None:
                events[l][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timed region ----
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(LAYERS)] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        t_start.record(stream)
        for s in range(args.steps):
            step(ev[s])
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms_total = max_over_ranks(t_start.elapsed_time(t_end))
    layer_ms = [ev[s][l][0].elapsed_time(ev[s][l][1]) for s in range(args.steps) for l in range(LAYERS)]
    launch_ms = max_over_ranks(float(np.mean(layer_ms)))
    ms_per_step = ms_total / args.steps

    # ---- end-to-end through the public API with host buffers ----
    q_host = [q.cpu().pin_memory() for q in qs]
    out_host = [torch.empty_like(q_host[0]).pin_memory() for _ in range(LAYERS)]
    bt_host = torch.from_numpy(st["bt"]).pin_memory()
    lens_host = torch.from_numpy(st["lens"]).pin_memory()

    def e2e_step():
        btd = bt_host.to(device, non_blocking=True)
        lnd = lens_host.to(device, non_blocking=True)
        for l in range(LAYERS):
            qd = q_host[l].to(device, non_blocking=True)
            o = page16_decode_attention(qd, k_pool[l], v_pool[l], btd, lnd, softmax_scale=scale, n_rep=HQ // HKV)
            out_host[l].copy_(o, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms_step = max_over_ranks(e0.elapsed_time(e1)) / args.steps

    bytes_layer = algorithmic_bytes(st["lens"])  # per rank (same distribution, own seed)
    bytes_step_all = max_over_ranks(0.0)  # placeholder to keep collectives symmetric
    total_bytes = bytes_layer * LAYERS
    if world > 1:
        t = torch.tensor([float(total_bytes)], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        total_bytes_all = float(t.item())
    else:
        total_bytes_all = float(total_bytes)
    del bytes_step_all
    peak, peak_kind = measured_peaks()
    gbs = total_bytes_all / (ms_per_step * 1e-3) / 1e9
    e2e_gbs = total_bytes_all / (e2e_ms_step * 1e-3) / 1e9
    launch_gbs = bytes_layer / (launch_ms * 1e-3) / 1e9  # one launch, one GPU
    tokens_per_s = world * BATCH / (ms_per_step * 1e-3)
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.5) q/k/v, random block tables)",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "batch_per_gpu": BATCH, "global_batch": BATCH * world,
                   "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "pool_pages_per_gpu": st["n_pages"],
                   "mean_ctx_rank0": float(np.mean(st["lens"])), "parallelism": f"request-sharded x{world}",
                   "l2": "no flush: each launch reads ~2.4 GB of KV, far above the 126 MB L2"},
        "tokens_per_s": round(tokens_per_s, 2),
        "hbm_frac_of_measured": round(gbs / world / peak, 4),
        "roofline": {"bound": "hbm", "achieved": round(launch_gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(launch_gbs / peak, 4), "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "kernel": "page16_decode_mma_kernel<bf16,128,8,3> + combine, per layer launch",
                     "avg_launch_ms": round(launch_ms, 4)},
        "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms_step, 4),
                "h2d_bytes_per_step": int(LAYERS * qs[0].numel() * 2 + bt_host.numel() * 4 + lens_host.numel() * 4),
                "d2h_bytes_per_step": int(LAYERS * qs[0].numel() * 2),
                "path": "unifiedkv_b200.page16_native.page16_decode_attention, pinned host q/table/out"},
        "gpu_launches": 2 * LAYERS * args.steps,
        "clocks": clocks.summary(),
    }
    if args.profile_small:
        line["config"]["workload"] += " [profiling case: 1 layer, compact pool]"
    if world == 1 and not args.no_cpu_baseline and not args.profile_small:
        line["cpu_baseline"] = cpu_baseline_block(cpu_sample())
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-small", action="store_true",
                    help="ncu case: 1 layer, pool of only the needed pages (same per-launch work)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
