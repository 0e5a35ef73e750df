"""Benchmark of the branchcraft B200 hot path.

Default workload (the configuration the headline metric is
quoted on): one speculative-verification step for a batch of 8 requests that
share a 2040-token paged prefix — `tree_verify` over every request's 7-node
draft tree, then the copy-on-write commit of every request's accepted path
(7 shared-page clones + the path rows) — Hq=32, Hkv=8, D=128, FP16 inputs,
FP32 accumulation and output.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1). Every rank runs its own batch
(weak scaling, no data-path collective: requests are independent); `value` is
the whole-job algorithmic HBM traffic rate (all ranks' bytes / max-over-ranks
device time). The inputs (~10 MB) fit in L2, so L2 is flushed (a 256 MiB
device write) between timed steps, outside the per-step CUDA events.

`--impl reference` times the reference's own CPU implementation of the step
(its CPU oracle `cpu_tree_reference`, src/main.cu:204-240, compiled unmodified
from the reference sources into oracle/_ref/libbcref.so, run on one request per
host thread, plus the numpy page copies of the commit) on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "branchcraft-cuda_b200"))

METRIC = "tree_verify µs & HBM TB/s per B200; decode tokens/s at 1/2/4/8 GPUs"
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
FLUSH_BYTES = 256 << 20


def load_peaks():
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, 1590.0, "fallback"


# --------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the
    background; `window(t0, t1)` summarises the samples inside [t0, t1]."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.samples = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def window(self, t0, t1):
        inside = [p for t, p in self.samples if t0 - 0.05 <= t <= t1 + 0.05]
        if not inside and self.samples:  # region shorter than a sample period
            inside = [min(self.samples, key=lambda s: abs(s[0] - (t0 + t1) / 2))[1]]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(p[1]) for p in inside if num(p[1]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for p in inside:
            for name, val in zip(names, p[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(inside[0][2]), "reasons": sorted(reasons),
                "samples": len(inside)}


# --------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def to_dev(torch, a, device):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.float16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def pinned(torch, a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16).copy()).view(torch.float16)
    else:
        t = torch.from_numpy(a.copy())
    return t.pin_memory()


# --------------------------------------------------------------- our arm
def run_ours(args):
    import torch

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    device = torch.device("cuda", torch.cuda.current_device())

    import bc_capi as C
    from bc_workloads import TreeCowWorkload

    hbm_peak, _, peak_kind = load_peaks()
    wl = TreeCowWorkload(seed=2040 + rank)
    plan, _ = wl.plan()
    shape = C.make_shape(*wl.shape())
    k0, v0 = wl.initial_cache()
    cache_k, cache_v = to_dev(torch, k0, device), to_dev(torch, v0, device)
    host = {  # per-step inputs, pinned for the end-to-end leg
        "draft_q": pinned(torch, wl.draft_q), "draft_k": pinned(torch, wl.draft_k),
        "draft_v": pinned(torch, wl.draft_v), "parent": pinned(torch, wl.parent),
        "pages": pinned(torch, wl.pages), "lengths": pinned(torch, wl.lengths),
        "clone_src": pinned(torch, np.array(plan.clone_src, np.int32)),
        "clone_dst": pinned(torch, np.array(plan.clone_dst, np.int32)),
        "e_req": pinned(torch, np.array(plan.entry_request, np.int32)),
        "e_node": pinned(torch, np.array(plan.entry_node, np.int32)),
        "e_page": pinned(torch, np.array(plan.entry_page, np.int32)),
        "e_slot": pinned(torch, np.array(plan.entry_slot, np.int32)),
    }
    dev = {n: t.to(device) for n, t in host.items()}
    out = torch.empty(wl.batch, wl.nodes, wl.hq, wl.dim, device=device, dtype=torch.float32)
    out_host = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    flush = torch.empty(FLUSH_BYTES // 4, device=device, dtype=torch.float32)
    stream = torch.cuda.current_stream()

    launches_per_step = 1 + (1 if plan.clone_src else 0) + (1 if plan.entry_node else 0)

    def device_step(t_ev=None):
        if t_ev:
            t_ev[0].record(stream)
        C.tree_verify(shape, dev["draft_q"], cache_k, cache_v, dev["pages"], dev["lengths"],
                      dev["draft_k"], dev["draft_v"], dev["parent"], out, wl.nodes)
        if t_ev:
            t_ev[1].record(stream)
        C.commit_batch(shape, wl.nodes, dev["draft_k"], dev["draft_v"], cache_k, cache_v,
                       dev["clone_src"], dev["clone_dst"], dev["e_req"], dev["e_node"],
                       dev["e_page"], dev["e_slot"])

    def e2e_step():
        for n, t in host.items():
            dev[n].copy_(t, non_blocking=True)
        device_step()
        out_host.copy_(out, non_blocking=True)

    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()

    # Correctness gate before timing: the first step against the oracle on
    # rank 0 is done by the test-suite; here only the device error word.
    for _ in range(args.warmup):
        flush.fill_(1.0)
        device_step()
        e2e_step()
    torch.cuda.synchronize()
    if C.last_device_error() != 0:
        raise SystemExit("device error word set during warm-up")

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    sampler = ClockSampler(device.index)
    time.sleep(0.3)
    # ---- device-resident timed region
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    tev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    t0 = time.time()
    for i in range(args.steps):
        flush.fill_(1.0)
        evs[i][0].record(stream)
        device_step(tev[i])
        evs[i][1].record(stream)
    barrier()
    t1 = time.time()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    tree_ms = [a.elapsed_time(b) for a, b in tev]
    # ---- end-to-end timed region (pinned host inputs -> device -> host output)
    eevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        flush.fill_(1.0)
        eevs[i][0].record(stream)
        e2e_step()
        eevs[i][1].record(stream)
    barrier()
    sampler.stop()
    e2e_ms = [a.elapsed_time(b) for a, b in eevs]
    err = C.last_device_error()

    total_ms = sum(step_ms)
    total_e2e_ms = sum(e2e_ms)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([total_ms, total_e2e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, total_e2e_ms = float(t[0]), float(t[1])
        e = torch.tensor([err], device=device, dtype=torch.int64)
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
        err = int(e[0])

    step_bytes = wl.verify_bytes() + wl.commit_bytes(plan)
    all_bytes = step_bytes * args.steps * world
    value_tbs = all_bytes / (total_ms * 1e-3) / 1e12
    e2e_tbs = all_bytes / (total_e2e_ms * 1e-3) / 1e12
    tree_us = statistics.mean(tree_ms) * 1e3
    achieved_gbs = wl.verify_bytes() / (tree_us * 1e-6) / 1e9
    clocks = sampler.window(t0, t1)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value_tbs, 6),
            "unit": "TB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 6),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 in / f32 accumulate",
            "data": "synthetic (seeded N(0,1) FP16, per-rank seed)",
            "config": {
                "workload": "BASELINE config 2: batched shared-prefix tree_verify + COW "
                            "commit_path_ (8 requests, shared 2040-token prefix, 7-node "
                            "random trees, Hq=32 Hkv=8 D=128, page 16)",
                "requests_per_gpu": wl.batch, "prefix_tokens": wl.prefix,
                "tree_nodes": wl.nodes, "parallelism": f"request-sharded x{world}",
                "l2": "flushed between timed steps (256 MiB device write, outside the "
                      "step events)",
                "step_bytes": step_bytes,
                "tree_verify_us": round(tree_us, 3),
                "verify_bytes_per_launch": wl.verify_bytes(),
                "verify_flops_per_launch": wl.verify_flops(),
                "commit_clones": len(plan.clone_src),
                "commit_rows": len(plan.entry_node),
            },
            "e2e": {"value": round(e2e_tbs, 6), "unit": "TB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(total_e2e_ms / args.steps, 6)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {
                "kernel": "attn_kernel (tree_verify)",
                "bound": "hbm",
                "achieved": round(achieved_gbs, 2),
                "peak": hbm_peak,
                "unit": "GB/s",
                "frac": round(achieved_gbs / hbm_peak, 4),
                "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": args.traffic,
            },
            "clocks": clocks,
            "device_error_word": err,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_tree_cow(wl, plan, step_bytes)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------- CPU legs
def cpu_baseline_tree_cow(wl, plan, step_bytes):
    """The oracle port (oracle/bc_oracle.cpp, OpenMP over rows) timed on one
    full step of the same workload: tree verify + sequential COW commits."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from cow_oracle import CowOracle

    threads = O.max_threads()
    k0, v0 = wl.initial_cache()
    t = time.perf_counter()
    O.tree(wl.shape(), wl.nodes, wl.draft_q, k0, v0, wl.pages, wl.lengths, wl.draft_k,
           wl.draft_v, wl.parent, threads=threads)
    cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
    r0 = cow.new(wl.prefix_k, wl.prefix_v)
    reqs = [r0] + [cow.fork(r0) for _ in range(wl.batch - 1)]
    for b in range(wl.batch):
        cow.commit(reqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])
    dt = time.perf_counter() - t
    return {"value": round(step_bytes / dt / 1e12, 9), "unit": "TB/s", "cores": threads,
            "kind": "port", "sample": "1 full step (8-request tree verify + 8 COW commits)",
            "seconds": round(dt, 4)}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from concurrent.futures import ThreadPoolExecutor

    from bc_workloads import TreeCowWorkload
    from cow_oracle import CowOracle

    if not O.ref_available():
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/libbcref.so (the reference built from its "
                                         "sources) is missing"}))
        return
    wl = TreeCowWorkload(seed=2040)
    plan, _ = wl.plan()
    k0, v0 = wl.initial_cache()
    step_bytes = wl.verify_bytes() + wl.commit_bytes(plan)
    cores = min(wl.batch, os.cpu_count() or 1)

    def one_request(b):
        s = (1, wl.hq, wl.hkv, wl.dim, wl.max_pages, wl.pool_pages)
        return O.ref_cpu_tree_reference(s, wl.nodes, wl.draft_q[b:b + 1], k0, v0,
                                        wl.pages[b:b + 1], wl.lengths[b:b + 1],
                                        wl.draft_k[b:b + 1], wl.draft_v[b:b + 1],
                                        wl.parent[b:b + 1])

    def step(pool):
        list(pool.map(one_request, range(wl.batch)))
        cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
        r0 = cow.new(wl.prefix_k, wl.prefix_v)
        reqs = [r0] + [cow.fork(r0) for _ in range(wl.batch - 1)]
        for b in range(wl.batch):
            cow.commit(reqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])

    with ThreadPoolExecutor(max_workers=cores) as pool:
        for _ in range(args.warmup):
            step(pool)
        times = []
        for _ in range(args.steps):  # bounded: stop once the CPU budget is spent
            t = time.perf_counter()
            step(pool)
            times.append(time.perf_counter() - t)
            if sum(times) > args.reference_budget_s:
                break
    total = sum(times)
    value = step_bytes * len(times) / total / 1e12
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 9),
        "unit": "TB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total / len(times) * 1e3, 3),
        "steps_timed": len(times),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 in / f64 accumulate (reference CPU oracle)",
        "data": "synthetic (seeded N(0,1) FP16)",
        "config": {"workload": "BASELINE config 2 (same inputs as the CUDA arm, rank 0 seed)",
                   "step_bytes": step_bytes},
        "cpu_baseline": {"value": round(value, 9), "unit": "TB/s", "cores": cores,
                         "kind": "reference",
                         "sample": "each step = the full 8-request step: the reference's "
                                   "cpu_tree_reference (one request per host thread) + "
                                   "the sequential COW commits"},
        "e2e": {"value": round(value, 9), "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu-measured DRAM bytes per tree_verify launch, if known")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reference-budget-s", type=float, default=60.0,
                    help="CPU seconds after which the reference arm stops timing steps")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
