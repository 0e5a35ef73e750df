"""Benchmark of the branchcraft B200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--repeats R]
                    [--impl ours|reference] [--workload W] [--no-extras]

Headline workload `tree-cow` (the configuration the
headline metric is quoted on): one speculative-verification step for 8
requests that share a 2040-token paged prefix — `tree_verify` over every
request's 7-node draft tree, then the copy-on-write commit of every request's
accepted path (7 shared-page clones + the path rows) — Hq=32, Hkv=8, D=128,
FP16 inputs, FP32 accumulation and output. `value` is the whole-job
algorithmic HBM traffic rate (all ranks' bytes / max-over-ranks device time,
TB/s); `ms_per_step` is the verify+commit step time.

The same run measures every other BASELINE configuration under the key
`configs` (the driver's BENCH and SCALE runs therefore cover them):
  tree-oracle  config 1: 1 request, 2048-token prefix, 7 nodes, FP16 output
  decode       config 3: paged split-KV decode, 4 x 131072 (batch per rank)
  packed       config 4: vLLM-layout packed decode, B=256, lengths U[512, 8192]
  tree-scale   config 5a: 1024 requests x 63-node trees, 4096-token prefix per 16
               (strong scaling: the 64 prefix groups are split across ranks)
  longctx      config 5b: one 1,048,576-token context split across ranks; each
               rank's FP32 partials in one buffer, ONE NCCL all-gather, one
               on-device merge (strong scaling; decode tokens/s)

Protocol, per workload: W untimed warm-up steps; then R timed regions of K
steps each, every region bracketed by a barrier and a device synchronisation
and timed by one pair of CUDA events on the launching stream; the reported
time is the median region (each region's time the max over ranks). Three
kinds of region: device steps (inputs resident in HBM; the tiny tree steps
are replayed from one CUDA graph per rotating input copy, holding exactly the
C-ABI calls a step makes), the dominant kernel alone (K launches back to back
through the C ABI: its average launch duration, for the roofline), and end to
end (each step's inputs copied from pinned host memory and its result copied
back, through the C ABI). Workloads whose one-step working set is smaller than
L2 (tree-cow, tree-oracle) rotate over enough independent copies of it (K/V
pool, step inputs, output) to exceed twice the L2 size, so every step reads
cold data; the others stream more than L2 per step.

One process per GPU (torchrun for N > 1). Request-sharded workloads run every
rank on its own batch (weak scaling, no data-path collective).

`--impl reference` times the reference's own CPU implementation on rank 0 (its
CPU oracle, compiled unmodified from src/main.cu into oracle/_ref/libbcref.so,
one request per host thread), on the same inputs and in the same unit, and
beside it the reference's own GPU kernels (its src/*.cu built for sm_100a)
on the configurations they can run.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
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
SCALE = 1.0 / math.sqrt(128.0)
L2_BYTES = 126 << 20

# DRAM bytes per launch of each workload's dominant kernel (dram__bytes_read.sum
# + dram__bytes_write.sum) from one ncu capture of `python bench.py --workload W
# --steps 1..3 --warmup 3 --no-cpu-baseline --no-extras` on a B200. `packed`
# was captured at --batch 64 (266,106 tokens) and is scaled by tokens to the
# 256-request batch (1,142,306 tokens): its traffic is a per-token stream.
# `tree-scale` was captured at --batch 256 (16 of the 64 prefix groups) and is
# scaled by 4: every group is the same work.
NCU_TRAFFIC = {
    "tree-cow": 9246464,
    "tree-oracle": 8603904,
    # captured at --context 262144: the K/V stream (reads) scales by 4, the
    # partials (writes) do not
    "longctx": 4 * 1073859840 + 3932928,
    "tree-scale": 4 * (468512768 + 114427648),  # a quarter of the requests, captured
    "decode": 2147777536 + 7383040,
    "packed": round((1092800512 + 7438080) * 1142306 / 266106),
}


def load_peaks():
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# --------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons every 100 ms in the background;
    `window(t0, t1)` summarises the samples inside [t0, t1] (with the samples
    just before and after it when fewer than two fall inside)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int):
        self.samples = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
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

    @classmethod
    def _reasons(cls, rows):
        out = set()
        for p in rows:
            for name, val in zip(cls.NAMES, p[5:9]):
                if val.lower().startswith("active"):
                    out.add(name)
        return sorted(out)

    def window(self, t0, t1):
        inside = [p for t, p in self.samples if t0 <= t <= t1]
        bracket = []
        if len(inside) < 2 and self.samples:
            # A region shorter than two sample periods: the last sample before
            # it and the first after it bound its clocks.
            before = [s for s in self.samples if s[0] < t0]
            after = [s for s in self.samples if s[0] > t1]
            bracket = (([max(before, key=lambda s: s[0])[1]] if before else []) +
                       ([min(after, key=lambda s: s[0])[1]] if after else []))
        rows = inside + bracket
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(p[1]) for p in rows if num(p[1]) is not None]
        out = {"sm_mhz": statistics.median(sm) if sm else None,
               "sm_max_mhz": num(rows[0][2]), "samples": len(rows)}
        # Throttle reasons come from the samples inside the region when there
        # are any; the bracketing samples' own reasons are listed apart.
        out["reasons"] = self._reasons(inside if inside else bracket)
        if bracket:
            out["bracketing"] = True
            out["samples_inside"] = len(inside)
            out["reasons_bracketing"] = self._reasons(bracket)
        return out


# --------------------------------------------------------------- helpers
def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))



def graph_kernel_nodes(g):
    """Kernel nodes of a captured torch CUDA graph (kept: keep_graph=True)."""
    from cuda.bindings import runtime as rt

    graph = rt.cudaGraph_t(init_value=g.raw_cuda_graph())
    err, _, n = rt.cudaGraphGetNodes(graph, 0)
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaGraphGetNodes: {err}")
    err, nodes, n = rt.cudaGraphGetNodes(graph, n)
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaGraphGetNodes: {err}")
    count = 0
    for node in nodes[:n]:
        err, kind = rt.cudaGraphNodeGetType(node)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaGraphNodeGetType: {err}")
        count += kind == rt.cudaGraphNodeType.cudaGraphNodeTypeKernel
    return count


def to_dev(torch, a, device):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.float16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def half_bits(torch, t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def oracle_module():
    """The CPU oracle (test infrastructure): loaded only by the CPU-baseline
    leg and the reference arm."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    return O


def region(torch, fn, steps, stream):
    """Device time (ms) of `steps` calls of fn between one pair of CUDA events
    recorded on `stream`."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b)


class CudaRt:
    """The few CUDA runtime calls the pipelined end-to-end loop makes, called
    directly (torch's stream/event/copy wrappers cost several microseconds of
    host time each, which would make a 20 µs step host-bound)."""

    def __init__(self):
        import glob

        import torch  # noqa: F401  (loads the runtime torch uses)

        cands = glob.glob(str(Path(torch.__file__).parent.parent / "nvidia" / "cuda_runtime" /
                              "lib" / "libcudart.so*")) + ["libcudart.so.12", "libcudart.so"]
        for c in cands:
            try:
                self.rt = ctypes.CDLL(c)
                break
            except OSError:
                continue
        vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        self.rt.cudaMemcpyAsync.argtypes = [vp, vp, sz, i, vp]
        self.rt.cudaEventCreateWithFlags.argtypes = [ctypes.POINTER(vp), ctypes.c_uint]
        self.rt.cudaEventRecord.argtypes = [vp, vp]
        self.rt.cudaStreamWaitEvent.argtypes = [vp, vp, ctypes.c_uint]

    def event(self):
        e = ctypes.c_void_p()
        assert self.rt.cudaEventCreateWithFlags(ctypes.byref(e), 2) == 0  # no timing
        return e

    def copy(self, dst, src, nbytes, kind, stream):  # kind 1: H2D, 2: D2H, 3: D2D
        assert self.rt.cudaMemcpyAsync(dst, src, nbytes, kind, stream) == 0

    def record(self, ev, stream):
        assert self.rt.cudaEventRecord(ev, stream) == 0

    def wait(self, stream, ev):
        assert self.rt.cudaStreamWaitEvent(stream, ev, 0) == 0


class PackedInputs:
    """A step's host inputs packed into one pinned buffer (256-byte aligned
    fields) with a device twin, so the end-to-end leg moves them with one
    host-to-device copy; `dev[name]` are typed views into the device buffer."""

    def __init__(self, torch, arrays, device):
        offs, off = {}, 0
        tens = {}
        for n, a in arrays.items():
            t = a if isinstance(a, torch.Tensor) else (
                torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).view(torch.float16)
                if np.asarray(a).dtype == np.uint16 else torch.from_numpy(np.ascontiguousarray(a).copy()))
            t = t.contiguous().cpu()
            tens[n] = t
            offs[n] = off
            off += (t.numel() * t.element_size() + 255) // 256 * 256
        self.nbytes = off
        self.host = torch.empty(off, dtype=torch.uint8).pin_memory()
        for n, t in tens.items():
            nb = t.numel() * t.element_size()
            self.host[offs[n]:offs[n] + nb].copy_(t.view(-1).view(torch.uint8))
        self.buf = self.host.to(device)
        self.dev = {n: self.buf[offs[n]:offs[n] + t.numel() * t.element_size()]
                    .view(t.dtype).view(t.shape) for n, t in tens.items()}
        self.payload = sum(t.numel() * t.element_size() for t in tens.values())


# --------------------------------------------------------------- workloads
# Each workload: device_step() (one step, inputs resident), kernel_step() (the
# dominant kernel alone), e2e_region(K) or e2e_step() (host copies included),
# and the facts of its JSON entry.
class Workload:
    flush = False
    higher_is_better = True
    scaling = "weak"
    kernel_launches = 1  # launches per kernel_step

    def prepare(self):
        """After warm-up, before timing (e.g. capture CUDA graphs)."""

    def step_form(self):
        return "the step's C-ABI calls issued directly"

    def e2e_form(self):
        return "sequential: H2D, compute, D2H per step"

    def release(self):
        """Drop device memory before the next workload."""
        for n in list(vars(self)):
            if n not in ("torch", "C", "device"):
                delattr(self, n)

    def l2_note(self):
        return "inputs larger than L2 (no flush)"

    def reference_step(self, pool):
        return None


class TreeCow(Workload):
    """Config 2. The working set of one step (K/V pool, draft inputs, output)
    is far below L2, so the bench rotates over `copies` independent copies of
    all of it, more than twice the L2 size in total: each step touches data
    last used `copies` steps earlier (cold in L2) and no flush kernel runs
    between steps. A step is ONE C-ABI call, bc_tree_step: the device planner
    (the copy-on-write page bookkeeping of the batch) and the verify launch
    that also executes the planned commit. Every step reads the same pool
    state and writes the state after it to separate arrays (the bench replays
    one transaction). Device steps are replayed from one CUDA graph per copy
    holding that call."""

    name = "tree-cow"
    unit = "TB/s"

    def __init__(self, torch, C, device, rank, world, **_):
        from bc_workloads import TreeCowWorkload

        self.torch, self.C, self.device = torch, C, device
        wl = self.wl = TreeCowWorkload(seed=2040 + rank)
        self.plan, _ = wl.plan()
        plan = self.plan
        self.shape = C.make_shape(*wl.shape())
        self.io_arrays = {
            "draft_q": wl.draft_q, "draft_k": wl.draft_k, "draft_v": wl.draft_v,
            "parent": wl.parent, "pages": wl.pages, "lengths": wl.lengths,
            "clone_src": np.array(plan.clone_src, np.int32),
            "clone_dst": np.array(plan.clone_dst, np.int32),
            "e_req": np.array(plan.entry_request, np.int32),
            "e_node": np.array(plan.entry_node, np.int32),
            "e_page": np.array(plan.entry_page, np.int32),
            "e_slot": np.array(plan.entry_slot, np.int32),
            "path_len": np.array([len(p) for p in wl.paths], np.int32),
            "path_nodes": np.array([p + [-1] * (wl.nodes - len(p)) for p in wl.paths], np.int32)}
        self.out_shape = (wl.batch, wl.nodes, wl.hq, wl.dim)
        self.out_dtype = torch.float32
        self.nodes = wl.nodes
        # One C-ABI call per step, bc_tree_step: the device planner (page
        # bookkeeping of the 8 commits) and the verify launch that also runs
        # the planned commit (7 clones, 23 rows) on its idle warps. The plan
        # is made by one extra cluster of the verify launch when the grid
        # stays one wave, else by a planner launch before it; `prepare`
        # counts the launches in the captured step.
        self.fused = len(plan.clone_src) <= 256
        self.launches = 2 if self.fused else 3
        self.step_bytes = wl.verify_bytes() + wl.commit_bytes(plan)
        self.kernel_bytes = self.step_bytes if self.fused else wl.verify_bytes()
        self.kernel = ("tree_mma_kernel (tree_verify + the fused COW commit)" if self.fused
                       else "tree_mma_kernel (tree_verify)")
        self.bound = "hbm"
        self._make_copies(*wl.initial_cache())

    def _make_copies(self, k0, v0):
        torch = self.torch
        per_copy = 2 * k0.nbytes + 2 * int(np.prod(self.out_shape)) * 4
        self.copies = max(2, -(-2 * L2_BYTES // per_copy))
        self.caches = [(to_dev(torch, k0, self.device), to_dev(torch, v0, self.device))
                       for _ in range(self.copies)]
        self.ios = [PackedInputs(torch, self.io_arrays, self.device) for _ in range(self.copies)]
        self.outs = [torch.empty(self.out_shape, dtype=self.out_dtype, device=self.device)
                     for _ in range(self.copies)]
        self.out_hosts = [torch.empty(self.out_shape, dtype=self.out_dtype).pin_memory()
                          for _ in range(self.copies)]
        self.rot = 0
        self._argv = {}
        if getattr(self, "wl", None) is not None and hasattr(self.wl, "pool"):
            # The page pool's device state before the step (refcounts, free
            # stack, free count; 2 KB), which every step reads, and the state
            # after it, which it writes (one per rotating copy): the bench
            # replays one step, and each replay plans from the same state.
            pool = self.wl.pool
            P = pool.physical_pages
            st = np.array(pool.refcount + pool.free + [0] * (P - len(pool.free)) +
                          [len(pool.free)], np.int32)
            self.state0 = torch.from_numpy(st).to(self.device)
            self.states = [self.state0.clone() for _ in range(self.copies)]
            self.plans = [self.C.CowPlan(self.wl.batch, self.wl.nodes, self.wl.max_pages,
                                         self.device) for _ in range(self.copies)]

    def _next(self):
        c = self.rot
        self.rot = (self.rot + 1) % self.copies
        return c

    def _args(self, c, stream):
        """The C-ABI argument tuples of copy c on `stream` (built once: a
        step then costs one foreign call per entry point)."""
        key = (c, stream.cuda_stream)
        if key not in self._argv:
            d, C = self.ios[c].dev, self.C
            ck, cv = self.caches[c]
            P = C._ptr
            st = ctypes.c_void_p(stream.cuda_stream)
            tv = (ctypes.byref(self.shape), P(d["draft_q"]), P(ck), P(cv), P(d["pages"]),
                  P(d["lengths"]), P(d["draft_k"]), P(d["draft_v"]), P(d["parent"]),
                  P(self.outs[c]), self.nodes, st)
            cb = fv = None
            if "clone_src" in d:
                cb = (ctypes.byref(self.shape), self.nodes, P(d["draft_k"]), P(d["draft_v"]),
                      P(ck), P(cv), P(d["clone_src"]), P(d["clone_dst"]),
                      int(d["clone_src"].numel()), P(d["e_req"]), P(d["e_node"]),
                      P(d["e_page"]), P(d["e_slot"]), int(d["e_node"].numel()), st)
                fv = (ctypes.byref(self.shape), P(d["draft_q"]), P(ck), P(cv), P(d["pages"]),
                      P(d["lengths"]), P(d["draft_k"]), P(d["draft_v"]), P(d["parent"]),
                      P(self.outs[c]), int(self.out_dtype == self.torch.float16), self.nodes,
                      P(d["clone_src"]), P(d["clone_dst"]), int(d["clone_src"].numel()),
                      P(d["e_req"]), P(d["e_node"]), P(d["e_page"]), P(d["e_slot"]),
                      int(d["e_node"].numel()), st)
            sv = None
            if "path_len" in d and hasattr(self, "states"):
                npool = self.wl.pool_pages
                stt = self.states[c]
                sv = (ctypes.byref(self.shape), P(d["draft_q"]), P(ck), P(cv), P(d["pages"]),
                      P(d["lengths"]), P(d["draft_k"]), P(d["draft_v"]), P(d["parent"]),
                      P(self.outs[c]), int(self.out_dtype == self.torch.float16), self.nodes,
                      P(d["path_len"]), P(d["path_nodes"]), P(self.state0[:npool]),
                      P(self.state0[npool:2 * npool]), P(self.state0[2 * npool:]),
                      P(stt[:npool]), P(stt[npool:2 * npool]), P(stt[2 * npool:]),
                      *self.plans[c].args(), st)
            fn = (C.lib().bc_tree_verify_f16 if self.out_dtype == self.torch.float16
                  else C.lib().bc_tree_verify)
            self._argv[key] = (fn, tv, cb, fv, sv)
        return self._argv[key]

    def launch(self, c, stream=None, verify_only=False, host_plan=False):
        """One step on copy c: bc_tree_step (the device plan made from the
        pool state before the step, the state after it written to copy c's
        arrays, and the verify with the fused commit); with host_plan the
        fused verify + commit of the plan made once on the host
        (bc_tree_verify_commit); verify_only: bc_tree_verify alone."""
        stream = stream or self.torch.cuda.current_stream()
        fn, tv, cb, fv, sv = self._args(c, stream)
        if sv is not None and not verify_only and not host_plan:
            rc = self.C.lib().bc_tree_step(*sv)
        elif fv is not None and getattr(self, "fused", False) and not verify_only:
            rc = self.C.lib().bc_tree_verify_commit(*fv)
        else:
            rc = fn(*tv)
            if cb is not None and rc == 0 and not verify_only:
                rc = self.C.lib().bc_commit_batch(*cb)
        if rc != 0:
            raise self.C.BranchcraftError(f"bench step failed with cudaError {rc}")

    # The headline step issues the C-ABI call directly: consecutive steps'
    # kernels are then programmatic dependents (the next launch's set-up
    # overlaps the previous one's tail), which graph replays are not. The
    # graph replay of the same step is timed beside it. The end-to-end loop
    # either issues each step's copies and call on three streams (config 2:
    # 1.6 MB of copies a step, bound by PCIe: 28.5 us a step against 32.8
    # with graphs, measured) or replays one graph per step holding the
    # previous step's result copy, this step and the next step's input copy
    # (config 1: small copies, bound by the host's issue of ten runtime calls
    # a step: 15.5 us against 19.2 with streams).
    direct_steps = True
    graph_e2e = False

    def prepare(self):
        """One CUDA graph per rotating copy, captured from the step's C-ABI
        calls (the library's per-device caches are warm by now), and the
        end-to-end loop's graphs. The step's launch count is read from the
        captured graphs: their kernel nodes."""
        torch = self.torch
        self.graphs = []
        cap = torch.cuda.Stream()
        kernels = set()
        for c in range(self.copies):
            g = torch.cuda.CUDAGraph(keep_graph=True)
            with torch.cuda.graph(g, stream=cap):
                self.launch(c, cap)
            kernels.add(graph_kernel_nodes(g))
            g.instantiate()
            self.graphs.append(g)
        torch.cuda.synchronize()
        if len(kernels) != 1:
            raise RuntimeError(f"the rotating copies' step graphs differ: {sorted(kernels)}")
        self.launches = kernels.pop()
        if self.graph_e2e:
            self._capture_e2e(cap)

    def step_form(self):
        return ("the step's C-ABI call issued directly (consecutive steps' kernels are "
                "programmatic dependents)" if self.direct_steps else
                "one CUDA graph replay per step (the step's C-ABI calls, captured per rotating "
                "input copy)")

    def e2e_form(self):
        if self.graph_e2e:
            return ("pipelined, one CUDA graph per step: the previous step's result D2H, this "
                    "step's C-ABI call and the next step's input H2D (three branches); the "
                    "first H2D and the last D2H outside the graphs, so the region moves one "
                    "input and one result more than its steps use")
        return "pipelined: next step's H2D and previous step's D2H overlap the compute"

    def device_step(self):
        c = self._next()
        if self.direct_steps:
            self.launch(c)
        else:
            self.graphs[c].replay()

    def kernel_step(self):
        # the dominant kernel: verify with the fused commit (of the host-made
        # plan: the planner is a separate launch), or the verify alone
        self.launch(self._next(), verify_only=not getattr(self, "fused", False), host_plan=True)

    def alt_steps(self):
        """Other forms of the same step, timed beside the headline one:
        name -> (one step, its launches)."""
        alts = {}
        if getattr(self, "graphs", None):
            if self.direct_steps:
                alts["the same step replayed from a CUDA graph (one per rotating copy)"] = (
                    lambda: self.graphs[self._next()].replay(), self.launches)
            else:
                alts["the same step's C-ABI call issued directly"] = (
                    lambda: self.launch(self._next()), self.launches)
        if hasattr(self, "states"):
            alts["plan made once on the host (bc_tree_verify_commit: one launch)"] = (
                lambda: self.launch(self._next(), host_plan=True), 1)
        return alts

    def e2e_step(self):
        c = self._next()
        io = self.ios[c]
        io.buf.copy_(io.host, non_blocking=True)
        self.launch(c)
        self.out_hosts[c].copy_(self.outs[c], non_blocking=True)

    def _capture_e2e(self, cap):
        """Graph c: D2H of copy c-1's result, the step on copy c, H2D of copy
        c+1's inputs, as three branches joined at the end (copy c+1's inputs
        were last read by an earlier graph, copy c-1's result was written by
        the graph before: both complete, by stream order)."""
        torch = self.torch
        n = self.copies
        h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
        self.e2e_graphs = []
        for c in range(n):
            prev, nxt = (c - 1) % n, (c + 1) % n
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                h2d.wait_stream(cap)
                d2h.wait_stream(cap)
                with torch.cuda.stream(d2h):
                    self.out_hosts[prev].copy_(self.outs[prev], non_blocking=True)
                with torch.cuda.stream(h2d):
                    self.ios[nxt].buf.copy_(self.ios[nxt].host, non_blocking=True)
                self.launch(c, cap)
                cap.wait_stream(d2h)
                cap.wait_stream(h2d)
            self.e2e_graphs.append(g)
        torch.cuda.synchronize()

    def e2e_region(self, steps):
        """`steps` end-to-end steps as a serving loop runs them (see
        e2e_form); every step's inputs go host-to-device and its result
        device-to-host inside the timed region. Returns the device time (ms)."""
        if self.graph_e2e:
            torch = self.torch
            main = torch.cuda.current_stream()
            n = self.copies
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(main)
            self.ios[0].buf.copy_(self.ios[0].host, non_blocking=True)
            for i in range(steps):
                self.e2e_graphs[i % n].replay()
            last = (steps - 1) % n
            self.out_hosts[last].copy_(self.outs[last], non_blocking=True)
            t1.record(main)
            t1.synchronize()
            self.rot = steps % n
            return t0.elapsed_time(t1)
        return self._e2e_streams(steps)

    def _e2e_streams(self, steps):
        """`steps` end-to-end steps as a serving loop runs them: step i's
        inputs go host-to-device on one copy stream, its result device-to-host
        on another, so copies of neighbouring steps overlap the compute; the
        compute is the step's two C-ABI calls. Returns the device time (ms)."""
        torch = self.torch
        if not hasattr(self, "h2d"):
            self.h2d, self.d2h = torch.cuda.Stream(), torch.cuda.Stream()
            self.rt = CudaRt()
            n = self.copies
            self.ev_up = [self.rt.event() for _ in range(n)]
            self.ev_done = [self.rt.event() for _ in range(n)]
            self.ev_down = [self.rt.event() for _ in range(n)]
        rt, n = self.rt, self.copies
        main = torch.cuda.current_stream()
        ms, hs, ds = (ctypes.c_void_p(x.cuda_stream) for x in (main, self.h2d, self.d2h))
        out_bytes = int(np.prod(self.out_shape)) * (4 if self.out_dtype == torch.float32 else 2)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(main)
        self.h2d.wait_stream(main)
        self.d2h.wait_stream(main)
        self.rot = 0
        for i in range(steps):
            c = self._next()
            io = self.ios[c]
            if i >= n:
                rt.wait(hs, self.ev_done[c])  # copy c's inputs are no longer read
            rt.copy(io.buf.data_ptr(), io.host.data_ptr(), io.nbytes, 1, hs)
            rt.record(self.ev_up[c], hs)
            rt.wait(ms, self.ev_up[c])
            if i >= n:
                rt.wait(ms, self.ev_down[c])  # copy c's previous result has been read back
            self.launch(c, main)
            rt.record(self.ev_done[c], ms)
            rt.wait(ds, self.ev_done[c])
            rt.copy(self.out_hosts[c].data_ptr(), self.outs[c].data_ptr(), out_bytes, 2, ds)
            rt.record(self.ev_down[c], ds)
        main.wait_stream(self.h2d)
        main.wait_stream(self.d2h)
        t1.record(main)
        t1.synchronize()
        return t0.elapsed_time(t1)

    def io_bytes(self):
        return self.ios[0].nbytes, int(np.prod(self.out_shape)) * (
            4 if self.out_dtype == self.torch.float32 else 2)

    def l2_note(self):
        per = 2 * self.caches[0][0].numel() * 2 + self.ios[0].nbytes + \
            int(np.prod(self.out_shape)) * (4 if self.out_dtype == self.torch.float32 else 2)
        return (f"inputs larger than L2: {self.copies} rotating copies of the K/V pool, step "
                f"inputs and output ({per / 2**20:.1f} MiB each, {self.copies * per / 2**20:.0f} "
                f"MiB in total, L2 126 MiB); no flush kernel")

    def value(self, steps_all_ranks, seconds):
        return self.step_bytes * steps_all_ranks / seconds / 1e12

    def config(self):
        wl = self.wl
        return {"workload": "BASELINE config 2: batched shared-prefix tree_verify + COW "
                            "commit_path_ (8 requests, shared 2040-token prefix, 7-node random "
                            "trees, Hq=32 Hkv=8 D=128, page 16)",
                "requests_per_gpu": wl.batch, "prefix_tokens": wl.prefix,
                "tree_nodes": wl.nodes, "step_bytes": self.step_bytes,
                "verify_bytes_per_launch": wl.verify_bytes(),
                "verify_flops_per_launch": wl.verify_flops(),
                "commit_clones": len(self.plan.clone_src),
                "commit_rows": len(self.plan.entry_node),
                "step": ("bc_tree_step: device COW planner (pool state in -> out), verify "
                         "launch executing the planned commit" if hasattr(self, "states")
                         else "bc_tree_verify + bc_commit_batch")}

    def cpu_baseline(self):
        """The oracle port (OpenMP over rows) on one full step."""
        O = oracle_module()
        from cow_oracle import CowOracle

        wl = self.wl
        k0, v0 = wl.initial_cache()
        t = time.perf_counter()
        O.tree(wl.shape(), wl.nodes, wl.draft_q, k0, v0, wl.pages, wl.lengths, wl.draft_k,
               wl.draft_v, wl.parent, threads=O.max_threads())
        cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
        r0 = cow.new(wl.prefix_k, wl.prefix_v)
        reqs = [r0] + [cow.fork(r0) for _ in range(wl.batch - 1)]
        for b in range(wl.batch):
            cow.commit(reqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])
        dt = time.perf_counter() - t
        return {"value": self.step_bytes / dt / 1e12, "unit": self.unit,
                "cores": O.max_threads(), "kind": "port",
                "sample": "1 full step (8-request tree verify + 8 COW commits)",
                "seconds": round(dt, 4)}

    def reference_step(self, pool):
        """The reference's cpu_tree_reference per request (one per thread) +
        the sequential COW commits; returns (seconds, bytes, units)."""
        O = oracle_module()
        from cow_oracle import CowOracle

        wl = self.wl
        k0, v0 = wl.initial_cache()

        def one(b):
            s = (1, wl.hq, wl.hkv, wl.dim, wl.max_pages, wl.pool_pages)
            return O.ref_cpu_tree_reference(s, wl.nodes, wl.draft_q[b:b + 1], k0, v0,
                                            wl.pages[b:b + 1], wl.lengths[b:b + 1],
                                            wl.draft_k[b:b + 1], wl.draft_v[b:b + 1],
                                            wl.parent[b:b + 1])

        t = time.perf_counter()
        list(pool.map(one, range(wl.batch)))
        cow = CowOracle(wl.pool_pages, wl.hkv, wl.dim)
        r0 = cow.new(wl.prefix_k, wl.prefix_v)
        reqs = [r0] + [cow.fork(r0) for _ in range(wl.batch - 1)]
        for b in range(wl.batch):
            cow.commit(reqs[b], wl.paths[b], wl.draft_k[b], wl.draft_v[b])
        return time.perf_counter() - t, self.step_bytes, wl.batch


class TreeOracle(TreeCow):
    """one request, 2048-token prefix in a seeded permutation
    of a 256-page pool, parents [-1,0,0,1,1,2,2], FP16 output; the step is one
    bc_tree_verify_f16 call (its graph replay timed beside it)."""

    name = "tree-oracle"
    graph_e2e = True

    def __init__(self, torch, C, device, rank, world, **_):
        from bc_workloads import rand_half

        self.torch, self.C, self.device = torch, C, device
        rng = np.random.default_rng(2048 + rank)
        P, prefix, N = 256, 2048, 7
        self.N = self.nodes = N
        self.prefix = prefix
        self.k = rand_half(rng, (P, 16, 8, 128))
        self.v = rand_half(rng, (P, 16, 8, 128))
        self.pages = rng.permutation(P).astype(np.int32)[:prefix // 16].reshape(1, -1)
        self.lengths = np.array([prefix], np.int32)
        self.dq = rand_half(rng, (1, N, 32, 128))
        self.dk = rand_half(rng, (1, N, 8, 128))
        self.dv = rand_half(rng, (1, N, 8, 128))
        self.parent = np.array([[-1, 0, 0, 1, 1, 2, 2]], np.int32)
        self.shape = C.make_shape(1, 32, 8, 128, prefix // 16, P)
        self.io_arrays = {"draft_q": self.dq, "draft_k": self.dk, "draft_v": self.dv,
                          "parent": self.parent, "pages": self.pages, "lengths": self.lengths}
        self.out_shape = (1, N, 32, 128)
        self.out_dtype = torch.float16
        self.launches = 1
        self.step_bytes = (prefix * 4096 + N * 8 * 128 * 2 * 2 + N * 32 * 128 * 2
                           + N * 32 * 128 * 2 + prefix // 16 * 4 + 4 + N * 4)
        self.kernel_bytes = self.step_bytes
        self.kernel = "tree_mma_kernel (tree_verify, FP16 out)"
        self.bound = "hbm"
        self._make_copies(self.k, self.v)

    def config(self):
        return {"workload": "BASELINE config 1: tree_verify, 1 request, 2048-token prefix in a "
                            "permuted 256-page pool, parents [-1,0,0,1,1,2,2], FP16 output",
                "step_bytes": self.step_bytes}

    def cpu_baseline(self):
        O = oracle_module()
        t = time.perf_counter()
        O.tree(self.shape_tuple(), self.N, self.dq, self.k, self.v, self.pages, self.lengths,
               self.dk, self.dv, self.parent, threads=O.max_threads())
        dt = time.perf_counter() - t
        return {"value": self.step_bytes / dt / 1e12, "unit": self.unit,
                "cores": O.max_threads(), "kind": "port", "sample": "1 full step",
                "seconds": round(dt, 4)}

    def shape_tuple(self):
        s = self.shape
        return (s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages)

    def reference_step(self, pool):
        O = oracle_module()
        t = time.perf_counter()
        O.ref_cpu_tree_reference(self.shape_tuple(), self.N, self.dq, self.k, self.v,
                                 self.pages, self.lengths, self.dk, self.dv, self.parent)
        return time.perf_counter() - t, self.step_bytes, 1


class TreeHbm(TreeCow):
    """Tree verify where every request has its own prefix (no sharing): 256
    requests x 2040-token private prefixes, 7-node random trees (config-2
    shapes), FP32 output. Not a BASELINE config: it shows the verifier
    against the HBM roofline on a workload large enough to be bandwidth-bound
    (2.1 GB of K/V per step, two rotating copies: inputs larger than L2)."""

    name = "tree-hbm"

    def __init__(self, torch, C, device, rank, world, batch=0, **_):
        from bc_workloads import rand_half, random_parents

        self.torch, self.C, self.device = torch, C, device
        B = batch or 256
        rng = np.random.default_rng(4096 + rank)
        prefix, N, npg = 2040, 7, 128
        self.batch, self.N, self.nodes, self.prefix = B, N, N, prefix
        P = B * npg + 8
        self.pages = rng.permutation(P).astype(np.int32)[:B * npg].reshape(B, npg)
        self.lengths = np.full(B, prefix, np.int32)
        self.dq = rand_half(rng, (B, N, 32, 128))
        self.dk = rand_half(rng, (B, N, 8, 128))
        self.dv = rand_half(rng, (B, N, 8, 128))
        self.parent = np.stack([random_parents(rng, N) for _ in range(B)]).astype(np.int32)
        self.shape = C.make_shape(B, 32, 8, 128, npg, P)
        self.P = P
        self.io_arrays = {"draft_q": self.dq, "draft_k": self.dk, "draft_v": self.dv,
                          "parent": self.parent, "pages": self.pages, "lengths": self.lengths}
        self.out_shape = (B, N, 32, 128)
        self.out_dtype = torch.float32
        self.launches = 1
        self.step_bytes = (B * prefix * 4096 + 2 * B * N * 8 * 128 * 2 + B * N * 32 * 128 * 2
                           + B * N * 32 * 128 * 4 + B * npg * 4 + B * 4 + B * N * 4)
        self.kernel_bytes = self.step_bytes
        self.kernel = "tree_mma_kernel (tree_verify, private prefixes)"
        self.bound = "hbm"
        self._make_copies(None, None)

    def _make_copies(self, k0, v0):
        torch = self.torch
        self.copies = 2  # 4.2 GB of K/V in all, far above L2
        g = torch.Generator(device=self.device)
        g.manual_seed(11)
        shape = (self.P, 16, 8, 128)
        self.caches = [(torch.randn(shape, device=self.device, dtype=torch.float16, generator=g),
                        torch.randn(shape, device=self.device, dtype=torch.float16, generator=g))
                       for _ in range(self.copies)]
        self.ios = [PackedInputs(torch, self.io_arrays, self.device) for _ in range(self.copies)]
        self.outs = [torch.empty(self.out_shape, dtype=self.out_dtype, device=self.device)
                     for _ in range(self.copies)]
        self.out_hosts = [torch.empty(self.out_shape, dtype=self.out_dtype).pin_memory()
                          for _ in range(self.copies)]
        self.rot = 0
        self._argv = {}

    def prepare(self):
        """Half-millisecond steps: direct calls, no graph."""

    def config(self):
        return {"workload": f"tree_verify, {self.batch} requests x {self.prefix}-token private "
                            "prefixes (no sharing), 7-node random trees, FP32 output (not a "
                            "BASELINE config: the verifier on an HBM-bound workload)",
                "step_bytes": self.step_bytes}

    def cpu_baseline(self):
        O = oracle_module()
        torch = self.torch
        ck, cv = self.caches[0]
        ids = torch.from_numpy(self.pages[0].astype(np.int64)).to(self.device)
        k = half_bits(torch, ck[ids])
        v = half_bits(torch, cv[ids])
        pages = np.arange(self.pages.shape[1], dtype=np.int32).reshape(1, -1)
        s = (1, 32, 8, 128, pages.shape[1], pages.shape[1])
        t = time.perf_counter()
        O.tree(s, self.N, self.dq[:1], k, v, pages, self.lengths[:1], self.dk[:1], self.dv[:1],
               self.parent[:1], threads=O.max_threads())
        dt = time.perf_counter() - t
        per_step = dt * self.batch
        return {"value": self.step_bytes / per_step / 1e12, "unit": self.unit,
                "cores": O.max_threads(), "kind": "port",
                "sample": f"request 0 of {self.batch}, scaled linearly to the batch",
                "seconds": round(dt, 4)}

    def reference_step(self, pool):
        return None


class Decode(Workload):
    """paged split-KV decode of `batch` one-token requests
    over `context` tokens each (pages in a seeded random permutation); every
    rank its own batch (weak scaling)."""

    name = "decode"
    unit = "tokens/s"

    def __init__(self, torch, C, device, rank, world, batch=0, context=0, splits=0, **_):
        self.torch, self.C, self.device = torch, C, device
        batch, context = batch or 4, context or 131072
        self.batch, self.context = batch, context
        g = torch.Generator(device=device)
        g.manual_seed(3 + rank)
        npg = context // 16
        P = batch * npg + 8
        self.k = torch.randn(P, 16, 8, 128, device=device, dtype=torch.float16, generator=g)
        self.v = torch.randn(P, 16, 8, 128, device=device, dtype=torch.float16, generator=g)
        perm = torch.randperm(P, device=device, generator=g).to(torch.int32)
        self.pages = perm[:batch * npg].view(batch, npg).contiguous()
        self.lengths = torch.full((batch,), context, device=device, dtype=torch.int32)
        self.shape = C.make_shape(batch, 32, 8, 128, npg, P)
        self.splits = splits or C.auto_splits(self.shape, context, 148)
        rows = batch * 32
        self.pa = torch.empty(self.splits * rows * 128, device=device)
        self.pml = torch.empty(self.splits * rows * 2, device=device)
        self.q_host = torch.randn(batch, 32, 128, dtype=torch.float16).pin_memory()
        self.q = self.q_host.to(device)
        self.out = torch.empty(batch, 32, 128, device=device)
        self.out_host = torch.empty(self.out.shape).pin_memory()
        self.launches = 1 + (self.splits > 8)
        self.kernel_launches = self.launches
        self.kernel_bytes = batch * context * 4096 + rows * 128 * 2 + rows * 128 * 4
        self.step_bytes = self.kernel_bytes
        self.kernel = ("attn_kernel (paged decode)" +
                       (" + merge_kernel (the events bracket both)" if self.splits > 8 else ""))
        self.bound = "hbm"

    def device_step(self):
        self.C.decode(self.shape, self.q, self.k, self.v, self.pages, self.lengths, self.out,
                      self.pa, self.pml, self.splits)

    kernel_step = device_step

    def e2e_step(self):
        self.q.copy_(self.q_host, non_blocking=True)
        self.device_step()
        self.out_host.copy_(self.out, non_blocking=True)

    def io_bytes(self):
        return self.q_host.numel() * 2, self.out_host.numel() * 4

    def value(self, steps_all_ranks, seconds):
        return self.batch * steps_all_ranks / seconds

    def config(self):
        return {"workload": f"BASELINE config 3: paged GQA split-KV decode, batch {self.batch} x "
                            f"context {self.context}, Hq=32 Hkv=8 D=128",
                "splits": self.splits, "kv_bytes": self.batch * self.context * 4096}

    def _sample(self, tokens):
        """Host copy of request 0's first `tokens` tokens as a compact fixture."""
        torch = self.torch
        npg = tokens // 16
        ids = self.pages[0, :npg].long()
        k = half_bits(torch, self.k[ids])
        v = half_bits(torch, self.v[ids])
        q = half_bits(torch, self.q[:1])
        pages = np.arange(npg, dtype=np.int32).reshape(1, -1)
        return (1, 32, 8, 128, npg, npg), q, k, v, pages, np.array([tokens], np.int32)

    def cpu_baseline(self, tokens=16384):
        O = oracle_module()
        s, q, k, v, pages, lengths = self._sample(tokens)
        t = time.perf_counter()
        O.decode(s, q, k, v, pages, lengths, threads=O.max_threads())
        dt = time.perf_counter() - t
        per_step = dt * (self.context / tokens) * self.batch
        return {"value": self.batch / per_step, "unit": self.unit, "cores": O.max_threads(),
                "kind": "port", "sample": f"request 0, first {tokens} tokens, scaled linearly "
                                          f"to {self.batch} x {self.context}",
                "seconds": round(dt, 4)}

    def reference_step(self, pool, tokens=8192):
        O = oracle_module()
        s, q, k, v, pages, lengths = self._sample(tokens)
        t = time.perf_counter()
        O.ref_cpu_reference(s, q, k, v, pages, lengths)
        dt = (time.perf_counter() - t) * (self.context / tokens) * self.batch
        return dt, self.step_bytes, self.batch


class Packed(Decode):
    """vLLM-layout packed decode, B=256, lengths U[512, 8192];
    every rank its own batch (weak scaling)."""

    name = "packed"

    def __init__(self, torch, C, device, rank, world, batch=0, **_):
        self.torch, self.C, self.device = torch, C, device
        batch = batch or 256
        rng = np.random.default_rng(256 + rank)
        lens = rng.integers(512, 8193, size=batch).astype(np.int32)
        npg = (lens + 15) // 16
        nb, mp = int(npg.sum()), int(npg.max())
        perm = rng.permutation(nb).astype(np.int32)
        pages = np.full((batch, mp), -1, np.int32)
        cur = 0
        for b in range(batch):
            pages[b, :npg[b]] = perm[cur:cur + npg[b]]
            cur += npg[b]
        g = torch.Generator(device=device)
        g.manual_seed(4 + rank)
        self.cache = torch.randn(nb, 2, 16, 8, 128, device=device, dtype=torch.float16,
                                 generator=g)
        self.pages = torch.from_numpy(pages).to(device)
        self.lengths = torch.from_numpy(lens).to(device)
        self.lens = lens
        self.batch = batch
        self.nb, self.mp = nb, mp
        self.shape = C.make_shape(batch, 32, 8, 128, mp, nb)
        self.q_host = torch.randn(batch, 32, 128, dtype=torch.float16).pin_memory()
        self.q = self.q_host.to(device)
        self.out = torch.empty(batch, 32, 128, device=device, dtype=torch.float16)
        self.out_host = torch.empty(self.out.shape, dtype=torch.float16).pin_memory()
        self.launches = self.kernel_launches = 1
        rows = batch * 32
        self.kernel_bytes = int(lens.sum()) * 4096 + rows * 128 * 2 * 2 + batch * mp * 4
        self.step_bytes = self.kernel_bytes
        self.kernel = "attn_kernel (packed decode)"
        self.bound = "hbm"

    def device_step(self):
        self.C.packed_decode_kv(self.shape, self.q, self.cache, self.pages, self.lengths,
                                self.out, 2 * 16 * 8 * 128, 128, 8 * 128, 16 * 8 * 128, SCALE, 0)

    kernel_step = device_step

    def io_bytes(self):
        return self.q_host.numel() * 2, self.out_host.numel() * 2

    def config(self):
        return {"workload": "BASELINE config 4: vLLM-layout [num_blocks,2,16,8,128] packed "
                            "decode, batch 256, lengths U[512,8192] (seeded)",
                "tokens": int(self.lens.sum()), "kv_bytes": int(self.lens.sum()) * 4096}

    def cpu_baseline(self, requests=8):
        O = oracle_module()
        torch = self.torch
        # the first `requests` requests, their pages copied to a compact host cache
        pages = self.pages[:requests].cpu().numpy()
        used = sorted({int(p) for p in pages.ravel() if p >= 0})
        remap = {p: i for i, p in enumerate(used)}
        cache = half_bits(torch, self.cache[torch.tensor(used, device=self.device)])
        pages = np.vectorize(lambda p: remap.get(int(p), -1))(pages).astype(np.int32)
        q = half_bits(torch, self.q[:requests])
        s = (requests, 32, 8, 128, pages.shape[1], len(used))
        t = time.perf_counter()
        O.packed_decode(s, q, cache, pages, self.lens[:requests], 2 * 16 * 8 * 128, 128,
                        8 * 128, 16 * 8 * 128, SCALE, threads=O.max_threads())
        dt = time.perf_counter() - t
        return {"value": requests / dt, "unit": self.unit, "cores": O.max_threads(),
                "kind": "port", "sample": f"the first {requests} requests of the batch",
                "seconds": round(dt, 4)}

    def reference_step(self, pool):
        return None


class TreeScale(Workload):
    """BASELINE config 5a: 1024 requests (whole 16-request prefix groups split
    across ranks), each a 63-node full binary tree over a 4096-token prefix
    shared by its group; FP16 output. Tensor-bound: value = whole-job
    TFLOP/s."""

    name = "tree-scale"
    unit = "TFLOP/s"
    scaling = "strong"

    def __init__(self, torch, C, device, rank, world, total=1024, group=16, prefix=4096,
                 nodes=63, batch=0, **_):
        from bc_dist import shard_requests

        # (--batch: fewer requests, whole groups; for small profiling runs)
        total = max(group, batch // group * group) if batch else total
        self.total = total
        self.torch, self.C, self.device = torch, C, device
        reqs = shard_requests(total // group, world, rank)  # whole prefix groups
        ngroups = len(reqs)
        B = ngroups * group
        self.B, self.N, self.prefix, self.group = B, nodes, prefix, group
        npg = prefix // 16
        P = ngroups * npg + 8
        g = torch.Generator(device=device)
        g.manual_seed(55 + rank)
        self.k = torch.randn(P, 16, 8, 128, device=device, dtype=torch.float16, generator=g)
        self.v = torch.randn(P, 16, 8, 128, device=device, dtype=torch.float16, generator=g)
        perm = torch.randperm(P, device=device, generator=g).to(torch.int32)
        gp = perm[:ngroups * npg].view(ngroups, npg)
        self.pages = gp.repeat_interleave(group, dim=0).contiguous()
        self.lengths = torch.full((B,), prefix, device=device, dtype=torch.int32)
        self.dq = torch.randn(B, nodes, 32, 128, device=device, dtype=torch.float16, generator=g)
        self.dk = torch.randn(B, nodes, 8, 128, device=device, dtype=torch.float16, generator=g)
        self.dv = torch.randn(B, nodes, 8, 128, device=device, dtype=torch.float16, generator=g)
        par = [-1] + [(n - 1) // 2 for n in range(1, nodes)]
        self.parent = torch.tensor([par] * B, device=device, dtype=torch.int32)
        self.shape = C.make_shape(B, 32, 8, 128, npg, P)
        self.out = torch.empty(B, nodes, 32, 128, device=device, dtype=torch.float16)
        depth_sum = sum(int(math.log2(n + 1)) + 1 for n in range(nodes))
        self.flops = 32 * 4 * 128 * B * (nodes * prefix + depth_sum)
        self.unique_bytes = (ngroups * prefix * 4096 + B * nodes * 8 * 128 * 4
                             + B * nodes * 32 * 128 * 4 + B * npg * 4)
        self.kernel_bytes = self.unique_bytes
        self.launches = 1
        self.kernel = "tree_mma_kernel (tree_verify, FP16 out)"
        self.bound = "tensor"
        # end-to-end leg: this step's draft tensors and tables from pinned host
        # memory, the FP16 verification output back
        self.host = {n: getattr(self, n).cpu().pin_memory()
                     for n in ("dq", "dk", "dv", "parent", "pages", "lengths")}
        self.out_host = torch.empty(self.out.shape, dtype=torch.float16).pin_memory()

    def device_step(self):
        self.C.tree_verify(self.shape, self.dq, self.k, self.v, self.pages, self.lengths,
                           self.dk, self.dv, self.parent, self.out, self.N)

    kernel_step = device_step

    def e2e_step(self):
        for n, t in self.host.items():
            getattr(self, n).copy_(t, non_blocking=True)
        self.device_step()
        self.out_host.copy_(self.out, non_blocking=True)

    def io_bytes(self):
        return (sum(t.numel() * t.element_size() for t in self.host.values()),
                self.out_host.numel() * 2)

    def value(self, steps_all_ranks, seconds):
        return self.flops * steps_all_ranks / seconds / 1e12

    def config(self):
        return {"workload": f"BASELINE config 5a: tree_verify, {self.total} requests x 63-node "
                            "full binary trees, 4096-token prefix shared per 16 requests, FP16 out"
                            + ("" if self.total == 1024 else " (a reduced batch, not the config)"),
                "requests_per_gpu": self.B, "flops_per_step": self.flops,
                "unique_bytes_per_step": self.unique_bytes,
                "parallelism": "request-sharded (whole prefix groups)"}

    def cpu_baseline(self):
        O = oracle_module()
        torch = self.torch
        npg = self.prefix // 16
        ids = self.pages[0].long()
        k, v = half_bits(torch, self.k[ids]), half_bits(torch, self.v[ids])
        s = (1, 32, 8, 128, npg, npg)
        pages = np.arange(npg, dtype=np.int32).reshape(1, -1)
        t = time.perf_counter()
        O.tree(s, self.N, half_bits(torch, self.dq[:1]), k, v, pages,
               np.array([self.prefix], np.int32), half_bits(torch, self.dk[:1]),
               half_bits(torch, self.dv[:1]), self.parent[:1].cpu().numpy(),
               threads=O.max_threads())
        dt = time.perf_counter() - t
        return {"value": (self.flops / self.B) / dt / 1e12, "unit": self.unit,
                "cores": O.max_threads(), "kind": "port",
                "sample": "1 request (63 nodes x 4096-token prefix)", "seconds": round(dt, 4)}


class LongCtx(Workload):
    """BASELINE config 5b: one request of 1,048,576 tokens; rank r holds a
    contiguous 1/world shard of its pages and reduces it to FP32 partials
    (m, l, acc), `splits` of them per q-head. With more than one rank, ONE
    kernel per rank (bc_merge_exchange) reduces them to one state per q-head,
    writes it into every rank's exchange buffer over NVLink (peer memory,
    mapped once through CUDA IPC), waits on the device for the peers' flags and
    merges the world's states; the NCCL form of the same step (reduction, one
    all-gather of 16,640 bytes per rank, merge) is timed beside it. value =
    tokens/s (one decoded token per job step); strong scaling."""

    name = "longctx"
    unit = "tokens/s"
    scaling = "strong"

    def __init__(self, torch, C, device, rank, world, total=1 << 20, splits=0, context=0, **_):
        from bc_dist import block_floats, block_views, shard_pages

        total = context or total  # (--context: a shorter context, for profiling runs)

        self.torch, self.C, self.device, self.world = torch, C, device, world
        npg_total = total // 16
        mine = shard_pages(npg_total, world, rank)
        npg = len(mine)
        g = torch.Generator(device=device)
        g.manual_seed(77 + rank)
        P = npg + 8
        self.k = torch.randn(P, 16, 8, 128, device=device, dtype=torch.float16, generator=g)
        self.v = torch.randn(P, 16, 8, 128, device=device, dtype=torch.float16, generator=g)
        perm = torch.randperm(P, device=device, generator=g).to(torch.int32)
        self.pages = perm[:npg].view(1, npg).contiguous()
        self.lengths = torch.tensor([npg * 16], device=device, dtype=torch.int32)
        self.shape = C.make_shape(1, 32, 8, 128, npg, P)
        # enough CTAs (8 KV heads x splits) for two per SM unless told otherwise
        self.splits = splits or min(C.MAX_SPLITS, max(9, -(-2 * 148 // 8)))
        self.S = self.splits if self.splits > 8 else 1
        gq = torch.Generator()
        gq.manual_seed(5)
        self.q_host = torch.randn(1, 32, 128, dtype=torch.float16, generator=gq).pin_memory()
        self.q = self.q_host.to(device)
        self.out_host = torch.empty(1, 32, 128).pin_memory()
        # this rank's splits; with more than one rank they are reduced to ONE
        # partial per row (bc_merge_to_partial) in the buffer that is gathered
        self.part = torch.empty(block_floats(self.S, 32, 128), device=device)
        self.pml, self.pa = block_views(self.part, self.S, 32, 128)
        self.buf = torch.empty(block_floats(1, 32, 128), device=device)
        self.send_ml, self.send_a = block_views(self.buf, 1, 32, 128)
        self.gathered = torch.empty(world, self.buf.numel(), device=device)
        self.out = torch.empty(32, 128, device=device)
        self.total = total
        self.kernel_bytes = npg * 16 * 4096 + 32 * 128 * 2 + self.S * 32 * 130 * 4
        self.step_bytes = self.kernel_bytes
        # partial decode, then the exchange kernel (world > 1) or the merge
        self.launches = 2
        self.kernel = "attn_kernel (paged decode partial)"
        self.bound = "hbm"
        self.group = self.exchange = None
        if world > 1:
            from bc_dist import PeerExchange, exchange_group

            self.group = exchange_group()
            self.exchange = PeerExchange(32, 128, group=self.group)

    def kernel_step(self):
        self.C.paged_decode_partial(self.shape, self.q, self.k, self.v, self.pages, self.lengths,
                                    self.pml, self.pa, self.splits)

    def device_step(self):
        self.kernel_step()
        if self.world > 1:
            self.exchange.merge(self.pml, self.pa, self.out)
        else:
            self.C.merge_gathered(self.part.view(1, -1), 1, self.S, 32, 128, self.out)

    def nccl_step(self):
        import torch.distributed as dist

        self.kernel_step()
        if self.S > 1:
            self.C.merge_to_partial(self.pml, self.pa, self.send_ml[0], self.send_a[0])
        else:
            self.buf.copy_(self.part)
        dist.all_gather_into_tensor(self.gathered, self.buf, group=self.group)
        self.C.merge_gathered(self.gathered, self.world, 1, 32, 128, self.out)

    def alt_steps(self):
        if self.world == 1:
            return {}
        return {"the same step with an NCCL all-gather instead of the peer-memory exchange "
                "(reduction, all_gather_into_tensor, merge)": (self.nccl_step, 2 + (self.S > 1))}

    def e2e_step(self):
        self.q.copy_(self.q_host, non_blocking=True)
        self.device_step()
        self.out_host.view(32, 128).copy_(self.out, non_blocking=True)

    def io_bytes(self):
        return self.q_host.numel() * 2, self.out_host.numel() * 4

    def value(self, steps_all_ranks, seconds):
        return (steps_all_ranks / self.world) / seconds  # one token per job step

    def config(self):
        return {"workload": f"BASELINE config 5b: one request, {self.total:,}-token context split "
                            "across ranks, each rank's FP32 partial states sent to every rank "
                            "over peer memory and merged on the device in one kernel"
                            + ("" if self.total == 1 << 20 else " (a shorter context, not the config)"),
                "tokens_per_gpu": int(self.lengths[0]), "splits_per_gpu": self.splits,
                "parallelism": f"context-split x{self.world}",
                "exchange": ("peer memory (bc_merge_exchange: NVLink stores through CUDA IPC, "
                             "device-side flags)" if self.world > 1 else "none"),
                "exchange_bytes_per_rank_to_each_peer": 32 * 132 * 4 if self.world > 1 else 0}

    def release(self):
        if getattr(self, "exchange", None) is not None:
            self.exchange.close()
        if getattr(self, "group", None) is not None:
            import torch.distributed as dist

            dist.destroy_process_group(self.group)
        super().release()

    def cpu_baseline(self, tokens=65536):
        O = oracle_module()
        torch = self.torch
        npg = tokens // 16
        ids = self.pages[0, :npg].long()
        k, v = half_bits(torch, self.k[ids]), half_bits(torch, self.v[ids])
        s = (1, 32, 8, 128, npg, npg)
        t = time.perf_counter()
        O.decode(s, half_bits(torch, self.q), k, v, np.arange(npg, dtype=np.int32).reshape(1, -1),
                 np.array([tokens], np.int32), threads=O.max_threads())
        dt = (time.perf_counter() - t) * self.total / tokens
        return {"value": 1 / dt, "unit": self.unit, "cores": O.max_threads(), "kind": "port",
                "sample": f"a {tokens}-token slice, scaled linearly to {self.total} tokens",
                "seconds": round(dt, 4)}


WORKLOADS = {w.name: w for w in (TreeCow, TreeOracle, TreeHbm, Decode, Packed, TreeScale, LongCtx)}
# Measured after the headline in the default run, each under line["configs"].
EXTRAS = ("tree-oracle", "decode", "packed", "tree-scale", "longctx")


# --------------------------------------------------------------- our arm
class Harness:
    """Process-group plumbing and the timed-region protocol shared by every
    workload of one run."""

    def __init__(self, torch, world, rank, device, repeats):
        self.torch, self.world, self.rank, self.device = torch, world, rank, device
        self.repeats = repeats
        self.hbm_peak, self.tensor_peak, self.peak_kind = load_peaks()

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, values):
        if self.world == 1:
            return list(values)
        import torch.distributed as dist

        t = self.torch.tensor(values, device=self.device, dtype=self.torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t]

    def measure(self, wl, steps, warmup, sampler, with_cpu):
        torch, C = self.torch, wl.C
        stream = torch.cuda.current_stream()
        for _ in range(warmup):
            wl.device_step()
            wl.kernel_step()
            wl.e2e_step()
        torch.cuda.synchronize()
        if C.last_device_error() != 0:
            raise SystemExit(f"device error word set during {wl.name} warm-up")
        wl.prepare()
        for _ in range(2):  # the captured form, once more untimed
            wl.device_step()
        torch.cuda.synchronize()
        R = self.repeats
        dev, kern, e2e = [], [], []
        t0 = time.time()
        for _ in range(R):
            self.barrier()
            dev.append(region(torch, wl.device_step, steps, stream))
        for _ in range(R):
            self.barrier()
            kern.append(region(torch, wl.kernel_step, steps, stream))
        alts = wl.alt_steps() if hasattr(wl, "alt_steps") else {}
        alt_ms = {}
        for name, (fn, _) in alts.items():
            ms = []
            for _ in range(R):
                self.barrier()
                ms.append(region(torch, fn, steps, stream))
            alt_ms[name] = ms
        for _ in range(R):
            self.barrier()
            if hasattr(wl, "e2e_region"):
                e2e.append(wl.e2e_region(steps))
            else:
                e2e.append(region(torch, wl.e2e_step, steps, stream))
        self.barrier()
        t1 = time.time()
        err = C.last_device_error()
        alt_flat = [x for ms in alt_ms.values() for x in ms]
        allv = self.max_over_ranks(dev + kern + e2e + alt_flat + [float(err)])
        dev, kern, e2e, err = allv[:R], allv[R:2 * R], allv[2 * R:3 * R], int(allv[-1])
        alt_all = allv[3 * R:-1]
        alt_ms = {name: alt_all[i * R:(i + 1) * R] for i, name in enumerate(alt_ms)}
        dev_ms, kern_ms, e2e_ms = (statistics.median(x) for x in (dev, kern, e2e))
        world = self.world
        value = wl.value(steps * world, dev_ms * 1e-3)
        e2e_value = wl.value(steps * world, e2e_ms * 1e-3)
        kern_us = kern_ms * 1e3 / steps
        if wl.bound == "tensor":
            achieved = wl.flops / (kern_us * 1e-6) / 1e12
            roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": self.tensor_peak,
                    "unit": "TFLOP/s", "frac": round(achieved / self.tensor_peak, 4),
                    "peak_source": f"{self.peak_kind} bf16_tflops (FP16 = BF16 rate)"}
        else:
            achieved = wl.kernel_bytes / (kern_us * 1e-6) / 1e9
            roof = {"bound": "hbm", "achieved": round(achieved, 2), "peak": self.hbm_peak,
                    "unit": "GB/s", "frac": round(achieved / self.hbm_peak, 4),
                    "peak_source": f"{self.peak_kind} hbm_gbs"}
        roof["kernel"] = wl.kernel
        roof["kernel_us"] = round(kern_us, 3)
        roof["timing"] = (f"median of {R} regions of {steps} back-to-back launches through the "
                          "C ABI, one event pair per region")
        roof["traffic"] = NCU_TRAFFIC.get(wl.name)
        h2d, d2h = wl.io_bytes()
        cfg = wl.config()
        cfg["l2"] = wl.l2_note()
        cfg.setdefault("parallelism", f"request-sharded x{world}")
        out = {
            "value": round(value, 6), "unit": wl.unit, "higher_is_better": wl.higher_is_better,
            "scaling": wl.scaling, "ms_per_step": round(dev_ms / steps, 6),
            "ms_per_step_regions": [round(x / steps, 6) for x in dev],
            "step_form": wl.step_form(),
            "config": cfg,
            "e2e": {"value": round(e2e_value, 6), "unit": wl.unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / steps, 6),
                    "mode": wl.e2e_form()},
            "gpu_launches": R * steps * (2 * wl.launches + wl.kernel_launches
                                         + sum(n for _, n in alts.values())),
            "roofline": roof, "clocks": sampler.window(t0, t1), "device_error_word": err,
        }
        if alt_ms:
            out["alternative_steps"] = {
                name: {"ms_per_step": round(statistics.median(ms) / steps, 6),
                       "value": round(wl.value(steps * world, statistics.median(ms) * 1e-3), 6)}
                for name, ms in alt_ms.items()}
        if with_cpu:
            cb = wl.cpu_baseline()
            cb["value"] = float(f"{cb['value']:.6g}")
            out["cpu_baseline"] = cb
        return out


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

    h = Harness(torch, world, rank, device, args.repeats)
    sampler = ClockSampler(device.index)
    time.sleep(0.3)
    with_cpu = world == 1 and not args.no_cpu_baseline
    kw = dict(batch=args.batch, context=args.context, splits=args.splits)
    wl = WORKLOADS[args.workload](torch, C, device, rank, world, **kw)
    head = h.measure(wl, args.steps, args.warmup, sampler, with_cpu and rank == 0)
    if args.batch or args.context or args.splits or args.traffic is not None:
        head["roofline"]["traffic"] = args.traffic
    wl.release()
    del wl
    torch.cuda.empty_cache()
    extras = {}
    if args.workload == "tree-cow" and not args.no_extras:
        for name in EXTRAS:
            w = WORKLOADS[name](torch, C, device, rank, world)
            extras[name] = h.measure(w, args.steps, args.warmup, sampler, with_cpu and rank == 0)
            w.release()
            del w
            torch.cuda.empty_cache()
    sampler.stop()
    if rank == 0:
        line = {"metric": METRIC, "value": head["value"], "unit": head["unit"],
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "repeats": args.repeats, "ms_per_step": head["ms_per_step"],
                "higher_is_better": head["higher_is_better"], "scaling": head["scaling"],
                "vs_baseline": None, "dtype": "f16 in / f32 accumulate",
                "data": "synthetic (seeded N(0,1) FP16, per-rank seed)"}
        line.update({k: v for k, v in head.items() if k not in line})
        line["gpu_launches"] = head["gpu_launches"] + sum(
            e["gpu_launches"] for e in extras.values())
        if extras:
            line["configs"] = extras
        emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------- reference arm
def _reference_gpu(torch, O, steps, warmup, repeats):
    """The reference's own GPU kernels (its src/*.cu compiled unmodified for
    sm_100a into oracle/_ref/libbcref.so) on the inputs of configs 1-4, each
    the median of `repeats` regions of `steps` calls, one event pair each."""
    import bc_capi as C
    from bc_cow import PagePool

    ref = O.ref()
    vp = ctypes.c_void_p
    P = C._ptr
    stream = torch.cuda.current_stream()
    st = vp(stream.cuda_stream)
    device = torch.device("cuda", 0)
    out = {}

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        ms = [region(torch, fn, steps, stream) for _ in range(repeats)]
        return statistics.median(ms) / steps

    def shape_of(s):
        return O.Shape(s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages)

    # config 2: tree verify + the per-request COW commits as the reference's
    # PagedTreeCache.commit issues them (a page copy, then commit_path)
    wl = TreeCow(torch, C, device, 0, 1)
    s = shape_of(wl.shape)
    pool = PagePool(wl.wl.pool_pages)
    reqs = [pool.new(wl.wl.prefix)] + [pool.fork(0) for _ in range(wl.wl.batch - 1)]
    per_req = []
    page_bytes = 16 * 8 * 128 * 2
    for b in range(wl.wl.batch):
        plan = pool.plan_commit_batch([(reqs[b], wl.wl.paths[b], b)], wl.nodes)
        arr = [torch.tensor(x, dtype=torch.int32, device=device)
               for x in (plan.entry_node, plan.entry_page, plan.entry_slot)]
        per_req.append((list(zip(plan.clone_src, plan.clone_dst)), arr))
    rt = CudaRt()
    rot = [0]

    def step2():
        c = rot[0]
        rot[0] = (c + 1) % wl.copies
        d = wl.ios[c].dev
        ck, cv = wl.caches[c]
        assert ref.bcr_gpu_tree_verify(ctypes.byref(s), wl.nodes, P(d["draft_q"]), P(ck), P(cv),
                                       P(d["pages"]), P(d["lengths"]), P(d["draft_k"]),
                                       P(d["draft_v"]), P(d["parent"]), P(wl.outs[c]), st) == 0
        for b, (clones, (nodes_t, pages_t, slots_t)) in enumerate(per_req):
            for src, dst in clones:
                for t in (ck, cv):
                    rt.copy(t.data_ptr() + dst * page_bytes, t.data_ptr() + src * page_bytes,
                            page_bytes, 3, st)
            assert ref.bcr_gpu_commit_path(ctypes.byref(s), P(d["draft_k"]), P(d["draft_v"]),
                                           P(ck), P(cv), P(nodes_t), P(pages_t), P(slots_t), b,
                                           wl.nodes, int(nodes_t.numel()), st) == 0

    ms = timed(step2)
    out["tree-cow"] = {"ms_per_step": round(ms, 6), "value": round(wl.step_bytes / ms / 1e9, 6),
                       "unit": "TB/s",
                       "what": "reference tree_kernel + per request a page copy and "
                               "commit_kernel (8 commit launches, 14 page copies)"}
    wl.release()

    # config 1 (the reference returns FP32; ours is timed with FP16 output)
    wl = TreeOracle(torch, C, device, 0, 1)
    s = shape_of(wl.shape)
    out32 = torch.empty(wl.out_shape, device=device)
    rot[0] = 0

    def step1():
        c = rot[0]
        rot[0] = (c + 1) % wl.copies
        d = wl.ios[c].dev
        ck, cv = wl.caches[c]
        assert ref.bcr_gpu_tree_verify(ctypes.byref(s), wl.nodes, P(d["draft_q"]), P(ck), P(cv),
                                       P(d["pages"]), P(d["lengths"]), P(d["draft_k"]),
                                       P(d["draft_v"]), P(d["parent"]), P(out32), st) == 0

    ms = timed(step1)
    out["tree-oracle"] = {"ms_per_step": round(ms, 6),
                          "value": round(wl.step_bytes / ms / 1e9, 6), "unit": "TB/s",
                          "what": "reference tree_kernel (FP32 output)"}
    wl.release()

    # config 3 at 4 x 131072: the reference caps the split count at 16
    wl = Decode(torch, C, device, 0, 1)
    s = shape_of(wl.shape)
    splits = min(16, int(ref.bcr_gpu_auto_splits(ctypes.byref(s), wl.context, 148)))
    splits = max(splits, 1)
    pa = torch.empty(splits * wl.batch * 32 * 128, device=device)
    pml = torch.empty(splits * wl.batch * 32 * 2, device=device)

    def step3():
        assert ref.bcr_gpu_decode(ctypes.byref(s), P(wl.q), P(wl.k), P(wl.v), P(wl.pages),
                                  P(wl.lengths), P(wl.out), P(pa), P(pml), splits, st) == 0

    ms = timed(step3)
    out["decode"] = {"ms_per_step": round(ms, 6), "value": round(wl.batch / ms * 1e3, 3),
                     "unit": "tokens/s", "splits": splits,
                     "what": "reference decode_kernel + merge_kernel"}
    wl.release()

    # config 4: the same values in the reference's packed layout [P, Hkv, 16, 2D]
    # (V at +D), which the reference kernel requires
    wl = Packed(torch, C, device, 0, 1)
    refcache = wl.cache.permute(0, 3, 2, 1, 4).contiguous()  # [nb, 8, 16, 2, 128]
    wl.cache = None
    s = shape_of(wl.shape)

    def step4():
        assert ref.bcr_gpu_packed_decode(ctypes.byref(s), P(wl.q), P(refcache), P(wl.pages),
                                         P(wl.lengths), P(wl.out), ctypes.c_longlong(8 * 16 * 256),
                                         ctypes.c_longlong(16 * 256), ctypes.c_longlong(256),
                                         ctypes.c_float(SCALE), st) == 0

    ms = timed(step4)
    out["packed"] = {"ms_per_step": round(ms, 6), "value": round(wl.batch / ms * 1e3, 3),
                     "unit": "tokens/s",
                     "what": "reference packed_decode_kernel on the [P,Hkv,16,2D] layout"}
    del refcache
    wl.release()
    torch.cuda.empty_cache()
    return out


def _reference_sigs(ref):
    vp, i, ll, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float
    ref.bcr_gpu_tree_verify.argtypes = [vp, i] + [vp] * 9 + [vp]
    ref.bcr_gpu_commit_path.argtypes = [vp] + [vp] * 7 + [i, i, i, vp]
    ref.bcr_gpu_decode.argtypes = [vp] + [vp] * 8 + [i, vp]
    ref.bcr_gpu_auto_splits.argtypes = [vp, i, i]
    ref.bcr_gpu_packed_decode.argtypes = [vp] + [vp] * 5 + [ll, ll, ll, f, vp]
    for fn in (ref.bcr_gpu_tree_verify, ref.bcr_gpu_commit_path, ref.bcr_gpu_decode,
               ref.bcr_gpu_auto_splits, ref.bcr_gpu_packed_decode):
        fn.restype = i


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    O = oracle_module()
    if not O.ref_available():
        emit({"impl": "reference", "unavailable": "oracle/_ref/libbcref.so (the reference "
                                                 "built from its sources) is missing"})
        return
    if args.workload not in ("tree-cow", "tree-oracle", "decode"):
        emit({"impl": "reference", "unavailable": f"no reference CPU path measured "
                                                 f"for workload {args.workload}"})
        return
    from concurrent.futures import ThreadPoolExecutor

    import torch

    device = torch.device("cuda", 0) if torch.cuda.is_available() else None
    if args.workload == "tree-cow":
        wl = TreeCow.__new__(TreeCow)
        from bc_workloads import TreeCowWorkload

        wl.wl = TreeCowWorkload(seed=2040)
        wl.plan, _ = wl.wl.plan()
        wl.step_bytes = wl.wl.verify_bytes() + wl.wl.commit_bytes(wl.plan)
        unit = TreeCow.unit
    else:
        if device is None:
            emit({"impl": "reference", "unavailable": "this workload's inputs are "
                                                     "generated on a GPU"})
            return
        import bc_capi as C

        wl = WORKLOADS[args.workload](torch, C, device, 0, 1)
        unit = wl.unit
    cores = min(8, os.cpu_count() or 1)
    times, bytes_, units = [], 0, 0
    with ThreadPoolExecutor(max_workers=cores) as pool:
        for _ in range(args.warmup):
            wl.reference_step(pool)
        for _ in range(args.steps):  # bounded: stop once the CPU budget is spent
            dt, b, u = wl.reference_step(pool)
            times.append(dt)
            bytes_ += b
            units += u
            if sum(times) > args.reference_budget_s:
                break
    total = sum(times)
    value = bytes_ / total / 1e12 if unit == "TB/s" else units / total
    line = {
        "impl": "reference", "metric": METRIC, "value": float(f"{value:.6g}"), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / len(times) * 1e3, 3), "steps_timed": len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 in / f64 accumulate (reference CPU oracle)",
        "data": "synthetic (seeded N(0,1) FP16, same inputs as the CUDA arm's rank 0)",
        "config": (TreeCow.config(wl) if args.workload == "tree-cow" else wl.config()),
        "cpu_baseline": {"value": float(f"{value:.6g}"), "unit": unit, "cores": cores,
                         "kind": "reference",
                         "sample": "tree-cow: each step = the full 8-request step (the "
                                   "reference's cpu_tree_reference, one request per host "
                                   "thread, + the sequential COW commits)"
                                   if args.workload == "tree-cow" else
                                   "a bounded slice of the step, scaled linearly"},
        "e2e": {"value": float(f"{value:.6g}"), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if args.workload == "tree-cow":
        # the headline config's l2/parallelism facts, as our arm states them
        line["config"]["l2"] = "CPU arm: host memory (no GPU cache involved)"
        line["config"]["parallelism"] = f"request-sharded x{world}"
    if device is not None and args.workload == "tree-cow" and not args.no_extras:
        try:
            _reference_sigs(O.ref())
            line["reference_gpu_sm100a"] = _reference_gpu(torch, O, args.steps, args.warmup,
                                                         args.repeats)
        except Exception as e:  # reported, never fatal to the CPU arm's line
            line["reference_gpu_sm100a"] = {"unavailable": f"{type(e).__name__}: {e}"}
    emit(line)


RESULT_OUT = sys.stdout


def emit(line):
    """Print the run's one JSON line on the real standard output."""
    print(json.dumps(line), file=RESULT_OUT, flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--repeats", type=int, default=7,
                    help="timed regions per measurement (the median is reported; 7, the "
                         "reference's protocol)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="tree-cow")
    ap.add_argument("--no-extras", action="store_true",
                    help="measure only the chosen workload (no `configs` key)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu-measured DRAM bytes per launch of the dominant kernel, if known")
    ap.add_argument("--batch", type=int, default=0, help="decode/packed batch (0: config's)")
    ap.add_argument("--context", type=int, default=0,
                    help="decode context tokens (0: 131072); longctx: the context (0: 1,048,576)")
    ap.add_argument("--splits", type=int, default=0, help="decode/longctx KV splits (0: auto)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reference-budget-s", type=float, default=60.0,
                    help="CPU seconds after which the reference arm stops timing steps")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"tree-cow": 200, "tree-oracle": 200}.get(args.workload, 20)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.repeats < 1:
        ap.error("--repeats must be at least 1")
    # stdout carries exactly the one JSON line: anything else written to file
    # descriptor 1 (library banners such as NCCL's version line) goes to stderr.
    global RESULT_OUT
    RESULT_OUT = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
