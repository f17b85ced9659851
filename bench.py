"""Benchmark of the DVAttn paged decode on B200 (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload: BASELINE config 2 (bf16 batched paged decode, W=32, 64/4 heads, E=128,
R=64, KV lengths U[512, 8192] in two turns, page 16).  A step is one call of the op over
one batch (one layer-step).  Metric: algorithmic HBM GB/s of the op (attended K/V rows +
q + out + cos/sin + tables), and microseconds per layer-step.

* value: device-resident inputs, K calls of the C ABI (libdvattn_b200.so) captured once
  in a CUDA graph and replayed, timed with CUDA events on the launching stream; the rep
  of K steps is repeated (>= 25 reps, ~1 s) and the median rep is reported with its
  spread; between steps the call rotates over three copies of the KV page pool (each
  larger than the 126 MB L2), so no step reads K/V from L2 left by the previous one.
* e2e: the same metric through the public torch op (torch.ops.libdvatt.dvattn_paged_sdpa)
  with every step's inputs (q, cos/sin, locations, fragment lengths, block tables) copied
  from pinned host memory and its output copied back inside the timed region (H2D issued
  in groups of 1, 2, 4, 8 steps ahead of the compute, D2H right after each op); the KV cache stays
  resident, as in a serving engine.
* roofline: the attention kernel alone (C-ABI phase ATTEND between CUDA events), against
  the measured HBM copy bandwidth of MEASURED_PEAKS.json.
* cpu_baseline: the reference's pure-PyTorch path (oracle restatement of
  dvattn_sdpa_pt + apply_rotary_pos_emb) on a bounded sample, on rank 0 only.
* strong_scaling (default workload): config 2's batch split over the ranks (N > 1), and
  config 3's long context split by KV chunk with the partials exchanged over peer memory
  (dvattn_lse_merge_peers; the NCCL all-gather path timed beside it), each with its
  efficiency against the same work on one GPU.
* prefill_config4 (default workload): config 4 on the tensor-core prefill kernel, TFLOP/s
  of whole calls and of the kernel alone against the measured bf16 peak.
* Multi-GPU (torchrun): value is weak scaling -- every rank decodes its own batch of the
  same shape, no collective on the data path; value = all ranks' bytes / max-over-ranks
  time.  --workload long3: config 3 KV-chunk-sharded alone, one JSON line.
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

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attn HBM GB/s (% of peak) and µs/layer-step at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def _wl():
    """dvattn_b200/workloads.py loaded by file path: the seeded input generators (torch and
    numpy only).  Importing it this way does not run the package's __init__, so the
    reference arm never loads this repository's native libraries."""
    import importlib.util
    name = "dvattn_b200_workloads"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "dvattn_b200", "workloads.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


WORKLOAD_DESC = {
    "config1": "config1: fp32 W=1 Hq=16 Hkv=1 E=128 R=64 L=1024 BS=16",
    "config2": "config2: bf16 batched paged decode W=32 Hq=64 Hkv=4 E=128 R=64 BS=16 2 turns",
    "config3": "config3: fp16 long context W=4 Hq=128 Hkv=8 E=128 R=128 L=131072 BS=64",
    "config5": "config5: fp16 serving mix W=256 Hq=32 Hkv=2 E=256 R=64 BS=64 1-4 turns",
}


def paged_config(name: str, nbytes: int, world: int, pool_bytes: int) -> dict:
    """The `config` object of a paged-decode bench line (identical in both arms)."""
    return {"workload": WORKLOAD_DESC[name], "bytes_per_step_per_gpu": nbytes,
            "parallelism": f"batch-replica x{world}",
            "l2": "inputs larger than L2: 3 rotating KV pools of %.0f MB each" % (pool_bytes / 1e6)}


def timed_reps(step, steps: int, world: int, stream, min_reps: int = 25, min_s: float = 1.0):
    """Time `steps` calls of step(i) between CUDA events on `stream`, repeated: at least
    `min_reps` times and until about `min_s` seconds of timed work (the rep count is agreed
    over the ranks).  Each rep is bracketed by a barrier and a device synchronise; its
    duration is the max over ranks.  Returns the per-rep ms list and the total wall time."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k = 0

    def rep():
        nonlocal k
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            step(k)
            k += 1
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    first = rep()
    reps = int(max_over_ranks(float(max(min_reps, min(5000, int(min_s * 1e3 / max(first, 1e-3)) + 1))), world))
    times = [first] + [rep() for _ in range(reps - 1)]
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor(times, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times = t.tolist()
    return times


def spread(per_rep_ms, steps: int) -> dict:
    v = sorted(x / steps for x in per_rep_ms)
    q = lambda f: v[min(len(v) - 1, int(f * (len(v) - 1) + 0.5))]  # noqa: E731
    return {"reps": len(v), "min": round(v[0], 5), "p10": round(q(0.1), 5), "median": round(q(0.5), 5),
            "p90": round(q(0.9), 5), "max": round(v[-1], 5), "unit": "ms per step"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def traffic_from_profiles(workload: str):
    """DRAM bytes per launch of the attention kernel from the committed ncu summary
    (profiles/traffic.txt: `<workload> <kernel> <bytes_per_launch>` lines), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) >= 3 and parts[0] == workload and not line.startswith("#"):
            try:
                return int(float(parts[2]))
            except ValueError:
                return None
    return None


def group_starts(nsteps: int, cap: int):
    """Step indices where the H2D groups start: sizes 1, 2, 4, ... up to `cap`, so the first
    group (whose copy nothing can hide) is short and later ones amortise their wait."""
    starts, i, size = [], 0, 1
    while i < nsteps:
        starts.append(i)
        i += size
        size = min(cap, size * 2)
    return starts + [nsteps]


def pipelined_e2e(host_in, out_like, launch, steps, warmup, world, group: int = 8):
    """End-to-end step time through a public API with host inputs and a host result, run
    the way a serving loop runs it: every step's inputs (pinned host tensors, packed into
    one buffer) go to the device in ONE copy on an H2D stream, the op runs on the compute
    stream, and every step's output comes back to pinned host memory on a D2H stream right
    after its op.  The H2D copies are issued in groups of 1, 2, 4, ... up to `group` steps,
    one group ahead of the compute, and the compute stream waits once per group (a wait in
    front of a kernel costs it the programmatic overlap with the kernel before it, so the
    waits are batched); device buffers form a ring of at least two groups; the K steps are
    captured once in a CUDA graph and replayed.  Every step's H2D and D2H copy is inside the
    timed region.  `launch(dev_inputs, out, i)` enqueues the op on the current stream.
    Returns (ms per step, H2D bytes, D2H bytes per step, mode)."""
    dev = out_like.device
    sizes = [t.numel() * t.element_size() for t in host_in]
    offs, n = [], 0
    for b in sizes:
        offs.append(n)
        n += (b + 255) // 256 * 256
    host_flat = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    for t, o, b in zip(host_in, offs, sizes):
        host_flat[o:o + b].copy_(t.contiguous().reshape(-1).view(torch.uint8))
    out_b = out_like.numel() * out_like.element_size()
    # device buffers: a ring of R steps (at least two of the largest groups), all K steps
    # when they fit in ~1 GB
    fit = max(1, (1 << 30) // (n + out_b))
    R = max(2 * group, min(steps, fit))
    dev_flat = torch.empty((R, n), dtype=torch.uint8, device=dev)
    views = [[dev_flat[k][o:o + b].view(t.dtype).view(t.shape) for t, o, b in zip(host_in, offs, sizes)]
             for k in range(R)]
    outs = [torch.empty_like(out_like) for _ in range(R)]
    host_out = [torch.empty(out_like.shape, dtype=out_like.dtype, pin_memory=True) for _ in range(2)]
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def run(nsteps):
        main = torch.cuda.current_stream()
        h2d_s.wait_stream(main)
        d2h_s.wait_stream(main)
        st = group_starts(nsteps, group)
        ngroups = len(st) - 1
        ev_in, ev_op, ev_d2h = [None] * ngroups, [None] * nsteps, [None] * nsteps

        def issue_h2d(g):
            with torch.cuda.stream(h2d_s):
                reuse = st[g + 1] - 1 - R  # last op that read these input buffers
                if reuse >= 0:
                    h2d_s.wait_event(ev_op[reuse])
                for i in range(st[g], st[g + 1]):
                    dev_flat[i % R].copy_(host_flat, non_blocking=True)
                ev_in[g] = torch.cuda.Event()
                ev_in[g].record(h2d_s)

        issue_h2d(0)
        for g in range(ngroups):
            if g + 1 < ngroups:
                issue_h2d(g + 1)  # one group ahead of the compute
            main.wait_event(ev_in[g])
            reuse = st[g + 1] - 1 - R  # last D2H that read these output buffers
            if reuse >= 0:
                main.wait_event(ev_d2h[reuse])
            for i in range(st[g], st[g + 1]):
                launch(views[i % R], outs[i % R], i)
                ev_op[i] = torch.cuda.Event()
                ev_op[i].record(main)
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(ev_op[i])
                    host_out[i % 2].copy_(outs[i % R], non_blocking=True)
                    ev_d2h[i] = torch.cuda.Event()
                    ev_d2h[i].record(d2h_s)
        main.wait_stream(h2d_s)
        main.wait_stream(d2h_s)

    run(warmup)
    torch.cuda.synchronize()
    mode = f"cuda-graph, H2D in groups of 1, 2, 4, ... {group} steps"
    graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run(steps)
        graph.replay()
        torch.cuda.synchronize()
    except Exception:  # capture unsupported for this op: issue eagerly
        graph, mode = None, f"eager, H2D in groups of 1, 2, 4, ... {group} steps"
        torch.cuda.synchronize()
    barrier(world)
    main = torch.cuda.current_stream()
    per_rep = timed_reps((lambda k: graph.replay()) if graph is not None else (lambda k: run(steps)), 1, world,
                         main, min_reps=10, min_s=0.3)
    ms = statistics.median(per_rep) / steps
    return ms, sum(sizes), host_out[0].numel() * host_out[0].element_size(), mode


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms; only the samples taken
    between begin() and end() (the timed region) are summarised."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t0 = None
        self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def begin(self):
        self.t0 = time.time()

    def end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t0 = (self.t0 or 0.0) - 0.025
        t1 = (self.t1 or time.time()) + 0.025
        for ts, ln in self.lines:
            if not t0 <= ts <= t1:
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ------------------------------------------------------------------------------------
# CPU baseline: the reference's pure-PyTorch path on a bounded sample
# ------------------------------------------------------------------------------------
def reference_cpu_work(name: str):
    """The reference's CPU path on workload `name`: (list of call argument tuples for
    oracle.paged_via_sdpa_pt, the case, same_config, description).  Configs 1 and 2 run
    whole, one reference call per sequence with its fragments cut at the sequence's own
    visible length; the larger configs run on a bounded sample."""
    wl = _wl()
    if name in ("config1", "config2"):
        c = wl.config1() if name == "config1" else wl.config2()
        W = c.queries.size(0)
        subs = [(c.scale, c.locations[:, w:w + 1], c.queries[w:w + 1], c.cosines[:, w:w + 1], c.sines[:, w:w + 1],
                 c.fragment_lengths, c.k_cache, c.v_cache, c.block_tables[w:w + 1]) for w in range(W)]
        return subs, c, True, f"the whole workload ({W} sequences, one reference call per sequence)"
    n, desc = CPU_SAMPLE[name]
    c = cpu_case_fn(name)(n)
    return [(c.scale, c.locations, c.queries, c.cosines, c.sines, c.fragment_lengths, c.k_cache, c.v_cache,
             c.block_tables)], c, False, desc


def cpu_sample_gbs(name: str, reps: int = 3):
    """Time the reference's CPU path (reference_cpu_work) on the host cores; returns
    (GB/s, threads, description)."""
    from oracle import dvattn_oracle as O
    wl = _wl()
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    subs, c, _, desc = reference_cpu_work(name)

    def step():
        for a in subs:
            O.paged_via_sdpa_pt(*a, trim=True)

    step()  # warm-up (also the page gather)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    return wl.paged_bytes(c) / statistics.median(ts) / 1e9, threads, desc


# ------------------------------------------------------------------------------------
# workloads
# ------------------------------------------------------------------------------------
def workload_case(name: str, device: str, rank: int = 0, world: int = 1):
    wl = _wl()
    fn = {"config1": wl.config1, "config2": wl.config2, "config3": wl.config3, "config5": wl.config5}.get(name)
    if fn is None:
        raise SystemExit(f"unknown workload {name}")
    return fn(device=device), WORKLOAD_DESC[name]


def cpu_case_fn(name: str):
    wl = _wl()
    if name == "config2":
        return lambda n: wl.make_paged(wl.config2_lengths(2, 32)[:n], Hq=64, Hkv=4, E=128, R=64, BS=16,
                                       dtype=torch.bfloat16, seed=2)
    if name == "config1":
        return lambda n: wl.config1()
    if name in ("config3", "long3"):
        return lambda n: wl.make_paged([[131072 // 16]], Hq=128, Hkv=8, E=128, R=128, BS=64, dtype=torch.float16,
                                       seed=3)
    if name == "config5":
        return lambda n: wl.make_paged(wl.config5_lengths(5, 256)[:n], Hq=32, Hkv=2, E=256, R=64, BS=64,
                                       dtype=torch.float16, seed=5)
    raise SystemExit(name)


CPU_SAMPLE = {"config2": (4, "first 4 of the 32 sequences of config 2"),
              "config1": (1, "config 1 whole"),
              "config3": (1, "1 sequence of 8192 keys (1/16 of one config-3 sequence), 128/8 heads"),
              "long3": (1, "1 sequence of 8192 keys (1/16 of one config-3 sequence), 128/8 heads"),
              "config5": (24, "first 24 of the 256 sequences of config 5")}


def run_reference(args, world, rank):
    """--impl reference: the reference's own CPU implementation of the path (its
    pure-PyTorch dvattn_sdpa_pt + apply_rotary_pos_emb, restated in oracle/) on the host
    cores.  Nothing of this repository's native code is loaded: the inputs come from
    workloads.py loaded by path.  Config 2 (the default) and config 1 run whole; the larger
    configs run on a bounded sample (named in the line, same_config false)."""
    if rank != 0:
        return
    name = "config3" if args.workload == "long3" else args.workload
    if name not in WORKLOAD_DESC:
        print(json.dumps({"impl": "reference", "unavailable": f"no reference arm for workload {args.workload}"}))
        return
    wl = _wl()
    from oracle import dvattn_oracle as O
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    # one reference call per sequence, each sequence's fragments cut at its own visible
    # length (a caller of the eager path holds per-sequence fragments)
    subs, c, same, desc = reference_cpu_work(name)

    def step():
        for a in subs:
            O.paged_via_sdpa_pt(*a, trim=True)

    for _ in range(args.warmup):
        step()
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    nbytes = wl.paged_bytes(c)
    gbs = nbytes / t / 1e9
    pool = (c.k_cache.numel() + c.v_cache.numel()) * c.k_cache.element_size()
    cfg = paged_config(name, nbytes, args.gpus, pool) if same else {"workload": WORKLOAD_DESC[name] + " (sample)",
                                                                   "sample": desc}
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
            "us_per_layer_step": round(t * 1e6, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": str(c.dtype).replace("torch.", ""),
            "data": "synthetic (seeded N(0,1) q/k/v, seeded lengths/turns/page permutation)",
            "config": cfg, "same_config": same,
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    rc = reference_cuda_timing(name) if not args.no_ref_cuda else None
    if rc:
        line["reference_cuda_gpu"] = rc
    print(json.dumps(line), flush=True)


def reference_cuda_timing(name):
    """The reference's own CUDA op (its src/binding.cu built for sm_100a into oracle/_ref)
    on the full workload, in a subprocess (it registers the same torch.ops.libdvatt
    namespace), device-resident inputs, mean over 20 calls.  None when unavailable
    (library not built, no GPU, or a shape its kernels reject: they need E = 128, GQA 16)."""
    import subprocess
    import tempfile
    so = os.path.join(ROOT, "oracle", "_ref", "dvatt_ref.so")
    if not os.path.exists(so) or not torch.cuda.is_available() or name not in ("config1", "config2", "config3"):
        return None
    wl = _wl()
    case = {"config1": wl.config1, "config2": wl.config2, "config3": wl.config3}[name]()
    with tempfile.TemporaryDirectory() as d:
        src, dst = os.path.join(d, "in.pt"), os.path.join(d, "out.pt")
        torch.save(dict(kind="paged", args=case.op_args(None)[1:], out_shape=tuple(case.new_out().shape),
                        dtype=case.dtype), src)
        r = subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "run_ref.py"), src, dst, "20"],
                           capture_output=True, text=True, timeout=900)
        if r.returncode != 0:
            return {"unavailable": (r.stderr.strip().splitlines() or ["failed"])[-1][:200]}
        us = torch.load(dst)["us"]
    return {"value": round(wl.paged_bytes(case) / (us * 1e-6) / 1e9, 2), "unit": "GB/s",
            "us_per_layer_step": round(us, 2),
            "note": "reference's own CUDA op (oracle/_ref, built for sm_100a) on the same config, device inputs"}


def run_ours(args, world, rank, local):
    import dvattn_b200
    from dvattn_b200 import capi
    from dvattn_b200 import workloads as wl
    dev = f"cuda:{local}"
    hbm_peak, _, peak_kind = load_peaks()
    case, desc = workload_case(args.workload, dev, rank, world)
    nbytes = wl.paged_bytes(case)
    # three KV pools (rotation defeats L2 reuse between steps)
    pools = [(case.k_cache, case.v_cache)]
    for i in range(2):
        pools.append((torch.randn_like(case.k_cache, dtype=torch.float32).to(case.dtype),
                      torch.randn_like(case.v_cache, dtype=torch.float32).to(case.dtype)))
    out = case.new_out()
    calls = []
    ws = None
    for kc, vc in pools:
        call = capi.PagedCall(out, case.scale, case.locations, case.queries, case.cosines, case.sines,
                              case.fragment_lengths, kc, vc, case.block_tables, workspace=ws)
        ws = call.workspace
        calls.append(call)
    stream = torch.cuda.current_stream()
    launches_per_step = 3

    # ---- value: device-resident inputs, C-ABI call ----
    for i in range(args.warmup):
        calls[i % 3]()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.begin()
    # K steps captured once in a CUDA graph (as a serving loop issues a decode step) and
    # replayed; each replay is one rep of K steps, repeated (>= 25, ~1 s of work) for the
    # clock record and the spread; value = the median rep
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            calls[i % 3]()
    graph.replay()
    torch.cuda.synchronize()
    per_rep = timed_reps(lambda k: graph.replay(), 1, world, stream)
    t_ms = statistics.median(per_rep) / args.steps
    # the same K calls issued eagerly from the host (no graph), for comparison
    per_rep_eager = timed_reps(lambda i: calls[i % 3](), args.steps, world, stream, min_reps=10, min_s=0.2)
    t_eager = statistics.median(per_rep_eager) / args.steps

    # ---- attention kernel alone (roofline), same stream, events between phases ----
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        c = calls[i % 3]
        c.phase(capi.DVATTN_PHASE_SCHEDULE)
        kev[i][0].record(stream)
        c.phase(capi.DVATTN_PHASE_ATTEND)
        kev[i][1].record(stream)
        c.phase(capi.DVATTN_PHASE_MERGE)
    torch.cuda.synchronize()
    # the attention kernel back to back: consecutive launches overlap (each starts
    # streaming while the previous one drains), which is how the calls run in the loop
    e0b, e1b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0b.record(stream)
    for i in range(args.steps):
        calls[i % 3].phase(capi.DVATTN_PHASE_ATTEND)
    e1b.record(stream)
    torch.cuda.synchronize()
    if sampler:
        sampler.end()
    clocks = sampler.stop() if sampler else None
    k_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    k_ms = max_over_ranks(k_ms, world)
    kb_ms = max_over_ranks(e0b.elapsed_time(e1b), world) / args.steps

    # ---- e2e: public torch op, host (pinned) inputs in, output out (pipelined) ----
    host_in = [t.cpu().pin_memory() for t in (case.queries, case.cosines, case.sines, case.locations,
                                              case.fragment_lengths, case.block_tables)]

    def e2e_launch(d, o, i):
        q, cs, sn, loc, L, bt = d
        kc, vc = pools[i % 3]
        torch.ops.libdvatt.dvattn_paged_sdpa(o, case.scale, loc, q, cs, sn, L, kc, vc, bt)

    e2e_ms, h2d, d2h, e2e_mode = pipelined_e2e(host_in, out, e2e_launch, args.steps, args.warmup, world)

    total_bytes = sum_over_ranks(float(nbytes), world)
    value = total_bytes / (t_ms * 1e-3) / 1e9
    e2e_val = total_bytes / (e2e_ms * 1e-3) / 1e9
    achieved = nbytes / (k_ms * 1e-3) / 1e9

    extra = {}
    if args.workload == "config2" and not args.no_extra:
        # strong scaling (same total work at every N): the batch split over the ranks, and
        # config 3's long context split by KV chunk with its NCCL exchange
        # a failing leg is reported in the line instead of ending the run (both legs make
        # the same collective calls on every rank, so a failure is seen by all of them)
        for key, fn in (("config2_batch", (lambda: batch_strong_scaling(case, world, rank, args.steps))
                         if world > 1 else None),
                        ("long3", lambda: long3_scaling(world, rank, dev, args.steps)),
                        ("prefill_config4", lambda: prefill_leg(dev, 10, 3, world))):
            if fn is None:
                continue
            try:
                extra[key] = fn()
            except Exception as e:  # noqa: BLE001
                torch.cuda.synchronize()
                extra[key] = {"error": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, threads, sdesc = cpu_sample_gbs(args.workload)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sdesc}
    if rank == 0:
        traffic = traffic_from_profiles(args.workload)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms, 5), "us_per_layer_step": round(t_ms * 1e3, 2),
            "pct_of_peak_hbm": round(100.0 * value / world / hbm_peak, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": str(case.dtype).replace("torch.", ""),
            "data": "synthetic (seeded N(0,1) q/k/v, seeded lengths/turns/page permutation)",
            "config": paged_config(args.workload, nbytes, world,
                                   (case.k_cache.numel() + case.v_cache.numel()) * case.k_cache.element_size()),
            "timing": dict(spread(per_rep, args.steps), value_from="median rep; each rep = one CUDA-graph replay "
                           "of the K C-ABI calls between CUDA events after a barrier and a synchronise, max over "
                           "ranks", us_per_step_eager=round(t_eager * 1e3, 2)),
            "roofline": {"bound": "hbm", "kernel": "decode_row_kernel" if case.dtype != torch.float32 else
                         "decode_f32_kernel", "achieved": round(achieved, 2), "peak": hbm_peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "kernel_us": round(k_ms * 1e3, 2), "traffic": traffic,
                         "timing": "achieved/kernel_us: one launch between CUDA events (isolated); "
                                   "back_to_back: K launches in a row, which overlap",
                         "kernel_us_back_to_back": round(kb_ms * 1e3, 2),
                         "achieved_back_to_back": round(nbytes / (kb_ms * 1e-3) / 1e9, 2),
                         "frac_back_to_back": round(nbytes / (kb_ms * 1e-3) / 1e9 / hbm_peak, 4)},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "us_per_layer_step": round(e2e_ms * 1e3, 2), "api": "torch.ops.libdvatt.dvattn_paged_sdpa", "issue": e2e_mode,
                    "copies": "per step one packed H2D of its inputs (issued in groups of 1, 2, 4, 8 steps, "
                              "one group ahead of the compute) and one D2H of its output right after its op, on "
                              "copy streams"},
            "gpu_launches": launches_per_step * args.steps * len(per_rep),
            "gpu_launches_per_step": launches_per_step,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if "prefill_config4" in extra:
            line["prefill_config4"] = extra.pop("prefill_config4")
        if extra:
            line["strong_scaling"] = extra
        print(json.dumps(line), flush=True)


def prefill_leg(dev, steps, warmup, world):
    """Config 4 (bf16 varlen chunked prefill on the tcgen05 prefill_kernel) as an extra key of
    the default line: whole calls over the C ABI back to back with three rotating KV pools
    (inputs resident), and the attention kernel alone between events; TFLOP/s of the
    attended q.k and p.v products, max over ranks, each rank its own batch."""
    from dvattn_b200 import capi
    from dvattn_b200 import workloads as wl
    _, tf_peak, peak_kind = load_peaks()
    case = wl.config4(device=dev)
    flops = wl.varlen_flops(case)
    out = case.new_out()
    pools = [(case.k_cache, case.v_cache)]
    for _ in range(2):
        pools.append((torch.randn_like(case.k_cache, dtype=torch.float32).to(case.dtype),
                      torch.randn_like(case.v_cache, dtype=torch.float32).to(case.dtype)))
    calls, ws = [], None
    for kc, vc in pools:
        a = list(case.capi_args(out))
        a[7], a[8] = kc, vc
        call = capi.VarlenCall(*a, workspace=ws)
        ws = call.workspace
        calls.append(call)
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        calls[i % 3]()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        calls[i % 3]()
    e1.record(stream)
    torch.cuda.synchronize()
    t_ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        c = calls[i % 3]
        c.phase(capi.DVATTN_PHASE_SCHEDULE)
        kev[i][0].record(stream)
        c.phase(capi.DVATTN_PHASE_ATTEND)
        kev[i][1].record(stream)
        c.phase(capi.DVATTN_PHASE_MERGE)
    torch.cuda.synchronize()
    k_ms = max_over_ranks(statistics.mean(x.elapsed_time(y) for x, y in kev), world)
    achieved = flops / (k_ms * 1e-3) / 1e12
    del pools, calls
    return {"workload": "config4: bf16 varlen chunked prefill, 16 seqs, 32/2 heads, E=128, R=32, page 16",
            "value": round(sum_over_ranks(float(flops), world) / (t_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "us_per_step": round(t_ms * 1e3, 1), "kernel": "prefill_kernel", "kernel_us": round(k_ms * 1e3, 1),
            "achieved": round(achieved, 1), "peak": tf_peak, "peak_kind": peak_kind,
            "frac": round(achieved / tf_peak, 4), "steps": steps, "scaling": "weak"}


def run_varlen(args, world, rank, local):
    """Config 4 (bf16 varlen chunked prefill): tensor-bound; metric TFLOP/s of the attended
    q.k and p.v products (4 * E flops per visible (query head, key) pair).  Weak scaling:
    every rank runs its own batch of 16 sequences.  Same legs as run_ours: value over the
    C ABI with resident inputs (three rotating KV pools), the attention kernel alone between
    events (phase ATTEND), e2e through torch.ops.libdvatt.dvattn_varlen_paged_sdpa with the
    step's inputs copied from pinned host memory and the output copied back."""
    import dvattn_b200  # registers torch.ops.libdvatt
    from dvattn_b200 import capi
    from dvattn_b200 import workloads as wl
    from oracle import dvattn_oracle as O  # CPU baseline leg only
    dev = f"cuda:{local}"
    _, tf_peak, peak_kind = load_peaks()
    case = wl.config4(device=dev)
    flops = wl.varlen_flops(case)
    out = case.new_out()
    pools = [(case.k_cache, case.v_cache)]
    for _ in range(2):
        pools.append((torch.randn_like(case.k_cache, dtype=torch.float32).to(case.dtype),
                      torch.randn_like(case.v_cache, dtype=torch.float32).to(case.dtype)))
    calls, ws = [], None
    for kc, vc in pools:
        a = list(case.capi_args(out))
        a[7], a[8] = kc, vc
        call = capi.VarlenCall(*a, workspace=ws)
        ws = call.workspace
        calls.append(call)
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        calls[i % 3]()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.begin()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        calls[i % 3]()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    t_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        c = calls[i % 3]
        c.phase(capi.DVATTN_PHASE_SCHEDULE)
        kev[i][0].record(stream)
        c.phase(capi.DVATTN_PHASE_ATTEND)
        kev[i][1].record(stream)
        c.phase(capi.DVATTN_PHASE_MERGE)
    torch.cuda.synchronize()
    if sampler:
        sampler.end()
    clocks = sampler.stop() if sampler else None
    k_ms = max_over_ranks(statistics.mean(x.elapsed_time(y) for x, y in kev), world)

    host_in = [t.cpu().pin_memory() for t in (case.queries, case.cosines, case.sines, case.locations,
                                              case.fragment_lengths, case.block_tables, case.cu_seqlens_q)]

    def e2e_launch(d, o, i):
        q, cs, sn, loc, L, bt, cu = d
        kc, vc = pools[i % 3]
        torch.ops.libdvatt.dvattn_varlen_paged_sdpa(o, case.scale, loc, q, cs, sn, L, kc, vc, bt, cu, cu)

    e2e_ms, h2d, d2h, e2e_mode = pipelined_e2e(host_in, out, e2e_launch, args.steps, args.warmup, world)

    total = sum_over_ranks(float(flops), world)
    value = total / (t_ms * 1e-3) / 1e12
    e2e_val = total / (e2e_ms * 1e-3) / 1e12
    achieved = flops / (k_ms * 1e-3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        tl, ql = wl.config4_lengths(4, 16)
        cs = wl.make_varlen(tl[:1], ql[:1], Hq=32, Hkv=2, E=128, R=32, BS=16, dtype=torch.bfloat16, seed=4)
        a = (cs.scale, cs.locations, cs.queries, cs.cosines, cs.sines, cs.fragment_lengths, cs.k_cache, cs.v_cache,
             cs.block_tables, cs.cu_seqlens_q)
        O.varlen_paged_sdpa_f32(*a)
        t0 = time.perf_counter()
        O.varlen_paged_sdpa_f32(*a)
        dt = time.perf_counter() - t0
        cpu = {"value": round(wl.varlen_flops(cs) / dt / 1e12, 5), "unit": "TFLOP/s", "cores": threads,
               "kind": "port", "sample": "first sequence of config 4"}
    if rank == 0:
        ks = "prefill_kernel" if case.queries.size(0) * case.k_cache.size(2) >= 148 * 16 else "decode_row_kernel"
        print(json.dumps({
            "metric": "varlen prefill attention TFLOP/s", "value": round(value, 3), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bfloat16",
            "data": "synthetic (seeded N(0,1) q/k/v, seeded lengths and page permutation)",
            "config": {"workload": "config4: bf16 varlen chunked prefill, 16 seqs, q ~ U[1,2048] after U[0,16384] "
                                   "cached keys, 32/2 heads, E=128, R=32, page 16",
                       "flops_per_step_per_gpu": flops, "parallelism": f"batch-replica x{world}",
                       "l2": "3 rotating KV pools of %.0f MB each" %
                             ((case.k_cache.numel() + case.v_cache.numel()) * case.k_cache.element_size() / 1e6)},
            "roofline": {"bound": "tensor", "kernel": ks, "achieved": round(achieved, 3), "peak": tf_peak,
                         "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": round(achieved / tf_peak, 4),
                         "kernel_us": round(k_ms * 1e3, 2), "traffic": traffic_from_profiles("config4")},
            "e2e": {"value": round(e2e_val, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_step": round(e2e_ms * 1e3, 2),
                    "api": "torch.ops.libdvatt.dvattn_varlen_paged_sdpa", "issue": e2e_mode},
            "gpu_launches": 2 * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu}), flush=True)


def run_sdpa(args, world, rank, local):
    """Config 2's shape on the contiguous-fragment op dvattn_sdpa (row f-1): one K and one V
    fragment per turn [W, Hkv, L_f, E], each worker attending its own keys.  Same legs as
    run_ours: value over the C ABI with three rotating fragment sets, e2e through
    torch.ops.libdvatt.dvattn_sdpa with the per-turn queries and locations copied from
    pinned host memory and the output copied back."""
    import dvattn_b200  # registers torch.ops.libdvatt
    from dvattn_b200 import capi
    from dvattn_b200 import workloads as wl
    from oracle import dvattn_oracle as O  # CPU baseline leg only
    dev = f"cuda:{local}"
    hbm_peak, _, peak_kind = load_peaks()
    case = wl.config2_sdpa(device=dev)
    nbytes = wl.sdpa_bytes(case)
    sets = [(case.keys, case.values)]
    for _ in range(2):
        sets.append(([torch.randn_like(k, dtype=torch.float32).to(k.dtype) for k in case.keys],
                     [torch.randn_like(v, dtype=torch.float32).to(v.dtype) for v in case.values]))
    W, Hq, S, E = case.queries.shape
    out = torch.empty((W, Hq, S, E), dtype=case.dtype, device=dev)

    calls = [capi.SdpaCall(out, case.scale, case.locations, case.rotated, case.fragment_lengths, ks, vs)
             for ks, vs in sets]

    def step(i):
        calls[i % 3]()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.begin()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    if sampler:
        sampler.end()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    t_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps

    host_in = [t.cpu().pin_memory() for t in (case.rotated, case.locations)]

    def e2e_launch(d, o, i):
        rq, loc = d
        ks, vs = sets[i % 3]
        torch.ops.libdvatt.dvattn_sdpa(o, case.scale, loc, rq, case.fragment_lengths, ks, vs)

    e2e_ms, h2d, d2h, e2e_mode = pipelined_e2e(host_in, out, e2e_launch, args.steps, args.warmup, world)
    total = sum_over_ranks(float(nbytes), world)
    value = total / (t_ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        n = 2
        keys = [k[:n].cpu() for k in case.keys]
        vals = [v[:n].cpu() for v in case.values]
        rq, loc = case.rotated[:, :n].cpu(), case.locations[:, :n].cpu()
        O.sdpa_pt(rq, loc, keys, vals, case.scale)
        t0 = time.perf_counter()
        O.sdpa_pt(rq, loc, keys, vals, case.scale)
        dt = time.perf_counter() - t0
        sub = wl.SdpaCase(case.queries[:n], rq, case.cosines[:, :n], case.sines[:, :n], loc, case.fragment_lengths.cpu(),
                          keys, vals, case.scale, {})
        cpu = {"value": round(wl.sdpa_bytes(sub) / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": "first 2 of the 32 workers (reference dvattn_sdpa_pt restated, padded fragments)"}
    if rank == 0:
        print(json.dumps({
            "metric": "contiguous-fragment attention (dvattn_sdpa) HBM GB/s", "value": round(value, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bfloat16", "data": "synthetic (seeded N(0,1) q/k/v, config-2 lengths)",
            "config": {"workload": "sdpa2: config 2 on dvattn_sdpa, 2 turns of fragments [32, 4, L_f, 128] bf16, "
                                   "64 query heads", "bytes_per_step_per_gpu": nbytes,
                       "parallelism": f"batch-replica x{world}", "l2": "3 rotating fragment sets (~2 GB each)"},
            "roofline": {"bound": "hbm", "kernel": "decode_row_kernel (5-D TMA fragment boxes) + merge",
                         "achieved": round(nbytes / (t_ms * 1e-3) / 1e9, 2), "peak": hbm_peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(nbytes / (t_ms * 1e-3) / 1e9 / hbm_peak, 4),
                         "timing": "whole call (schedule + attention + merge), back to back",
                         "traffic": traffic_from_profiles("sdpa2")},
            "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_step": round(e2e_ms * 1e3, 2),
                    "api": "torch.ops.libdvatt.dvattn_sdpa", "issue": e2e_mode},
            "gpu_launches": 3 * args.steps, "clocks": clocks, "cpu_baseline": cpu}), flush=True)


def run_append(args, world, rank, local):
    """Paged KV append with fused K rotation (row f-3) on config 4's prefill shape: 16
    workers, n = 2048 padded new tokens, counts ~ U[1, 2048] (left padding), 2 KV heads,
    E = 128, R = 32, page 16, bf16.  Metric: algorithmic HBM GB/s = new K/V rows read +
    written + their cos/sin rows read."""
    import dvattn_b200  # registers torch.ops.libdvatt
    from dvattn_b200 import workloads as wl
    dev = f"cuda:{local}"
    hbm_peak, _, peak_kind = load_peaks()
    rs = np.random.RandomState(4)
    W, Hkv, n, E, R, BS = 16, 2, 2048, 128, 32, 16
    counts = rs.randint(1, n + 1, size=W).astype(np.int32)
    start = rs.randint(0, 16385, size=W).astype(np.int32)
    maxb = (16384 + n + BS - 1) // BS
    NB = W * maxb
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    kc = torch.zeros((NB, BS, Hkv, E), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    bt = torch.from_numpy(rs.permutation(NB).reshape(W, maxb).astype(np.int32)).to(dev)
    sets = []
    for _ in range(3):
        sets.append((torch.randn((W, Hkv, n, E), generator=g, device=dev).to(torch.bfloat16),
                     torch.randn((W, Hkv, n, E), generator=g, device=dev).to(torch.bfloat16)))
    cos, sin = wl.rope_angles(torch.from_numpy(rs.randint(0, 18000, (W, n))).to(dev), R)
    pos, cnt = torch.from_numpy(start).to(dev), torch.from_numpy(counts).to(dev)
    new = int(counts.sum())
    nbytes = new * Hkv * 2 * E * 2 * 2 + new * R * 4 * 2 + W * 8

    def step(i):
        k, v = sets[i % 3]
        torch.ops.libdvatt.dvattn_paged_append(kc, vc, k, v, cos, sin, bt, pos, cnt)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # a ~10 us kernel is shorter than one op dispatch from Python: the K timed launches are
    # replayed from a CUDA graph so the device time is not host-bound
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            step(i)
    graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.begin()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.end()
    clocks = sampler.stop() if sampler else None
    t_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    host = [t.cpu().pin_memory() for t in sets[0]]
    dk, dvv = torch.empty_like(sets[0][0]), torch.empty_like(sets[0][1])
    e0.record()
    for i in range(args.steps):
        dk.copy_(host[0], non_blocking=True)
        dvv.copy_(host[1], non_blocking=True)
        torch.ops.libdvatt.dvattn_paged_append(kc, vc, dk, dvv, cos, sin, bt, pos, cnt)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    total = sum_over_ranks(float(nbytes), world)
    if rank == 0:
        print(json.dumps({
            "metric": "paged KV append with K rotation HBM GB/s", "value": round(total / (t_ms * 1e-3) / 1e9, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bfloat16", "data": "synthetic (seeded)",
            "config": {"workload": "append4: 16 workers x U[1,2048] new tokens (padded to 2048), 2/128 KV heads, "
                                   "R=32, page 16", "bytes_per_step_per_gpu": nbytes,
                       "parallelism": f"batch-replica x{world}", "l2": "3 rotating new-token sets (34 MB each); each step writes its rows of a 302 MB cache"},
            "roofline": {"bound": "hbm", "kernel": "paged_append_kernel",
                         "achieved": round(nbytes / (t_ms * 1e-3) / 1e9, 2), "peak": hbm_peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(nbytes / (t_ms * 1e-3) / 1e9 / hbm_peak, 4),
                         "traffic": traffic_from_profiles("append4")},
            "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host), "d2h_bytes_per_step": 0,
                    "us_per_step": round(e2e_ms * 1e3, 2), "api": "torch.ops.libdvatt.dvattn_paged_append"},
            "gpu_launches": args.steps, "clocks": clocks, "cpu_baseline": None}), flush=True)


def run_views(args, world, rank, local):
    """Turn/view metadata builder (row f-2) on config 4's prefill shape: F = 4 cache
    segments shared by 16 workers in per-worker orders, n = 2048 new tokens per worker,
    rotary dim 32, theta 1e6, bf16 rounding.  Metric: HBM GB/s of the written locations
    and cos/sin rows (the inputs are a few hundred bytes)."""
    import dvattn_b200  # registers torch.ops.libdvatt
    from oracle import dvattn_oracle as O  # CPU baseline leg only
    dev = f"cuda:{local}"
    hbm_peak, _, peak_kind = load_peaks()
    rs = np.random.RandomState(5)
    F, W, n, R, base = 4, 16, 2048, 32, 1000000.0
    lens = torch.from_numpy(rs.randint(n, 16384, size=F).astype(np.int32)).to(dev)
    order = torch.from_numpy(np.stack([rs.permutation(F) for _ in range(W)]).astype(np.int32)).to(dev)
    loc = torch.empty((F, W, n), dtype=torch.int32, device=dev)
    cos = torch.empty((F, W, n, R), dtype=torch.float32, device=dev)
    sin = torch.empty_like(cos)
    inv = (1.0 / (base ** (torch.arange(0, R, 2, dtype=torch.int64).float() / R))).to(dev)
    nbytes = F * W * n * (4 + 2 * R * 4)

    def step():
        torch.ops.libdvatt.dvattn_build_views(loc, cos, sin, lens, order, inv, base, 1.0, 2)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(args.steps):
            step()
    graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.begin()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.end()
    clocks = sampler.stop() if sampler else None
    t_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    # end to end: segment lengths and orders from pinned host memory, the tables back
    h_in = [lens.cpu().pin_memory(), order.cpu().pin_memory()]
    d_in = [torch.empty_like(lens), torch.empty_like(order)]
    h_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (loc, cos, sin)]
    e0.record()
    for _ in range(args.steps):
        for h, d in zip(h_in, d_in):
            d.copy_(h, non_blocking=True)
        torch.ops.libdvatt.dvattn_build_views(loc, cos, sin, d_in[0], d_in[1], inv, base, 1.0, 2)
        for h, d in zip(h_out, (loc, cos, sin)):
            h.copy_(d, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    total = sum_over_ranks(float(nbytes), world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        lh, oh = lens.cpu().numpy(), order.cpu().numpy()
        O.build_views(lh, oh, n, R, base, 1.0, torch.bfloat16)
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            O.build_views(lh, oh, n, R, base, 1.0, torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        cpu = {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": "the whole workload (oracle restatement of DVAttnCache.update + the rotary module, torch on CPU)"}
    if rank == 0:
        print(json.dumps({
            "metric": "turn/view metadata build HBM GB/s", "value": round(total / (t_ms * 1e-3) / 1e9, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "float32 (bf16-rounded cos/sin)", "data": "synthetic (seeded)",
            "config": {"workload": "views4: 4 segments x 16 workers x 2048 new tokens, rotary dim 32, theta 1e6",
                       "bytes_per_step_per_gpu": nbytes, "parallelism": f"batch-replica x{world}",
                       "l2": "34 MB written per step (outputs rewritten each step)"},
            "roofline": {"bound": "hbm", "kernel": "build_views_vec_kernel",
                         "achieved": round(nbytes / (t_ms * 1e-3) / 1e9, 2), "peak": hbm_peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(nbytes / (t_ms * 1e-3) / 1e9 / hbm_peak, 4),
                         "traffic": traffic_from_profiles("views4")},
            "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in h_in),
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in h_out),
                    "us_per_step": round(e2e_ms * 1e3, 2), "api": "torch.ops.libdvatt.dvattn_build_views"},
            "gpu_launches": args.steps, "clocks": clocks, "cpu_baseline": cpu}), flush=True)


L2_BYTES = 126 * 1024 * 1024


def pool_copies(pool_bytes: int) -> int:
    """KV pool copies to rotate over so that consecutive steps never find their K/V in L2."""
    return max(1, min(8, -(-3 * L2_BYTES // max(pool_bytes, 1))))


def graph_step_ms(fns, steps: int, world: int, min_reps: int = 25, min_s: float = 0.5):
    """`steps` calls fns[i % len(fns)]() captured once in a CUDA graph (no host issue cost in
    the timed region) and replayed: per-rep ms per step (max over ranks), >= min_reps reps."""
    for i in range(3):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            fns[i % len(fns)]()
    g.replay()
    torch.cuda.synchronize()
    per_rep = timed_reps(lambda k: g.replay(), 1, world, torch.cuda.current_stream(), min_reps, min_s)
    del g
    return [x / steps for x in per_rep]


def kv_pools(case, n_pools: int):
    """The case's KV pool and n_pools - 1 random copies of it."""
    pools = [(case.k_cache, case.v_cache)]
    for _ in range(n_pools - 1):
        pools.append((torch.randn_like(case.k_cache, dtype=torch.float32).to(case.dtype),
                      torch.randn_like(case.v_cache, dtype=torch.float32).to(case.dtype)))
    return pools


def paged_calls(case, n_pools: int, out=None, workspace=None, **kw):
    """PagedCall objects over `n_pools` copies of the case's KV pool (one shared workspace)."""
    from dvattn_b200 import capi
    out = case.new_out() if out is None else out
    calls, ws = [], workspace
    for kc, vc in kv_pools(case, n_pools):
        c = capi.PagedCall(out, case.scale, case.locations, case.queries, case.cosines, case.sines,
                           case.fragment_lengths, kc, vc, case.block_tables, workspace=ws, **kw)
        ws = c.workspace
        calls.append(c)
    return calls, out


def batch_strong_scaling(case, world: int, rank: int, steps: int) -> dict:
    """The same batch split over the ranks (dist.balance: LPT on attended keys), each rank
    holding only its sequences' pages; efficiency against the whole batch on one GPU (every
    rank times the whole batch alone first).  No collective on the data path."""
    from dvattn_b200 import dist as ddist
    wl = _wl()
    pool_b = (case.k_cache.numel() + case.v_cache.numel()) * case.k_cache.element_size()
    calls, _ = paged_calls(case, pool_copies(pool_b))
    t1 = statistics.median(graph_step_ms(calls, steps, world))
    del calls
    weights = [int(x) for x in np.asarray(case.turn_lens).sum(axis=1)]
    bins = ddist.balance(weights, world)
    sub = ddist.shard_batch(case, bins[rank])
    sb = (sub.k_cache.numel() + sub.v_cache.numel()) * sub.k_cache.element_size()
    calls, _ = paged_calls(sub, pool_copies(sb))
    per = graph_step_ms(calls, steps, world)
    tn = statistics.median(per)
    loads = [sum(weights[i] for i in b) for b in bins]
    return {"us_per_step": round(tn * 1e3, 2), "us_per_step_1gpu": round(t1 * 1e3, 2),
            "gbs": round(wl.paged_bytes(case) / (tn * 1e-3) / 1e9, 1),
            "efficiency_vs_1gpu": round(t1 / (world * tn), 4),
            "sequences_per_rank": [len(b) for b in bins],
            "max_over_mean_keys": round(max(loads) / (sum(loads) / len(loads)), 4),
            "timing": "CUDA-graph replay of K steps, median of reps, max over ranks; KV pools rotated past L2"}


def long3_scaling(world: int, rank: int, dev: str, steps: int) -> dict:
    """Config 3 (one 4 x 131072-key fp16 context) split by page-aligned KV chunks over the
    ranks, each rank keeping only its chunk's pages.  A step = the attention on the chunk
    (f32 partial O + LSE packed in one buffer), one NCCL all-gather of the packed partials
    and the LSE merge, captured in a CUDA graph.  Efficiency is against the whole context on
    one GPU (every rank times it alone first)."""
    from dvattn_b200 import capi, dist as ddist
    wl = _wl()
    full = wl.config3(device=dev)
    nbytes = wl.paged_bytes(full)
    calls, _ = paged_calls(full, 1)
    t1 = statistics.median(graph_step_ms(calls, steps, world))
    del calls
    if world == 1:
        del full
        torch.cuda.empty_cache()
        return {"us_per_step": round(t1 * 1e3, 2), "gbs": round(nbytes / (t1 * 1e-3) / 1e9, 1),
                "parallelism": "kv-chunk x1 (no exchange)"}
    sh = ddist.kv_chunk_shard(full, rank, world, local_pages=True)
    del full
    torch.cuda.empty_cache()
    out = sh.new_out()
    merged = torch.empty_like(out)
    pb = (sh.k_cache.numel() + sh.v_cache.numel()) * sh.k_cache.element_size()
    n_pools = pool_copies(pb)
    steps_g = steps + (steps & 1)  # the peer exchange alternates two slots: an even count per replay
    Ev = out.size(-1)
    rows = out.numel() // Ev
    import torch.distributed as tdist

    # (a) peer-memory exchange: attention writes its partial into this rank's exchange
    # region; one kernel signals, waits for every rank and merges from the peers' memory
    ex = ddist.PeerExchange(out)
    pools = kv_pools(sh, n_pools)
    pcalls, ws = [], None
    for i in range(2 * n_pools):
        o32, lse = ex.outputs(i % 2)
        kc, vc = pools[i % n_pools]
        c = capi.PagedCall(out, sh.scale, sh.locations, sh.queries, sh.cosines, sh.sines, sh.fragment_lengths,
                           kc, vc, sh.block_tables, lse=lse, out_f32=o32, workspace=ws)
        ws = c.workspace
        pcalls.append(c)

    def peer_step(i):
        def f():
            pcalls[i]()
            ex.merge(i % 2, merged)
        return f

    def peer_merge(i):
        return lambda: ex.merge(i % 2, merged)

    # (b) NCCL: one all-gather of the packed partials + the packed merge
    packed, o32n, lsen = ddist.packed_partials(out)
    gathered = ddist.gather_buffer(packed)
    ncalls = [capi.PagedCall(out, sh.scale, sh.locations, sh.queries, sh.cosines, sh.sines, sh.fragment_lengths,
                             kc, vc, sh.block_tables, lse=lsen, out_f32=o32n, workspace=ws) for kc, vc in pools]

    def nccl_step(c):
        def f():
            c()
            ddist.allgather_merge_packed(packed, merged, gathered=gathered)
        return f

    def exchange():
        tdist.all_gather_into_tensor(gathered, packed)

    def nccl_merge():
        capi.lse_merge_packed(gathered.view(world, rows * (Ev + 1)), merged)

    med = lambda fns: statistics.median(graph_step_ms(fns, steps_g, world))  # noqa: E731
    tn = med([peer_step(i) for i in range(2 * n_pools)])
    t_att = med([(lambda c=c: c()) for c in pcalls])
    t_pm = med([peer_merge(i) for i in range(2)])
    assert ex.status() == 0, "peer exchange: a wait ran out"
    mode = "cuda-graph"
    try:
        tn_nccl = med([nccl_step(c) for c in ncalls])
        t_ex = med([exchange])
        t_mg = med([nccl_merge])
    except Exception as e:  # a collective that cannot be captured: time eagerly
        mode = "eager (%s)" % str(e).splitlines()[0][:80]
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        fs = [nccl_step(c) for c in ncalls]
        tn_nccl = statistics.median(timed_reps(lambda k: fs[k % len(fs)](), steps, world, st)) / steps
        t_ex = statistics.median(timed_reps(lambda k: exchange(), steps, world, st)) / steps
        t_mg = statistics.median(timed_reps(lambda k: nccl_merge(), steps, world, st)) / steps
    ex.close()
    return {"us_per_step": round(tn * 1e3, 2), "us_per_step_1gpu": round(t1 * 1e3, 2),
            "gbs": round(nbytes / (tn * 1e-3) / 1e9, 1), "efficiency_vs_1gpu": round(t1 / (world * tn), 4),
            "attention_us": round(t_att * 1e3, 2), "peer_merge_us": round(t_pm * 1e3, 2),
            "exchange": "peer memory: dvattn_lse_merge_peers (signal, bounded wait, merge reading the peers' "
                        "partials over NVLink), one kernel after the attention",
            "nccl": {"us_per_step": round(tn_nccl * 1e3, 2), "efficiency_vs_1gpu": round(t1 / (world * tn_nccl), 4),
                     "all_gather_us": round(t_ex * 1e3, 2), "merge_us": round(t_mg * 1e3, 2), "issue": mode},
            "exchange_bytes_per_rank": rows * (Ev + 1) * 4,
            "parallelism": f"kv-chunk x{world}, local pages only",
            "timing": "per step: attention + exchange + merge, CUDA-graph replay of K steps, median of reps, "
                      "max over ranks; the parts timed alone the same way"}


def run_long3(args, world, rank, local):
    """Config 3 with its KV split across the ranks (page-aligned chunks, local pages) and
    the partial outputs merged over NCCL (one all-gather of the packed f32 O + LSE, then the
    LSE-merge kernel), one JSON line."""
    dev = f"cuda:{local}"
    wl = _wl()
    r = long3_scaling(world, rank, dev, args.steps)
    if rank == 0:
        t_ms = r["us_per_step"] / 1e3
        print(json.dumps({"metric": METRIC, "value": r["gbs"], "unit": "GB/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms, 5),
                          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "float16",
                          "data": "synthetic", "config": {"workload": "config3 KV-chunk sharded + one NCCL all-gather "
                                                                      "+ LSE merge",
                                                          "parallelism": f"kv-chunk x{world}"},
                          "long3": r, "gpu_launches": args.steps * (3 + (1 if world > 1 else 0))}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config2",
                    choices=["config1", "config2", "config3", "config4", "config5", "long3", "sdpa2", "append4",
                             "views4"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-ref-cuda", action="store_true", help="reference arm: skip timing the reference CUDA op")
    ap.add_argument("--no-extra", action="store_true", help="skip the strong-scaling legs of the default workload")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return
    world, rank, local = dist_setup(args.gpus)
    if args.workload == "long3":
        run_long3(args, world, rank, local)
    elif args.workload == "config4":
        run_varlen(args, world, rank, local)
    elif args.workload == "sdpa2":
        run_sdpa(args, world, rank, local)
    elif args.workload == "append4":
        run_append(args, world, rank, local)
    elif args.workload == "views4":
        run_views(args, world, rank, local)
    else:
        run_ours(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
