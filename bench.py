#!/usr/bin/env python
"""Benchmark of the B200 GDN decode path; rank 0 prints one JSON line.

Workload (a "step"): one Gated DeltaNet decode step of a Qwen3-Next-shaped
layer at batch 256 — 16 q/k heads, 32 v-heads, K = V = 128, T = 1 — with the
fp32 state [256, 32, 128, 128] (512 MiB) updated in place in HBM.  With
``--gpus N`` (torchrun, one process per GPU) the 32 v-heads and their 16 q/k
heads are split across the N ranks (tensor parallel, total work fixed) and
every rank ends the step with the full bf16 output.

value   algorithmic HBM bytes of the whole job per second (GB/s): 4,219,008 B
        per batch entry + 256 B per call, times steps, over the device time of
        the timed steps (CUDA events, max over ranks).  Inputs are resident
        in HBM and larger than L2 (several layers' states updated round robin).
e2e     the same metric through the public API (``kernel_cuda_b200``; at N > 1
        ``TPDecode.capture_sequence``) with every step's inputs (q, k, v, a, b)
        copied from pinned host memory and its output read back to pinned host
        memory inside the timed region.  Copies run on their own streams, double
        buffered, so step i's kernel overlaps the upload of step i+1 and the
        read-back of step i-1 (ordered by CUDA events); the steps and their copies
        are recorded as one CUDA graph, so no per-step host work bounds a short
        step (a 25 us step at N = 8).
parity  before timing, one eager step and one replayed CUDA-graph step on the same
        seeded inputs (drawn identically on every rank and split by heads at N > 1)
        are compared with the CPU oracle on sampled batch entries: the gathered
        output on rank 0, each rank's own state shard.  A mismatch makes the run
        exit non-zero.
configs BASELINE's other single-GPU configurations at reduced iterations (N = 1):
        the batch sweep B in {1,8,32,64,128,256}, the 1024-slot pool with 256
        entries, T in {2,4} at B = 64 with intermediates, the bf16-stored state
        and the in-kernel q/k L2-norm; CUPTI medians, algorithmic GB/s, fraction of
        the measured copy peak.
latency_b1_us   the B=1 decode kernel's median device duration from CUPTI
        activity records (torch.profiler), L2 flushed before every launch, next to
        the floor of the method: this repository's own in-place state round trip
        with the decode kernel's grid and cache hints, same flush.
roofline        the decode kernel alone (CUDA events around the graph of steps).
cpu_baseline    the reference's CPU algorithm (oracle restatement of
        kernel_pt_reference, its per-head loop) on a bounded sample, host cores.

At N > 1 the output exchange is fused into the decode kernel (each rank stores its
rows into every rank's buffer over NVLink, then a bounded barrier); ``--tp-collective
nccl`` uses NCCL all-gather + the interleave kernel instead.
``--impl reference`` times that CPU implementation alone as the reference arm.
``--profile-case B`` runs a few launches of one small decode case and exits (for ncu).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(ROOT, "flashinfer-competition-codebase_b200")
for _p in (PKG_ROOT, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from gdn_b200.timing import (  # noqa: E402
    cupti_kernel_durations_us, cupti_kernels_and_spans, cupti_kernels_by_name, l2_flush_buffer)

METRIC = "GDN decode µs (CUPTI) at B=1; state-update HBM GB/s vs peak at B=256"
UNIT = "GB/s"
BATCH, H, HV, DIM = 256, 16, 32, 128
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
B200_L2_BYTES = 126 * 1024 * 1024     # used only where no GPU can be queried
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "gdn_step_kernel_b256.txt")
OUT_TOL = dict(atol=1e-2, rtol=1e-2)      # bf16 output (north star)
STATE_TOL = dict(atol=1e-3, rtol=1e-3)    # fp32 state (north star)
PARITY_ENTRIES = (0, 85, 170, 255)        # sampled batch entries checked against the oracle
# (label, sequence lengths, q/k heads, v-heads) of the prefill configurations
PREFILL_CASES = (("contest qk4v8, 1 x 6 tokens (reference prefill workload 0)", [6], 4, 8),
                 ("qwen3next 16/32, 8 x 512 tokens", [512] * 8, 16, 32),
                 ("qwen3next 16/32, 1 x 4096 tokens", [4096], 16, 32))
# further shapes on which the three prefill implementations are compared (the dispatch rule)
PREFILL_IMPL_CASES = (("qwen3next 16/32, 64 x 64 tokens", [64] * 64, 16, 32),
                      ("qwen3next 16/32, 16 x 256 tokens", [256] * 16, 16, 32),
                      ("qwen3next 16/32, 2 x 2048 tokens", [2048] * 2, 16, 32))

# NVML clock-event reason bits
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


def log(msg: str) -> None:
    sys.stderr.write(msg + "\n")
    sys.stderr.flush()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": FALLBACK_PEAKS["hbm_gbs"], "source": "fallback"}


def ncu_traffic_per_launch():
    """DRAM bytes (read + write) per launch of the B=256 decode kernel, from the
    committed ncu summary (line ``traffic_bytes_per_launch: N``), else None."""
    try:
        with open(PROFILE_SUMMARY) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock, power and clock-event reasons while the timed region runs.

    ``mode="smi"``: an ``nvidia-smi --query-gpu ... -lms`` subprocess (a separate
    process, so sampling cannot contend with this process's launches);
    ``mode="nvml"``: a background thread polling NVML; ``mode="none"``: off.
    Only one rank samples, for all GPUs of the node in use."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active")

    def __init__(self, device_indices, mode: str = "nvml", interval_ms: int = 2):
        self.mode = mode
        self.indices = list(device_indices)
        self.interval_ms = interval_ms
        self.samples = []           # (sm_mhz, reasons_mask, power_w)
        self.max_mhz = None
        self._proc = None
        self._thread = None
        self._stop = threading.Event()
        if mode == "nvml":
            try:
                import pynvml

                pynvml.nvmlInit()
                self._nv = pynvml
                self._h = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in self.indices]
                self._reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) \
                    or getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h[0], pynvml.NVML_CLOCK_SM)
            except Exception as e:
                log(f"[bench] NVML unavailable: {e}")
                self.mode = "none"

    def _run_nvml(self):
        nv = self._nv
        while not self._stop.is_set():
            for h in self._h:
                try:
                    self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                         self._reasons(h), nv.nvmlDeviceGetPowerUsage(h) / 1e3))
                except Exception:
                    pass
            time.sleep(self.interval_ms / 1e3)

    def start(self):
        if self.mode == "nvml":
            self._thread = threading.Thread(target=self._run_nvml, daemon=True)
            self._thread.start()
        elif self.mode == "smi":
            import subprocess

            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                     f"-lms={self.interval_ms}", "-i", ",".join(map(str, self.indices))],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                time.sleep(0.05)
            except OSError as e:
                log(f"[bench] nvidia-smi unavailable: {e}")
                self.mode = "none"

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        if self._proc is not None:
            time.sleep(self.interval_ms / 1e3)
            self._proc.terminate()
            text, _ = self._proc.communicate(timeout=10)
            for line in text.splitlines():
                parts = [x.strip() for x in line.split(",")]
                try:
                    self.samples.append((float(parts[1]), int(parts[4], 16), float(parts[3])))
                    self.max_mhz = float(parts[2])
                except (ValueError, IndexError):
                    pass
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": self.mode}
        busy = [x for x in self.samples if not (x[1] & 0x1)] or self.samples
        mask = 0
        for x in busy:
            mask |= x[1]
        return {
            "sm_mhz": statistics.median(x[0] for x in busy),
            "sm_max_mhz": self.max_mhz,
            "reasons": [n for bit, n in _REASONS.items() if mask & bit and bit != 0x1],
            "power_w_max": round(max(x[2] for x in busy), 1),
            "samples": len(busy),
            "gpus": len(self.indices),
            "source": "nvidia-smi" if self.mode == "smi" else self.mode,
        }


def _node_gpu_indices(world):
    """nvidia-smi / NVML indices of the GPUs this job uses (CUDA_VISIBLE_DEVICES
    order, one per rank)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if all(x.isdigit() for x in ids):
            return [int(x) for x in ids[:world]]
    return list(range(world))


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def l2_size_bytes() -> int:
    if torch.cuda.is_available():
        return int(torch.cuda.get_device_properties(0).L2_cache_size)
    return B200_L2_BYTES


def layer_count(world: int, l2_bytes: int):
    """Layers whose per-GPU states together hold >= 3x the L2, and one layer's bytes."""
    state_bytes = BATCH * (HV // world) * DIM * DIM * 4
    return max(1, math.ceil(3 * l2_bytes / state_bytes)), state_bytes


def workload_config(world, l2_bytes):
    """The workload, identical in both arms' lines."""
    layers, state_bytes = layer_count(world, l2_bytes)
    return {
        "workload": "gdn_decode_qwen3next_b256_t1",
        "global_batch": BATCH, "T": 1, "num_qk_heads": H, "num_v_heads": HV, "head_dim": DIM,
        "state": "fp32 [256,32,128,128] k-last, updated in place",
        "parallelism": f"tp{world}",
        "l2": (f"inputs larger than L2, no flush: {layers} layer state(s) of "
               f"{state_bytes >> 20} MiB per GPU updated round robin "
               f"({(layers * state_bytes) >> 20} MiB >= 3x the {l2_bytes >> 20} MiB L2)"),
    }


# ---------------------------------------------------------------------------
# CPU leg: the reference's algorithm on the host cores
# ---------------------------------------------------------------------------

def cpu_reference_sample(entries: int, seed: int = 0):
    from gdn_b200 import synthetic

    return synthetic.make_inputs(B=entries, seed=seed)


def time_cpu_reference(entries: int, min_seconds: float, max_calls: int = 1000):
    """Times oracle.decode_loop (the reference's per-head loop) on ``entries``
    batch entries until ``min_seconds`` elapse; returns (GB/s, seconds, calls)."""
    from gdn_b200 import synthetic
    from oracle import gdn_ref

    torch.set_num_threads(os.cpu_count() or 1)
    inp = cpu_reference_sample(entries)
    calls, t0 = 0, time.perf_counter()
    while True:
        gdn_ref.decode_loop(*inp.args())
        calls += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or calls >= max_calls:
            break
    gbs = synthetic.bytes_per_call(entries) * calls / el / 1e9
    return gbs, el, calls


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    from gdn_b200 import synthetic
    from oracle import gdn_ref

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    # size each step so the whole run takes about two minutes
    probe = cpu_reference_sample(1)
    t0 = time.perf_counter()
    gdn_ref.decode_loop(*probe.args())
    per_entry = time.perf_counter() - t0
    budget = 120.0 / max(1, args.steps + args.warmup)
    entries = int(max(1, min(BATCH, budget // max(per_entry, 1e-6))))
    inp = cpu_reference_sample(entries)
    for _ in range(args.warmup):
        gdn_ref.decode_loop(*inp.args())
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        gdn_ref.decode_loop(*inp.args())
        times.append(time.perf_counter() - t0)
    total = sum(times)
    gbs = synthetic.bytes_per_call(entries) * len(times) / total / 1e9
    sample = (f"{entries} of {BATCH} batch entries (x 32 v-heads) per step, oracle restatement of "
              f"kernel_pt_reference's per-head loop, torch CPU fp32")
    line = {
        "impl": "reference",
        "metric": METRIC, "value": round(gbs, 6), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / len(times), 3),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(world, l2_size_bytes()),
        "cpu_baseline": {"value": round(gbs, 6), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 6), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

def _probe_lib():
    from gdn_b200 import build

    if not os.path.exists(build.PROBE_LIB_PATH):
        raise RuntimeError(f"{build.PROBE_LIB_PATH} missing: run __graft_entry__.build()")
    lib = ctypes.CDLL(build.PROBE_LIB_PATH)
    lib.gdn_probe_state_roundtrip.restype = ctypes.c_int
    lib.gdn_probe_state_roundtrip.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    return lib


def b1_latency(device, iters=200):
    import gdn_b200
    from gdn_b200 import synthetic

    inp = synthetic.make_inputs(B=1, seed=0, device=device)
    out = torch.empty((1, 1, HV, DIM), dtype=torch.bfloat16, device=device)
    flush_buf = l2_flush_buffer(device)

    def fn():
        gdn_b200.kernel_cuda_b200(*inp.args(), out, inp.state)

    for _ in range(20):
        fn()
    d = cupti_kernel_durations_us(fn, iters, device, flush=flush_buf.bitwise_not_)
    d_warm = cupti_kernel_durations_us(fn, iters, device, flush=None)
    # floor of the method: this repository's own kernel that reads and writes the same
    # 2 MiB state in place with the decode kernel's grid, work split and cache hints
    # but no math, same flush, same CUPTI records
    probe = _probe_lib()
    scratch = inp.state.clone()
    stream = torch.cuda.current_stream(device).cuda_stream

    def floor_fn():
        rc = probe.gdn_probe_state_roundtrip(scratch.data_ptr(), HV, stream)
        if rc != 0:
            raise RuntimeError(f"gdn_probe_state_roundtrip failed ({rc})")

    for _ in range(20):
        floor_fn()
    floor = cupti_kernel_durations_us(floor_fn, iters, device, name="roundtrip_kernel",
                                      flush=flush_buf.bitwise_not_)
    res = {"median_us": None, "source": "cupti (torch.profiler activity records)",
           "l2": "flushed before every launch (256 MiB read and rewritten)", "iters": len(d)}
    if d:
        d.sort()
        res.update(median_us=round(statistics.median(d), 3), p10_us=round(d[len(d) // 10], 3),
                   p90_us=round(d[(9 * len(d)) // 10], 3))
    if d_warm:
        res["median_us_l2_warm"] = round(statistics.median(d_warm), 3)
    if floor:
        res["copy_floor_us"] = round(statistics.median(floor), 3)
        res["copy_floor"] = ("gdn_probe_state_roundtrip: in-place read+write of the same 2 MiB "
                             "state, decode kernel's grid (256 CTAs x 128 threads) and cache "
                             "hints, no math; L2 flushed; CUPTI")
    return res


class _PlainGraph:
    """Single-GPU steps (kernel_cuda_b200 on each argument tuple) recorded as one
    CUDA graph."""

    def __init__(self, device, step_args, out):
        import gdn_b200

        self.graph = torch.cuda.CUDAGraph()
        self.out = out
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.graph(self.graph, stream=stream):
            for a in step_args:
                gdn_b200.kernel_cuda_b200(*a, out, a[3])
        torch.cuda.current_stream(device).wait_stream(stream)

    def replay(self):
        self.graph.replay()
        return self.out


def _compare(got, want, tol):
    got, want = got.float(), want.float()
    err = (got - want).abs()
    bound = tol["atol"] + tol["rtol"] * want.abs()
    return float(err.max()), bool((err <= bound).all())


class _on_gpu_local_cpus:
    """Run the block with this process bound to the CPUs NVML lists as local to GPU
    ``index`` (so that pinned host memory allocated inside lands on the GPU's NUMA
    node), then restore the previous binding.  Yields a short description."""

    def __init__(self, index):
        self.index = index
        self.saved = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, 16)
            cpus = {w * 64 + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
            self.saved = os.sched_getaffinity(0)
            local = cpus & self.saved
            if not local:
                self.saved = None
                return "no GPU-local CPU available to this process"
            os.sched_setaffinity(0, local)
            return f"allocated from the {len(local)} CPUs local to the GPU"
        except Exception as e:                          # noqa: BLE001
            self.saved = None
            return f"GPU-local CPUs unknown ({type(e).__name__})"

    def __exit__(self, *exc):
        if self.saved is not None:
            os.sched_setaffinity(0, self.saved)
        return False


def _copy_bandwidth(device, host_src, host_dst, reps=10):
    """Standalone pinned-host <-> device copy bandwidth (GB/s, CUDA events) of the e2e
    leg's own buffers: the ceiling that host copies put on the end-to-end number."""
    dev_a = torch.empty_like(host_src, device=device)
    dev_b = torch.empty_like(host_dst, device=device)
    res = {}
    for name, dst, src in (("h2d_gbs", dev_a, host_src), ("d2h_gbs", host_dst, dev_b)):
        dst.copy_(src, non_blocking=True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize(device)
        res[name] = round(src.numel() * src.element_size() * reps / (e0.elapsed_time(e1) / 1e3)
                          / 1e9, 1)
    return res


class _E2EHooks:
    """The end-to-end pipeline around each step, recorded into the graph of the steps.

    Step i uses device input buffer j = i % 2: its inputs are copied from pinned host
    memory on a side stream once step i-2's kernel has read that buffer, and the step
    waits for the copy; the step's output rows are consumed on the step's stream
    (copied into dev_out[j] when the step returns another tensor, as the tensor-parallel
    buffer rule asks) and read back into pinned host memory on a second side stream,
    which step i+2 waits for before it writes dev_out[j] again.  ``before(i)`` and
    ``after(i, out)`` are called on the capturing stream around step i; step 0 forks
    the side streams and the last step joins them."""

    def __init__(self, device, steps, host_in, dev_copy, dev_out, host_out, r0=0):
        self.device, self.steps = device, steps
        self.host_in, self.dev_copy, self.dev_out, self.host_out = host_in, dev_copy, dev_out, host_out
        self.r0, self.rows = r0, dev_out[0].shape[0]
        self.s_h2d, self.s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        self.ev_h2d = [torch.cuda.Event() for _ in range(2)]
        self.ev_kern = [torch.cuda.Event() for _ in range(2)]
        self.ev_d2h = [torch.cuda.Event() for _ in range(2)]

    def before(self, i):
        cur = torch.cuda.current_stream(self.device)
        j = i & 1
        if i == 0:
            self.s_h2d.wait_stream(cur)
            self.s_d2h.wait_stream(cur)
        with torch.cuda.stream(self.s_h2d):
            if i >= 2:
                self.s_h2d.wait_event(self.ev_kern[j])
            for name, t in self.host_in.items():
                self.dev_copy[j][name].copy_(t, non_blocking=True)
            self.ev_h2d[j].record(self.s_h2d)
        cur.wait_event(self.ev_h2d[j])
        if i >= 2:
            cur.wait_event(self.ev_d2h[j])

    def after(self, i, out):
        cur = torch.cuda.current_stream(self.device)
        j = i & 1
        if out.data_ptr() != self.dev_out[j].data_ptr():
            self.dev_out[j].copy_(out[self.r0:self.r0 + self.rows])
        self.ev_kern[j].record(cur)
        with torch.cuda.stream(self.s_d2h):
            self.s_d2h.wait_event(self.ev_kern[j])
            self.host_out[j].copy_(self.dev_out[j], non_blocking=True)
            self.ev_d2h[j].record(self.s_d2h)
        if i == self.steps - 1:
            cur.wait_stream(self.s_d2h)
            cur.wait_stream(self.s_h2d)


class _HookedGraph:
    """``steps`` calls of ``run_step(i, j)`` (returning the step's output tensor) with
    the end-to-end hooks around each, recorded as one CUDA graph."""

    def __init__(self, device, steps, run_step, hooks):
        self.graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.graph(self.graph, stream=stream):
            for i in range(steps):
                hooks.before(i)
                hooks.after(i, run_step(i, i & 1))
        torch.cuda.current_stream(device).wait_stream(stream)

    def replay(self):
        self.graph.replay()


def _time_replay(device, world, graph):
    """CUDA-event time (ms) of one replay of ``graph``, after an untimed one."""
    graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1)


def run_b200_arm(args, rank, world, local_rank):
    import gdn_b200
    from gdn_b200 import synthetic
    from gdn_b200.tp import HeadShard, TPDecode
    from oracle import gdn_ref      # the parity checker only; nothing timed calls it

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    gdn_b200.load_library()
    shard = HeadShard(rank, world, H, HV)
    hl, hvl = shard.h_local, shard.hv_local

    # One set of full inputs drawn on the device from one seed, identical on every rank
    # (same generator, same device type), then cut into this rank's head shard.  The
    # sampled entries' inputs go to the host for the oracle before the state changes.
    full = synthetic.make_inputs(B=BATCH, seed=1234, device=device)
    sel = torch.tensor(PARITY_ENTRIES, device=device)
    ref_in = dict(q=full.q[sel].cpu(), k=full.k[sel].cpu(), v=full.v[sel].cpu(),
                  state=full.state[sel].cpu(), A_log=full.A_log.cpu(), a=full.a[sel].cpu(),
                  dt_bias=full.dt_bias.cpu(), b=full.b[sel].cpu())
    q, k, v, state0, A_log, a, dt_bias, b = shard.shard_inputs(
        full.q, full.k, full.v, full.state, full.A_log, full.a, full.dt_bias, full.b)
    scale = full.scale
    del full
    torch.cuda.empty_cache()

    # Each step updates one "layer's" state and the next step the next layer's (round
    # robin), like the GDN layers of a model: with enough layers the per-GPU working set
    # stays >= 3x the L2, so no step finds its state cached by the previous one (at N=8
    # one layer's shard is only 64 MiB).  q/k/v/a/b are shared by the layers.
    l2_bytes = l2_size_bytes()
    layers, state_bytes = layer_count(world, l2_bytes)
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    states = [state0] + [torch.randn(state0.shape, generator=gen, device=device).mul_(0.1)
                         for _ in range(layers - 1)]
    out = torch.empty((BATCH, 1, HV, DIM), dtype=torch.bfloat16, device=device)
    tp = (TPDecode(H=H, HV=HV, max_batch=BATCH, device=device, collective=args.tp_collective)
          if world > 1 else None)

    def layer_args(i, inputs=None):
        qq, kk, vv, aa, bb = inputs if inputs is not None else (q, k, v, a, b)
        return (qq, kk, vv, states[i % layers], A_log, aa, dt_bias, bb, scale)

    def eager_step(i):
        """One step of layer i through the public API."""
        if tp is not None:
            return tp.step(*layer_args(i), out=None if tp.collective == "peer" else out)
        gdn_b200.kernel_cuda_b200(*layer_args(i), out, states[i % layers])
        return out

    # ---- parity: one eager step, then one replayed CUDA-graph step, on layer 0 ----
    par_graph = tp.capture(*layer_args(0)) if tp is not None else \
        _PlainGraph(device, [layer_args(0)], out)
    got_out = [eager_step(0)[sel].cpu()]        # consumed before the next step is enqueued
    got_out.append(par_graph.replay()[sel].cpu())
    got_state = states[0][sel].cpu()
    del par_graph
    want_o1, want_s1 = gdn_ref.decode(ref_in["q"], ref_in["k"], ref_in["v"], ref_in["state"],
                                      ref_in["A_log"], ref_in["a"], ref_in["dt_bias"],
                                      ref_in["b"], scale)
    want_o2, want_s2 = gdn_ref.decode(ref_in["q"], ref_in["k"], ref_in["v"], want_s1,
                                      ref_in["A_log"], ref_in["a"], ref_in["dt_bias"],
                                      ref_in["b"], scale)
    e_o1, ok_o1 = _compare(got_out[0], want_o1, OUT_TOL)
    e_o2, ok_o2 = _compare(got_out[1], want_o2, OUT_TOL)
    e_s, ok_s = _compare(got_state, want_s2[:, shard.hv0:shard.hv1], STATE_TOL)
    par = torch.tensor([max(e_o1, e_o2), e_s, 0.0 if (ok_o1 and ok_o2 and ok_s) else 1.0],
                       dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(par, op=torch.distributed.ReduceOp.MAX)
    parity = {"entries": list(PARITY_ENTRIES), "steps": ["eager", "graph replay"],
              "checked": ("gathered output [entries, 1, 32, 128] on every rank; each rank's "
                          "state shard after both steps"),
              "max_err_out": float(par[0]), "max_err_state": float(par[1]),
              "tol": {"out": OUT_TOL, "state": STATE_TOL}, "ok": bool(par[2] == 0.0),
              "oracle": "oracle.gdn_ref.decode (CPU fp32), same seeded inputs"}

    # The timed region is one CUDA graph of all K steps (layer i % layers at step i),
    # as a model's decode graph holds all its layers: no host work and no graph
    # boundaries inside it (separate replays of short graphs left 40-60 us idle
    # gaps between them at N > 1).
    K = args.steps
    seq = [layer_args(i) for i in range(K)]
    graph = tp.capture_sequence(seq) if tp is not None else _PlainGraph(device, seq, out)
    for i in range(args.warmup):
        eager_step(i)
    graph.replay()                                        # upload + warm the graph, untimed
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    # Set up the sampler (NVML initialisation takes milliseconds) before the ranks
    # line up: anything slow between the barrier and a rank's launch shows up in
    # the other ranks' timings, which wait for it at the first in-graph barrier.
    sampler = ClockSampler(_node_gpu_indices(world), mode=args.clock_sampler
                           if rank == 0 else "none")
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize(device)
    wall0 = time.perf_counter()
    t_start.record()
    graph.replay()
    t_end.record()
    # The timed region is queued before sampling starts, so the sampler runs while
    # the GPU executes it and cannot delay a launch (measured: a sampler active
    # during enqueueing cost 17-170 % at N=8, a ~29 us step).
    sampler.start()
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - wall0
    clocks = sampler.stop()
    if world > 1:
        torch.distributed.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    kernel_ms = elapsed_ms / K          # steps run back to back inside the graph
    elapsed_ms_max = max_over_ranks(elapsed_ms, world, device)
    del graph

    total_bytes = synthetic.bytes_per_call(BATCH)            # whole job, all heads
    local_bytes = synthetic.bytes_per_call(BATCH, H=hl, HV=hvl)
    value = total_bytes * K / (elapsed_ms_max / 1e3) / 1e9

    # ---- end to end through the public API, host buffers in pinned memory ----
    names = ("q", "k", "v", "a", "b")
    local_in = dict(q=q, k=k, v=v, a=a, b=b)
    rows = BATCH // world                       # this rank reads back its batch rows
    r0 = rank * rows
    dev_out = [torch.empty((rows, 1, HV, DIM), dtype=torch.bfloat16, device=device)
               for _ in range(2)]
    # A step's inputs are packed into one pinned host buffer (one H2D copy per step, not
    # one per tensor); the device buffers are views into one allocation per pipeline slot.
    offs, nbytes = {}, 0
    for n in names:
        offs[n] = nbytes
        nbytes += (local_in[n].numel() * local_in[n].element_size() + 255) // 256 * 256

    def views(buf):
        return {n: buf[offs[n]:offs[n] + local_in[n].numel() * local_in[n].element_size()]
                .view(local_in[n].dtype).view(local_in[n].shape) for n in names}

    # pinned host buffers on the GPU's own NUMA node (allocated from its local CPUs)
    with _on_gpu_local_cpus(local_rank) as numa:
        host_pack = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        host_out = [torch.empty(dev_out[0].shape, dtype=torch.bfloat16).pin_memory()
                    for _ in range(2)]
    for n, t in views(host_pack).items():
        t.copy_(local_in[n].cpu())
    dev_pack = [torch.empty(nbytes, dtype=torch.uint8, device=device) for _ in range(2)]
    dev_in = [views(b) for b in dev_pack]
    host_in = {"packed inputs": host_pack}
    dev_copy = [{"packed inputs": b} for b in dev_pack]
    link = _copy_bandwidth(device, host_pack, host_out[0])
    h2d_rank = sum(t.numel() * t.element_size() for t in local_in.values())
    d2h_rank = host_out[0].numel() * host_out[0].element_size()
    K_e2e = max(1, min(K, 500))
    hooks = _E2EHooks(device, K_e2e, host_in, dev_copy, dev_out, host_out, r0=r0)
    if tp is None:
        def run_step(i, j):
            gdn_b200.kernel_cuda_b200(*layer_args(i, [dev_in[j][n] for n in names]),
                                      dev_out[j], states[i % layers])
            return dev_out[j]
        e2e_graph = _HookedGraph(device, K_e2e, run_step, hooks)
        api = ("gdn_b200.kernel_cuda_b200, one call per step; the steps and their copies "
               "recorded as one CUDA graph")
    else:
        e2e_graph = tp.capture_sequence(
            [layer_args(i, [dev_in[i & 1][n] for n in names]) for i in range(K_e2e)],
            before=hooks.before, after=hooks.after)
        api = ("gdn_b200.tp.TPDecode.capture_sequence with the copies recorded around each "
               "step (before/after hooks), each rank reading back its batch rows of the "
               "gathered output")
    e2e_ms = max_over_ranks(_time_replay(device, world, e2e_graph), world, device)
    e2e_value = total_bytes * K_e2e / (e2e_ms / 1e3) / 1e9
    del e2e_graph
    # the same pipeline with no step launched: what the host copies alone take per step
    # (next to the device-only step time, it shows whether the copies overlapped)
    copy_hooks = _E2EHooks(device, K_e2e, host_in, dev_copy, dev_out, host_out, r0=r0)
    copy_graph = _HookedGraph(device, K_e2e, lambda i, j: dev_out[j], copy_hooks)
    copy_ms = max_over_ranks(_time_replay(device, world, copy_graph), world, device)
    del copy_graph

    latency = b1_latency(device) if (world == 1 and not args.skip_b1) else None
    configs = run_configs(device, args.config_iters) if (world == 1 and not args.skip_configs) \
        else None

    cpu = None
    if world == 1 and rank == 0 and not args.skip_cpu:
        gbs, secs, calls = time_cpu_reference(entries=4, min_seconds=args.cpu_seconds)
        cpu = {"value": round(gbs, 6), "unit": UNIT, "cores": torch.get_num_threads(),
               "kind": "port",
               "sample": f"4 batch entries x 32 v-heads, {calls} calls in {secs:.1f} s "
                         "(oracle restatement of kernel_pt_reference's per-head loop, torch CPU fp32)"}

    if world > 1:
        if tp.collective == "peer":
            tp.check()
        torch.distributed.barrier()
        del tp
        torch.distributed.destroy_process_group()
    if rank != 0:
        if not parity["ok"]:
            sys.exit(1)
        return

    peaks = load_peaks()
    achieved = local_bytes / (kernel_ms / 1e3) / 1e9
    traffic = ncu_traffic_per_launch() if world == 1 else None
    # N>1: decode + barrier kernels (peer) or decode + interleave kernels (NCCL)
    launches_per_step = 1 if world == 1 else 2
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(elapsed_ms_max / K, 5),
        # (batch entry, v-head) state updates of the whole job per second
        "state_updates_per_s": round(BATCH * HV * K / (elapsed_ms_max / 1e3)),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE distributions)",
        "config": workload_config(world, l2_bytes),
        "timed_loop": f"one CUDA graph of the {K} steps",
        "parity": parity,
        "latency_b1_us": latency,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic, "peak_source": peaks["source"],
                     "kernel": "gdn_step_kernel", "kernel_us": round(kernel_ms * 1e3, 2),
                     "algorithmic_bytes_per_launch": local_bytes},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": h2d_rank * world, "d2h_bytes_per_step": d2h_rank * world,
                "per_rank": {"h2d": h2d_rank, "d2h": d2h_rank}, "steps": K_e2e, "api": api,
                "overlap": "H2D / D2H on side streams, double-buffered, ordered by CUDA events, "
                           "recorded with the steps as one CUDA graph (one replay is timed); "
                           "one packed H2D copy of q/k/v/a/b per step",
                "pinned": numa, "copy_bandwidth": link,
                "us_per_step": round(e2e_ms * 1e3 / K_e2e, 2),
                "copies_only_us_per_step": round(copy_ms * 1e3 / K_e2e, 2),
                "frac_of_value": round(e2e_value / value, 3)},
        "tp_exchange": None if world == 1 else (
            "fused: decode kernel stores outputs into every rank's buffer over NVLink, "
            "then a one-CTA barrier kernel (roofline.kernel_us covers both); CUDA graphs"
            if args.tp_collective == "peer" else
            "NCCL all_gather_into_tensor + interleave kernel; CUDA graphs"),
        "gpu_launches": launches_per_step * K,
        "clocks": clocks,
        "configs": configs,
        "cpu_baseline": cpu,
        "wall_s_timed": round(wall, 4),
    }
    print(json.dumps(line), flush=True)
    if not parity["ok"]:
        log(f"[bench] PARITY FAILED: {parity}")
        sys.exit(1)


def _short_kernel_name(name: str) -> str:
    """`void (anonymous namespace)::gdn_step_kernel<8, ...>(StepArgs)` -> `gdn_step_kernel`."""
    import re
    m = re.search(r"(gdn_\w+|roundtrip_\w+)", name)
    return m.group(1) if m else name[:60]


def run_configs(device, iters):
    """BASELINE's single-GPU configurations 2-4 (plus the bf16-stored state and the
    in-kernel q/k L2-norm) at reduced iterations: CUPTI median per call, algorithmic
    GB/s and fraction of the measured copy peak.  Small cases (whose state fits in L2)
    flush L2 before every launch; large ones exceed it."""
    import gdn_b200
    from gdn_b200 import synthetic

    peak = load_peaks()["hbm_gbs"]
    flush_buf = l2_flush_buffer(device)
    l2 = l2_size_bytes()

    def measure(fn, nbytes, state_bytes, extra):
        for _ in range(5):
            fn()
        flushed = state_bytes < 2 * l2
        # every kernel of this library a call launches (gdn_step_kernel, the prefill
        # kernels): one kernel's median duration, or for a call of several kernels the
        # median span from the first one's start to the last one's end (the two-launch
        # prefill's second kernel is a programmatic dependent that starts during the
        # first one's tail, so the sum of their durations would count that overlap twice)
        d, spans = cupti_kernels_and_spans(fn, iters, device,
                                           flush=flush_buf.bitwise_not_ if flushed else None)
        per_call = {n: statistics.median(v) for n, v in d.items()
                    if "gdn_" in n and len(v) >= 0.9 * iters}
        if not per_call:              # no CUPTI records (e.g. under another profiler)
            return dict(extra, median_us=None, GBps=None, frac=None, l2=None)
        med = sum(per_call.values())
        if len(per_call) > 1 and spans:
            med = statistics.median(spans)
        gbs = nbytes / med / 1e3
        r = dict(extra, median_us=round(med, 3), GBps=round(gbs, 1),
                 frac=round(gbs / peak, 4), l2="flushed" if flushed else "inputs > 2x L2")
        if len(per_call) > 1:
            r["kernels_us"] = {_short_kernel_name(n): round(t, 3) for n, t in per_call.items()}
            r["median_is"] = "span of a call: first kernel start to last kernel end"
        return r

    res = {"peak_gbs": peak, "iters": iters, "decode_batch_sweep": [], "decode_l2norm": [],
           "bf16_state": [], "mtp": []}
    for B in (1, 8, 32, 64, 128, 256):
        inp = synthetic.make_inputs(B=B, seed=B, device=device)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        fn = lambda: gdn_b200.kernel_cuda_b200(*inp.args(), out, inp.state)  # noqa: E731
        r = measure(fn, synthetic.bytes_per_call(B), inp.state.numel() * 4, {"B": B})
        if r["median_us"]:
            r["state_updates_per_s"] = round(B * HV / (r["median_us"] * 1e-6))
        res["decode_batch_sweep"].append(r)
        del inp, out
    # the same step with the in-kernel q/k L2-norm (FlashInfer's use_qk_l2norm=True;
    # the reference path itself never normalises)
    for B in (1, 64, 256):
        inp = synthetic.make_inputs(B=B, seed=B, device=device)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        fn = lambda: gdn_b200.gated_delta_rule_decode_pretranspose(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
            out, use_qk_l2norm=True)
        res["decode_l2norm"].append(measure(fn, synthetic.bytes_per_call(B),
                                            inp.state.numel() * 4, {"B": B}))
        del inp, out
    # pooled: pool of 1024 slots, 256 active entries drawn as a permutation, one -1
    P, B = 1024, 256
    inp = synthetic.make_inputs(B=B, slots=P, seed=7, device=device)
    idx = synthetic.make_pool_indices(B, P, seed=7, n_pad=1, device=device)
    out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
    fn = lambda: gdn_b200.gated_delta_rule_decode_pretranspose(  # noqa: E731
        inp.q, inp.k, inp.v, None, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale, out,
        use_qk_l2norm=False, initial_state=inp.state, initial_state_indices=idx)
    res["pooled"] = measure(fn, synthetic.bytes_per_call(B, active=B - 1),
                            inp.state.numel() * 4, {"pool": P, "B": B, "active": B - 1})
    del inp, out, idx
    # bf16-stored state (FlashInfer's bf16-state backend): half the state bytes
    for B in (1, 64, 256):
        inp = synthetic.make_inputs(B=B, seed=B, device=device)
        inp.state = inp.state.to(torch.bfloat16)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        fn = lambda: gdn_b200.decode_bf16_state(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale, out)
        res["bf16_state"].append(measure(fn, synthetic.bytes_per_call(B, state_elem_bytes=2),
                                         inp.state.numel() * 2, {"B": B}))
        del inp, out
    # the decode step fused with the layer's gated RMSNorm, against the same step followed
    # by the norm as separate PyTorch kernels (every kernel of a call counted)
    from oracle import gdn_ref  # the unfused norm below is the oracle's PyTorch ops, on GPU

    res["decode_gated_norm"] = []
    for B in (1, 256):
        inp = synthetic.make_inputs(B=B, seed=90 + B, device=device)
        gen = torch.Generator(device=device).manual_seed(B)
        z = torch.randn((B, 1, HV, DIM), generator=gen, device=device).to(torch.bfloat16)
        w = torch.ones(DIM, device=device, dtype=torch.bfloat16)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        fused = lambda: gdn_b200.gdn_decode_gated_norm(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, z, w,
            scale=inp.scale, output=out)

        def unfused():
            o, _ = gdn_b200.gated_delta_rule_decode_pretranspose(
                inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b,
                scale=inp.scale, output=out, use_qk_l2norm=True)
            return gdn_ref.gated_rmsnorm(o, z, w, 1e-6)

        r = measure(fused, synthetic.bytes_per_call(B) + 2 * B * HV * DIM * 2,
                    inp.state.numel() * 4, {"B": B})
        flushed = inp.state.numel() * 4 < 2 * l2
        for _ in range(5):
            unfused()
        d = cupti_kernels_by_name(unfused, iters, device, flush=flush_buf.bitwise_not_ if flushed else None)
        per_call = {n: statistics.median(v) for n, v in d.items() if len(v) >= iters}
        r["unfused_us"] = round(sum(per_call.values()), 3) if per_call else None
        r["unfused_kernels_per_call"] = len(per_call)
        res["decode_gated_norm"].append(r)
        del inp, out, z, w

    # variable-length prefill: the reference's prefill workload 0 shape (one 6-token
    # sequence, 4 q/k and 8 v-heads), a batch of prompts and one long prompt at the
    # Qwen3-Next heads (unit-norm q/k)
    res["prefill"] = []
    res["prefill_impls"] = []
    for label, lengths, H_, HV_ in PREFILL_CASES + PREFILL_IMPL_CASES:
        d = synthetic.make_prefill_inputs(lengths, H=H_, HV=HV_, seed=11, device=device)
        total, N = sum(lengths), len(lengths)
        out = torch.empty((total, HV_, DIM), dtype=torch.bfloat16, device=device)
        ns = torch.empty((N, HV_, DIM, DIM), dtype=torch.float32, device=device)
        fn = lambda: gdn_b200.kernel_prefill_b200(  # noqa: E731
            d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
            d["cu_seqlens"], d["scale"], out, ns)
        if (label, lengths, H_, HV_) in PREFILL_CASES:
            r = measure(fn, synthetic.prefill_bytes(lengths, H_, HV_), 2 * ns.numel() * 4,
                        {"case": label, "num_seqs": N, "tokens": total})
            if r["median_us"]:
                r["tokens_per_s"] = round(total / (r["median_us"] * 1e-6))
                r["ns_per_token_of_longest_sequence"] = round(r["median_us"] * 1e3 / max(lengths), 2)
            res["prefill"].append(r)
        # the three implementations behind gdn_prefill on the same case: the token loop,
        # the one-launch chunked kernel and the two-launch chunked form
        impls = {"token_loop": gdn_b200.prefill_tuned, "chunked_1launch": gdn_b200.prefill_chunked,
                 "chunked_2launch": gdn_b200.prefill_wy}
        row = {"case": label}
        for name, f in impls.items():
            call = lambda f=f: f(  # noqa: E731
                d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                d["cu_seqlens"], d["scale"], out, ns)
            row[name + "_us"] = measure(call, 1, 2 * ns.numel() * 4, {})["median_us"]
        res["prefill_impls"].append(row)
        del d, out, ns
    # multi-token speculative verify, B = 64, one intermediate state per token
    for T in (2, 4):
        B = 64
        inp = synthetic.make_inputs(B=B, T=T, seed=T, device=device)
        out = torch.empty((B, T, HV, DIM), dtype=torch.bfloat16, device=device)
        inter = torch.empty((B, T, HV, DIM, DIM), dtype=torch.float32, device=device)
        fn = lambda: gdn_b200.gated_delta_rule_mtp(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a, inp.dt_bias, inp.b,
            inp.scale, out, inter, disable_state_update=False, use_qk_l2norm=False)
        res["mtp"].append(measure(fn, synthetic.bytes_per_call(B, T=T, intermediates=True),
                                  (T + 1) * inp.state.numel() * 4, {"B": B, "T": T}))
        del inp, out, inter
    return res


COMPARE_GROUPS = ("decode_fp32", "decode_bf16", "mtp_fp32", "prefill")


def run_compare_isolated(iters, path):
    """run_compare with each group in a child process of its own: CUPTI activity records
    collected through torch.profiler went missing in one process after some library
    kernels had been JIT-built and run, so no group's timing depends on another's."""
    import subprocess

    merged = None
    for group in COMPARE_GROUPS:
        part = f"{path}.{group}.json"
        rc = subprocess.run([sys.executable, os.path.abspath(__file__), "--compare", part,
                             "--compare-group", group, "--config-iters", str(iters)]).returncode
        try:
            with open(part) as f:
                d = json.load(f)
        except (OSError, ValueError):
            d = {"rows": [{"config": group, "error": f"child exited {rc}, no results"}]}
        if merged is None:
            merged = d
        else:
            merged["rows"] += d["rows"]
            for key, val in d.items():
                merged.setdefault(key, val)
        os.remove(part) if os.path.exists(part) else None
    with open(path, "w") as f:
        json.dump(merged, f, indent=1)
    return merged


def run_compare(device, iters, path, group=None):
    """Same-GPU head-to-head with the kernels the reference measures against, on one
    GPU with local tensors only: FlashInfer's CuTe-DSL decode (fp32 state, exactly as
    the reference's kernel_fi_baseline calls it, solution/triton/kernel.py:124-147;
    and its bf16-state and multi-token paths) and flash-linear-attention's fused
    recurrent Triton kernel (fla 0.5.1, the package the reference's fla-recurrent kernel
    was taken from, solution/triton/kernel.py:150-203).  CUPTI device time per call
    (every kernel a call launches), L2 flushed before every call where the state fits
    in 2x L2.  Each competitor also runs once from the same inputs as this repository's
    kernel and the largest output / state difference is recorded."""
    import gdn_b200
    from gdn_b200 import synthetic

    res = {"method": "CUPTI (torch.profiler), median per kernel summed over the kernels of "
                     "one call; L2 flushed (256 MiB read and rewritten) when the state < 2x L2",
           "iters": iters, "rows": []}
    try:
        from flashinfer.gdn_decode import gated_delta_rule_decode_pretranspose as fi_decode
        from flashinfer.gdn_decode import gated_delta_rule_mtp as fi_mtp
        res["flashinfer"] = __import__("flashinfer").__version__
    except Exception as e:                              # noqa: BLE001
        fi_decode = fi_mtp = None
        res["flashinfer"] = f"unavailable: {type(e).__name__}: {e}"[:300]
    try:
        from fla.ops.gated_delta_rule import fused_recurrent_gated_delta_rule as fla_rec
        res["fla"] = __import__("fla").__version__
    except Exception as e:                              # noqa: BLE001
        fla_rec = None
        res["fla"] = f"unavailable: {type(e).__name__}: {e}"[:300]
    flush_buf = l2_flush_buffer(device)
    l2 = l2_size_bytes()

    def timed(fn, state_bytes):
        for _ in range(5):
            fn()
        torch.cuda.synchronize(device)
        flushed = state_bytes < 2 * l2
        d, spans = cupti_kernels_and_spans(fn, iters, device,
                                           flush=flush_buf.bitwise_not_ if flushed else None)
        # kernels seen once per call (CUPTI can drop a few records of a long run)
        per_call = {n: statistics.median(v) for n, v in d.items() if len(v) >= 0.9 * iters}
        total = sum(per_call.values())
        # this library's multi-kernel calls overlap their kernels (programmatic launch):
        # their time is the span of a call; other implementations' kernels run one after
        # another, and the sum of their durations leaves out the gaps between launches
        ours = len(per_call) > 1 and all("gdn_" in n for n in per_call)
        if ours and spans:
            total = statistics.median(spans)
        main = max(per_call, key=per_call.get) if per_call else None
        r = {"us": round(total, 3), "kernels": {n[:90]: round(t, 3) for n, t in per_call.items()},
             "main_kernel_us": round(per_call[main], 3) if main else None,
             "l2": "flushed" if flushed else "inputs > 2x L2",
             "cupti_events": {n[:60]: len(v) for n, v in d.items()}}
        if not per_call:
            raise RuntimeError(f"CUPTI recorded no kernel once per call: {r['cupti_events']}")
        return r

    def diff(a, b):
        return round(float((a.float() - b.float()).abs().max()), 6)

    def row(config, impl, fn, state_bytes, nbytes, agree=None):
        try:
            r = timed(fn, state_bytes)
            r.update(config=config, impl=impl, GBps=round(nbytes / r["us"] / 1e3, 1))
            if agree is not None:
                r["max_diff_vs_b200"] = agree
        except Exception as e:                          # noqa: BLE001
            r = {"config": config, "impl": impl, "error": f"{type(e).__name__}: {e}"[:300]}
        res["rows"].append(r)
        log(f"[compare] {config:24s} {impl:28s} {r.get('us', r.get('error'))}")

    for B in ((1, 8, 64, 256) if group in (None, "decode_fp32") else ()):
        base = synthetic.make_inputs(B=B, seed=500 + B, device=device)
        cfg = f"decode fp32 B={B}"
        nbytes = synthetic.bytes_per_call(B)
        sb = base.state.numel() * 4
        ours = base.clone()
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        # reference results for agreement: one step of this repository's kernel
        ref_state = base.state.clone()
        ref_out = torch.empty_like(out)
        gdn_b200.kernel_cuda_b200(base.q, base.k, base.v, ref_state, base.A_log, base.a,
                                  base.dt_bias, base.b, base.scale, ref_out, ref_state)
        row(cfg, "b200 (this repository)",
            lambda: gdn_b200.kernel_cuda_b200(*ours.args(), out, ours.state), sb, nbytes)
        if fi_decode is not None:
            fi = base.clone()
            fo = torch.empty_like(out)
            try:
                fi_decode(fi.q, fi.k, fi.v, fi.state, fi.A_log, fi.a, fi.dt_bias, fi.b,
                          scale=fi.scale, output=fo, use_qk_l2norm=False)
                torch.cuda.synchronize(device)
                agree = {"out": diff(fo, ref_out), "state": diff(fi.state, ref_state)}
            except Exception as e:                      # noqa: BLE001
                agree = {"error": f"{type(e).__name__}: {e}"[:200]}
            row(cfg, "flashinfer fp32 (fi-baseline)",
                lambda: fi_decode(fi.q, fi.k, fi.v, fi.state, fi.A_log, fi.a, fi.dt_bias, fi.b,
                                  scale=fi.scale, output=fo, use_qk_l2norm=False), sb, nbytes, agree)
        if fla_rec is not None:
            fl = base.clone()
            beta = torch.sigmoid(fl.b.float())          # fla takes beta; computed once, untimed
            try:
                fo, fs = fla_rec(fl.q, fl.k, fl.v, g=fl.a, beta=beta, scale=fl.scale,
                                 initial_state=fl.state, output_final_state=True,
                                 use_gate_in_kernel=True, A_log=fl.A_log, dt_bias=fl.dt_bias,
                                 transpose_state_layout=True)
                torch.cuda.synchronize(device)
                agree = {"out": diff(fo, ref_out), "state": diff(fs, ref_state)}
            except Exception as e:                      # noqa: BLE001
                agree = {"error": f"{type(e).__name__}: {e}"[:200]}
            row(cfg, "fla fused_recurrent (Triton)",
                lambda: fla_rec(fl.q, fl.k, fl.v, g=fl.a, beta=beta, scale=fl.scale,
                                initial_state=fl.state, output_final_state=True,
                                use_gate_in_kernel=True, A_log=fl.A_log, dt_bias=fl.dt_bias,
                                transpose_state_layout=True), sb, nbytes, agree)
        del base, ours, out, ref_state, ref_out
        torch.cuda.empty_cache()

    for B in ((1, 64, 256) if group in (None, "decode_bf16") else ()):
        base = synthetic.make_inputs(B=B, seed=600 + B, device=device)
        base.state = base.state.to(torch.bfloat16)
        cfg = f"decode bf16 state B={B}"
        nbytes = synthetic.bytes_per_call(B, state_elem_bytes=2)
        sb = base.state.numel() * 2
        ours = base.clone()
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        ref = base.clone()
        ref_out = gdn_b200.decode_bf16_state(ref.q, ref.k, ref.v, ref.state, ref.A_log, ref.a,
                                             ref.dt_bias, ref.b, ref.scale)
        row(cfg, "b200 (this repository)",
            lambda: gdn_b200.decode_bf16_state(ours.q, ours.k, ours.v, ours.state, ours.A_log,
                                               ours.a, ours.dt_bias, ours.b, ours.scale, out),
            sb, nbytes)
        if fi_decode is not None:
            fi = base.clone()
            fo = torch.empty_like(out)
            try:
                fi_decode(fi.q, fi.k, fi.v, fi.state, fi.A_log, fi.a, fi.dt_bias, fi.b,
                          scale=fi.scale, output=fo, use_qk_l2norm=False)
                torch.cuda.synchronize(device)
                agree = {"out": diff(fo, ref_out), "state": diff(fi.state, ref.state),
                         "state_bit_identical_frac": round(float(
                             (fi.state.view(torch.int16) == ref.state.view(torch.int16))
                             .float().mean()), 6)}
            except Exception as e:                      # noqa: BLE001
                agree = {"error": f"{type(e).__name__}: {e}"[:200]}
            row(cfg, "flashinfer bf16 state",
                lambda: fi_decode(fi.q, fi.k, fi.v, fi.state, fi.A_log, fi.a, fi.dt_bias, fi.b,
                                  scale=fi.scale, output=fo, use_qk_l2norm=False), sb, nbytes, agree)
        del base, ours, out, ref
        torch.cuda.empty_cache()

    for T in ((2, 4) if group in (None, "mtp_fp32") else ()):
        B = 64
        base = synthetic.make_inputs(B=B, T=T, seed=700 + T, device=device)
        cfg = f"mtp fp32 B={B} T={T}"
        nbytes = synthetic.bytes_per_call(B, T=T, intermediates=True)
        sb = (T + 1) * base.state.numel() * 4
        idx = torch.arange(B, dtype=torch.int32, device=device)
        ours = base.clone()
        out = torch.empty((B, T, HV, DIM), dtype=torch.bfloat16, device=device)
        inter = torch.empty((B, T, HV, DIM, DIM), dtype=torch.float32, device=device)
        ref = base.clone()
        ref_out, _ = gdn_b200.gated_delta_rule_mtp(
            ref.q, ref.k, ref.v, ref.state, idx, ref.A_log, ref.a, ref.dt_bias, ref.b, ref.scale,
            None, inter, disable_state_update=False, use_qk_l2norm=False)
        ref_inter = inter.clone()
        row(cfg, "b200 (this repository)",
            lambda: gdn_b200.gated_delta_rule_mtp(
                ours.q, ours.k, ours.v, ours.state, idx, ours.A_log, ours.a, ours.dt_bias, ours.b,
                ours.scale, out, inter, disable_state_update=False, use_qk_l2norm=False),
            sb, nbytes)
        if fi_mtp is not None:
            fi = base.clone()
            fo = torch.empty_like(out)
            finter = torch.empty_like(inter)
            try:
                fi_mtp(fi.q, fi.k, fi.v, fi.state, idx, fi.A_log, fi.a, fi.dt_bias, fi.b,
                       scale=fi.scale, output=fo, intermediate_states_buffer=finter,
                       disable_state_update=False, use_qk_l2norm=False)
                torch.cuda.synchronize(device)
                agree = {"out": diff(fo, ref_out), "state": diff(fi.state, ref.state),
                         "intermediates": diff(finter, ref_inter)}
            except Exception as e:                      # noqa: BLE001
                agree = {"error": f"{type(e).__name__}: {e}"[:200]}
            row(cfg, "flashinfer mtp fp32",
                lambda: fi_mtp(fi.q, fi.k, fi.v, fi.state, idx, fi.A_log, fi.a, fi.dt_bias, fi.b,
                               scale=fi.scale, output=fo, intermediate_states_buffer=finter,
                               disable_state_update=False, use_qk_l2norm=False),
                sb, nbytes, agree)
        del base, ours, out, inter, ref, ref_inter
        torch.cuda.empty_cache()

    # variable-length prefill: this repository's sequential kernel against fla's chunked
    # (WY) Triton prefill, the package the reference's prefill-fla-chunk code came from
    # (solution/triton/fla_prefill_code.py); the same gates, q/k expanded to the v-heads
    # and the state transposed to fla's [K, V] layout outside the timed call.
    try:
        from fla.ops.gated_delta_rule import chunk_gated_delta_rule as fla_chunk
    except Exception:                                   # noqa: BLE001
        fla_chunk = None
    if int((torch.version.cuda or "0").split(".")[0]) < 13:
        res["flashinfer_prefill"] = ("not run: FlashInfer's Blackwell prefill needs a CUDA 13 "
                                     "torch (this image's is " + str(torch.version.cuda) +
                                     "); its other path is an sm_90a kernel")
    import torch.nn.functional as F
    for label, lengths, H_, HV_ in (PREFILL_CASES if group in (None, "prefill") else ()):
        d = synthetic.make_prefill_inputs(lengths, H=H_, HV=HV_, seed=12, device=device)
        total, N = sum(lengths), len(lengths)
        cfg = f"prefill {label}"
        nbytes = synthetic.prefill_bytes(lengths, H_, HV_)
        sb = 2 * N * HV_ * DIM * DIM * 4
        out = torch.empty((total, HV_, DIM), dtype=torch.bfloat16, device=device)
        ns = torch.empty((N, HV_, DIM, DIM), dtype=torch.float32, device=device)
        gdn_b200.kernel_prefill_b200(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                     d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"], out, ns)
        ref_out, ref_ns = out.clone(), ns.clone()
        row(cfg, "b200 (this repository)",
            lambda: gdn_b200.kernel_prefill_b200(
                d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                d["cu_seqlens"], d["scale"], out, ns), sb, nbytes)
        if fla_chunk is not None:
            rep = HV_ // H_
            qe = d["q"].repeat_interleave(rep, dim=1)[None]
            ke = d["k"].repeat_interleave(rep, dim=1)[None]
            ve = d["v"][None]
            g = (-torch.exp(d["A_log"]) * F.softplus(d["a"].float() + d["dt_bias"]))[None]
            beta = torch.sigmoid(d["b"].float())[None]
            h0 = d["state"].transpose(-1, -2).contiguous()
            cu64 = d["cu_seqlens"].long()
            call = lambda: fla_chunk(qe, ke, ve, g, beta, scale=d["scale"],  # noqa: E731
                                     initial_state=h0, output_final_state=True,
                                     cu_seqlens=cu64)
            try:
                fo, fs = call()
                torch.cuda.synchronize(device)
                agree = {"out": diff(fo[0], ref_out),
                         "state": diff(fs.transpose(-1, -2), ref_ns)}
            except Exception as e:                      # noqa: BLE001
                agree = {"error": f"{type(e).__name__}: {e}"[:200]}
            row(cfg, "fla chunk_gated_delta_rule (Triton)", call, sb, nbytes, agree)
        del d, out, ns, ref_out, ref_ns
        torch.cuda.empty_cache()

    with open(path, "w") as f:
        json.dump(res, f, indent=1)
    return res


def run_profile_prefill(args):
    """A few variable-length prefill calls on cuda:0 (16/32 heads, unit-norm q/k), then
    exit: the command that ncu captures for the prefill kernels."""
    import gdn_b200
    from gdn_b200 import synthetic

    dev = torch.device("cuda:0")
    lengths = [int(x) for x in args.profile_prefill.split(",")]
    d = synthetic.make_prefill_inputs(lengths, seed=11, device=dev)
    total, N = sum(lengths), len(lengths)
    out = torch.empty((total, HV, DIM), dtype=torch.bfloat16, device=dev)
    ns = torch.empty((N, HV, DIM, DIM), dtype=torch.float32, device=dev)
    for _ in range(args.launches):
        gdn_b200.kernel_prefill_b200(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                     d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"], out, ns)
    torch.cuda.synchronize(dev)
    print(f"profile prefill ok: lengths={lengths[:4]}{'...' if N > 4 else ''} x{N} "
          f"launches={args.launches}")


def run_profile_case(args):
    """A few launches of one fixed decode case on cuda:0, then exit: the command that
    ncu captures.  Batch 128 holds 256 MiB of fp32 state, more than the 126 MB L2 (so
    DRAM counters mean something) and far below the sizes that make captures slow."""
    import gdn_b200
    from gdn_b200 import synthetic

    dev = torch.device("cuda:0")
    B, T = args.profile_case, args.T
    slots = 4 * B if args.pooled else B
    inp = synthetic.make_inputs(B=B, T=T, slots=slots, seed=0, device=dev)
    idx = synthetic.make_pool_indices(B, slots, seed=0, n_pad=1, device=dev) if args.pooled else None
    out = torch.empty((B, T, HV, DIM), dtype=torch.bfloat16, device=dev)
    if args.bf16_state:
        inp.state = inp.state.to(torch.bfloat16)
    if args.gated_norm:
        z = torch.randn((B, T, HV, DIM), device=dev).to(torch.bfloat16)
        w = torch.ones(DIM, device=dev, dtype=torch.bfloat16)
    for _ in range(args.launches):
        if args.gated_norm:
            gdn_b200.gdn_decode_gated_norm(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a,
                                           inp.dt_bias, inp.b, z, w, scale=inp.scale, output=out)
        elif args.bf16_state:
            gdn_b200.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a,
                                       inp.dt_bias, inp.b, inp.scale, out, state_indices=idx)
        else:
            gdn_b200.decode_tuned(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias,
                                  inp.b, inp.scale, out, state_indices=idx)
    torch.cuda.synchronize(dev)
    print(f"profile case ok: B={B} T={T} pooled={args.pooled} bf16_state={args.bf16_state} "
          f"gated_norm={args.gated_norm} launches={args.launches}")


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline leg")
    ap.add_argument("--skip-b1", action="store_true", help="omit the B=1 latency leg")
    ap.add_argument("--skip-configs", action="store_true",
                    help="omit BASELINE's other single-GPU configurations")
    ap.add_argument("--config-iters", type=int, default=50,
                    help="CUPTI launches per configuration")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--clock-sampler", choices=["nvml", "smi", "none"], default="nvml",
                    help="how rank 0 samples clocks during the timed region")
    ap.add_argument("--tp-collective", choices=["peer", "nccl"], default="peer",
                    help="output exchange at N > 1: fused peer stores (default) or NCCL")
    ap.add_argument("--profile-case", type=int, default=0, metavar="B",
                    help="run --launches decode steps at batch B on cuda:0 and exit (for ncu)")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--T", type=int, default=1, help="tokens per step of --profile-case")
    ap.add_argument("--pooled", action="store_true",
                    help="--profile-case: pool of 4*B slots, one -1 index")
    ap.add_argument("--bf16-state", action="store_true", help="--profile-case: bf16 state")
    ap.add_argument("--gated-norm", action="store_true",
                    help="--profile-case: the step fused with the gated RMSNorm")
    ap.add_argument("--profile-prefill", default=None, metavar="LENGTHS",
                    help="run --launches prefill calls with these comma-separated sequence "
                         "lengths on cuda:0 and exit (for ncu)")
    ap.add_argument("--compare", default=None, metavar="PATH",
                    help="time FlashInfer's and fla's decode kernels beside this one on cuda:0, "
                         "write the table as JSON to PATH and exit")
    ap.add_argument("--compare-group", choices=COMPARE_GROUPS, default=None,
                    help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
        return
    if args.profile_prefill:
        run_profile_prefill(args)
        return
    if args.compare:
        if args.compare_group is None:
            run_compare_isolated(args.config_iters, args.compare)
            return
        dev = torch.device("cuda:0")
        torch.cuda.set_device(dev)
        run_compare(dev, args.config_iters, args.compare, group=args.compare_group)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local_rank = dist_env()
    if world != args.gpus:
        log(f"[bench] WORLD_SIZE={world} but --gpus {args.gpus}; using WORLD_SIZE")
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    run_b200_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
