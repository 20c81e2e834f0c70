#!/usr/bin/env python
"""Benchmark of the B200 GDN decode path; rank 0 prints one JSON line.

Workload (a "step"): one Gated DeltaNet decode step of a Qwen3-Next-shaped
layer at batch 256 — 16 q/k heads, 32 v-heads, K = V = 128, T = 1 — with the
fp32 state [256, 32, 128, 128] (512 MiB) updated in place in HBM.  With
``--gpus N`` (torchrun, one process per GPU) the 32 v-heads and their 16 q/k
heads are split across the N ranks (tensor parallel, total work fixed) and
the bf16 outputs are all-gathered over NVLink by NCCL and head-interleaved.

value   algorithmic HBM bytes of the whole job per second (GB/s): 4,219,008 B
        per batch entry + 256 B per call, times steps, over the device time of
        the timed steps (CUDA events, max over ranks).  Inputs are resident
        in HBM; the 512 MiB state exceeds the 126 MB L2, so no flush is needed.
e2e     the same metric through the public API (``kernel_cuda_b200`` / the TP
        step) with the per-step inputs (q, k, v, a, b) copied from pinned host
        memory and the output read back to the host inside the timed region.
latency_b1_us   the B=1 decode kernel's median device duration from CUPTI
        activity records (torch.profiler), L2 flushed before every launch.
roofline        the decode kernel alone (CUDA events around each launch).
cpu_baseline    the reference's CPU algorithm (oracle restatement of
        kernel_pt_reference, its per-head loop) on a bounded sample, host cores.

At N > 1 the output exchange is fused into the decode kernel (each rank stores its
rows into every rank's buffer over NVLink, then a bounded barrier); ``--tp-collective
nccl`` uses NCCL all-gather + the interleave kernel instead.
``--impl reference`` times that CPU implementation alone as the reference arm.
``--sweep PATH`` also writes a batch sweep (B in 1..256, plus the pooled and
multi-token configurations) as JSON to PATH.
"""

from __future__ import annotations

import argparse
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

from gdn_b200.timing import cupti_kernel_durations_us, l2_flush_buffer  # noqa: E402

METRIC = "GDN decode µs (CUPTI) at B=1; state-update HBM GB/s vs peak at B=256"
UNIT = "GB/s"
BATCH, H, HV, DIM = 256, 16, 32, 128
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "gdn_step_kernel_b256.txt")

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
        "config": workload_config(world),
        "cpu_baseline": {"value": round(gbs, 6), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 6), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

def workload_config(world):
    return {
        "workload": "gdn_decode_qwen3next_b256_t1",
        "global_batch": BATCH, "T": 1, "num_qk_heads": H, "num_v_heads": HV, "head_dim": DIM,
        "state": "fp32 [256,32,128,128] k-last, updated in place",
        "parallelism": f"tp{world}",
    }


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
    d = cupti_kernel_durations_us(fn, iters, device, flush=flush_buf.zero_)
    d_warm = cupti_kernel_durations_us(fn, iters, device, flush=None)
    # floor of the method: the same 2 MiB state read and written in place by a plain
    # elementwise kernel (torch mul_), same flush, same CUPTI records
    scratch = inp.state.clone()
    floor = cupti_kernel_durations_us(lambda: scratch.mul_(1.0), iters, device,
                                      name="MulFunctor", flush=flush_buf.zero_)
    res = {"median_us": None, "source": "cupti (torch.profiler activity records)",
           "l2": "flushed before every launch (256 MiB write)", "iters": len(d)}
    if d:
        d.sort()
        res.update(median_us=round(statistics.median(d), 3), p10_us=round(d[len(d) // 10], 3),
                   p90_us=round(d[(9 * len(d)) // 10], 3))
    if d_warm:
        res["median_us_l2_warm"] = round(statistics.median(d_warm), 3)
    if floor:
        res["copy_floor_us"] = round(statistics.median(floor), 3)
        res["copy_floor"] = "torch in-place mul_ of the same 2 MiB state, L2 flushed, CUPTI"
    return res


def sanity_check(state, device, step_fn):
    """Runs the first step and checks, without any reference, that every output
    element is finite and that the state changed (parity with the reference is
    the GPU tests' job)."""
    before = state[:2].clone()
    out = step_fn()
    torch.cuda.synchronize(device)
    return {"outputs_finite": bool(torch.isfinite(out.float()).all()),
            "state_updated": bool(not torch.equal(before, state[:2]))}


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


def run_b200_arm(args, rank, world, local_rank):
    import gdn_b200
    from gdn_b200 import synthetic
    from gdn_b200.tp import HeadShard, TPDecode

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    gdn_b200.load_library()
    shard = HeadShard(rank, world, H, HV)
    hl, hvl = shard.h_local, shard.hv_local

    # Local shard inputs, drawn on the device.  Each step updates one "layer's"
    # state and the next step the next layer's (round robin), like the GDN layers of
    # a model: with enough layers the per-GPU working set stays >= 3x the L2, so no
    # step finds its state cached by the previous one (at N=8 one layer's shard is
    # only 64 MiB).  q/k/v/a/b are shared by the layers.
    inp = synthetic.make_inputs(B=BATCH, H=hl, HV=hvl, seed=1234 + rank, device=device)
    l2_bytes = torch.cuda.get_device_properties(device).L2_cache_size
    state_bytes = inp.state.numel() * inp.state.element_size()
    layers = max(1, math.ceil(3 * l2_bytes / state_bytes))
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    states = [inp.state] + [torch.randn(inp.state.shape, generator=gen, device=device).mul_(0.1)
                            for _ in range(layers - 1)]
    out = torch.empty((BATCH, 1, HV, DIM), dtype=torch.bfloat16, device=device)
    tp = (TPDecode(H=H, HV=HV, max_batch=BATCH, device=device, collective=args.tp_collective)
          if world > 1 else None)

    def layer_args(i):
        return (inp.q, inp.k, inp.v, states[i % layers], inp.A_log, inp.a, inp.dt_bias, inp.b,
                inp.scale)

    def eager_step(i):
        """One step of layer i through the public API."""
        if tp is not None:
            return tp.step(*layer_args(i), out=None if tp.collective == "peer" else out)
        gdn_b200.kernel_cuda_b200(*layer_args(i), out, states[i % layers])
        return out

    # The timed region is one CUDA graph of all K steps (layer i % layers at step i),
    # as a model's decode graph holds all its layers: no host work and no graph
    # boundaries inside it (separate replays of short graphs left 40-60 us idle
    # gaps between them at N > 1).
    K = args.steps
    seq = [layer_args(i) for i in range(K)]
    graph = tp.capture_sequence(seq) if tp is not None else _PlainGraph(device, seq, out)

    step_no = [0]

    def step():
        res = eager_step(step_no[0])
        step_no[0] += 1
        return res

    sanity = sanity_check(states[0], device, step)
    for _ in range(args.warmup):
        step()
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

    total_bytes = synthetic.bytes_per_call(BATCH)            # whole job, all heads
    local_bytes = synthetic.bytes_per_call(BATCH, H=hl, HV=hvl)
    value = total_bytes * K / (elapsed_ms_max / 1e3) / 1e9

    # end to end through the public API, host buffers in pinned memory
    host = {n: getattr(inp, n).cpu().pin_memory() for n in ("q", "k", "v", "a", "b")}
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()
    K_e2e = max(1, min(K, 500))

    def e2e_step():
        for n, t in host.items():
            getattr(inp, n).copy_(t, non_blocking=True)
        res = step()                       # public API call, next layer's state
        out_host.copy_(res, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K_e2e):
        e2e_step()
    e1.record()
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device)
    e2e_value = total_bytes * K_e2e / (e2e_ms / 1e3) / 1e9

    latency = b1_latency(device) if (world == 1 and not args.skip_b1) else None
    sweep = None
    if args.sweep and world == 1:
        sweep = run_sweep(device)
        with open(args.sweep, "w") as f:
            json.dump(sweep, f, indent=1)

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
        del graph, tp
        torch.distributed.destroy_process_group()
    if rank != 0:
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
        "config": dict(workload_config(world), l2=(
            f"inputs larger than L2, no flush: {layers} layer state(s) of {state_bytes >> 20} MiB "
            f"per GPU updated round robin ({(layers * state_bytes) >> 20} MiB >= 3x the "
            f"{l2_bytes >> 20} MiB L2)"), timed_loop=f"one CUDA graph of the {K} steps"),
        "latency_b1_us": latency,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic, "peak_source": peaks["source"],
                     "kernel": "gdn_step_kernel", "kernel_us": round(kernel_ms * 1e3, 2),
                     "algorithmic_bytes_per_launch": local_bytes},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": K_e2e, "api": "gdn_b200.kernel_cuda_b200"
                if world == 1 else "gdn_b200.tp.TPDecode.step (eager, one call per step)"},
        "tp_exchange": None if world == 1 else (
            "fused: decode kernel stores outputs into every rank's buffer over NVLink, "
            "then a one-CTA barrier kernel (roofline.kernel_us covers both); CUDA graphs"
            if args.tp_collective == "peer" else
            "NCCL all_gather_into_tensor + interleave kernel; CUDA graphs"),
        "gpu_launches": launches_per_step * K,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "sanity": sanity,
        "wall_s_timed": round(wall, 4),
    }
    print(json.dumps(line), flush=True)


def run_sweep(device):
    """Batch sweep and the pooled / multi-token configurations (1 GPU)."""
    import gdn_b200
    from gdn_b200 import synthetic

    res = {"decode": [], "pooled": None, "mtp": []}
    for B in (1, 8, 32, 64, 128, 256):
        inp = synthetic.make_inputs(B=B, seed=B, device=device)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        flush_buf = l2_flush_buffer(device) if B < 64 else None
        fn = lambda: gdn_b200.kernel_cuda_b200(*inp.args(), out, inp.state)  # noqa: E731
        for _ in range(10):
            fn()
        d = cupti_kernel_durations_us(fn, 100, device,
                                      flush=None if flush_buf is None else flush_buf.zero_)
        med = statistics.median(d)
        nb = synthetic.bytes_per_call(B)
        res["decode"].append({"B": B, "median_us": round(med, 3), "GBps": round(nb / med / 1e3, 1),
                              "state_updates_per_s": round(B * HV / (med * 1e-6)),
                              "l2": "flushed" if flush_buf is not None else "inputs > L2"})
        del inp, out
    # the same step with the in-kernel q/k L2-norm (FlashInfer's use_qk_l2norm=True;
    # the reference path itself never normalises)
    res["decode_l2norm"] = []
    for B in (1, 64, 256):
        inp = synthetic.make_inputs(B=B, seed=B, device=device)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        flush_buf = l2_flush_buffer(device) if B < 64 else None
        fn = lambda: gdn_b200.gated_delta_rule_decode_pretranspose(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
            out, use_qk_l2norm=True)
        for _ in range(10):
            fn()
        med = statistics.median(cupti_kernel_durations_us(
            fn, 100, device, flush=None if flush_buf is None else flush_buf.zero_))
        nb = synthetic.bytes_per_call(B)
        res["decode_l2norm"].append({"B": B, "median_us": round(med, 3),
                                     "GBps": round(nb / med / 1e3, 1),
                                     "l2": "flushed" if flush_buf is not None else "inputs > L2"})
        del inp, out
    # pooled: pool of 1024 slots, 256 active entries drawn as a permutation, one -1
    P, B = 1024, 256
    inp = synthetic.make_inputs(B=B, slots=P, seed=7, device=device)
    idx = synthetic.make_pool_indices(B, P, seed=7, n_pad=1, device=device)
    out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
    fn = lambda: gdn_b200.gated_delta_rule_decode_pretranspose(  # noqa: E731
        inp.q, inp.k, inp.v, None, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale, out,
        use_qk_l2norm=False, initial_state=inp.state, initial_state_indices=idx)
    for _ in range(10):
        fn()
    med = statistics.median(cupti_kernel_durations_us(fn, 50, device))
    nb = synthetic.bytes_per_call(B, active=B - 1)
    res["pooled"] = {"pool": P, "B": B, "active": B - 1, "median_us": round(med, 3),
                     "GBps": round(nb / med / 1e3, 1)}
    del inp, out
    # bf16-stored state (FlashInfer's bf16-state backend): half the state bytes
    res["bf16_state"] = []
    for B, flushed in ((1, True), (64, False), (256, False)):
        inp = synthetic.make_inputs(B=B, seed=B, device=device)
        inp.state = inp.state.to(torch.bfloat16)
        out = torch.empty((B, 1, HV, DIM), dtype=torch.bfloat16, device=device)
        flush_buf = l2_flush_buffer(device) if flushed else None
        fn = lambda: gdn_b200.decode_bf16_state(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale, out)
        for _ in range(10):
            fn()
        med = statistics.median(cupti_kernel_durations_us(
            fn, 100 if flushed else 50, device, flush=None if flush_buf is None else flush_buf.zero_))
        nb = synthetic.bytes_per_call(B, state_elem_bytes=2)
        res["bf16_state"].append({"B": B, "median_us": round(med, 3),
                                  "GBps": round(nb / med / 1e3, 1),
                                  "l2": "flushed" if flushed else "inputs > L2"})
        del inp, out
    for T in (2, 4):
        B = 64
        inp = synthetic.make_inputs(B=B, T=T, seed=T, device=device)
        out = torch.empty((B, T, HV, DIM), dtype=torch.bfloat16, device=device)
        inter = torch.empty((B, T, HV, DIM, DIM), dtype=torch.float32, device=device)
        fn = lambda: gdn_b200.gated_delta_rule_mtp(  # noqa: E731
            inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a, inp.dt_bias, inp.b,
            inp.scale, out, inter, disable_state_update=False, use_qk_l2norm=False)
        for _ in range(5):
            fn()
        med = statistics.median(cupti_kernel_durations_us(fn, 50, device))
        nb = synthetic.bytes_per_call(B, T=T, intermediates=True)
        res["mtp"].append({"B": B, "T": T, "median_us": round(med, 3),
                           "GBps": round(nb / med / 1e3, 1)})
        del inp, out, inter
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--sweep", default=None, help="also write the batch sweep JSON here")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline leg")
    ap.add_argument("--skip-b1", action="store_true", help="omit the B=1 latency leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--clock-sampler", choices=["nvml", "smi", "none"], default="nvml",
                    help="how rank 0 samples clocks during the timed region")
    ap.add_argument("--tp-collective", choices=["peer", "nccl"], default="peer",
                    help="output exchange at N > 1: fused peer stores (default) or NCCL")
    args = ap.parse_args()
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
