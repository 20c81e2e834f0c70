"""Device-time measurement used by the benchmark and the comparison tests.

Kernel durations come from CUPTI activity records through torch.profiler — the
GPU-side start/end of each launch, without host launch overhead — which is the
method the reference quotes its microsecond numbers with
(flashinfer.testing.bench_gpu_time(enable_cupti=True, cold_l2_cache=True),
scripts/bench_fi_timing.py:43-48).  A cold L2 is made the same way: a buffer
larger than the 126 MB L2 is zeroed before every launch.
"""

from __future__ import annotations

from typing import Callable, Dict, List, Optional, Tuple

import torch

L2_FLUSH_BYTES = 256 * 1024 * 1024


# The L2 flush is `buf.bitwise_not_()` on an int32 buffer larger than L2: a kernel
# whose name (torch's bitwise_not kernel) no timed implementation launches, so the
# timing helpers can drop it by name even when a profiling session misses records.
FLUSH_KERNEL_TAG = "bitwise_not"


def l2_flush_buffer(device) -> torch.Tensor:
    """int32 buffer of 256 MiB; flush L2 with ``buf.bitwise_not_()``."""
    return torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)


def cupti_kernel_durations_us(fn: Callable[[], object], iters: int, device,
                              name: str = "gdn_step_kernel",
                              flush: Optional[Callable[[], object]] = None) -> List[float]:
    """Device durations (µs) of the kernels whose name contains ``name`` over
    ``iters`` calls of ``fn``; ``flush`` runs before every call."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(iters):
            if flush is not None:
                flush()
            fn()
        torch.cuda.synchronize(device)
    out = []
    for e in prof.profiler.kineto_results.events():
        if name in e.name() and str(e.device_type()).endswith("CUDA"):
            out.append(e.duration_ns() / 1e3)
    return out


def _kernel_records(fn: Callable[[], object], iters: int, device,
                    flush: Optional[Callable[[], object]] = None) -> List[Tuple[str, int, int]]:
    """(name, start ns, end ns) of every kernel launched by ``iters`` calls of ``fn``,
    in start order; kernels that ``flush`` launches (it runs before every call, inside
    the profiled region) are left out by name."""
    from torch.profiler import ProfilerActivity, profile

    flush_names = set()
    if flush is not None:
        # the flush's own kernels, by name (a short session; it can come back without
        # records right after a JIT compile, so the flush's tag is dropped as well)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            flush()
            torch.cuda.synchronize(device)
        flush_names = {e.name() for e in prof.profiler.kineto_results.events()
                       if str(e.device_type()).endswith("CUDA")}
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(iters):
            if flush is not None:
                flush()
            fn()
        torch.cuda.synchronize(device)
    out = []
    for e in prof.profiler.kineto_results.events():
        if not str(e.device_type()).endswith("CUDA") or e.name() in flush_names:
            continue
        if flush is not None and FLUSH_KERNEL_TAG in e.name():
            continue
        if "Memcpy" in e.name() or "Memset" in e.name():
            continue
        out.append((e.name(), e.start_ns(), e.start_ns() + e.duration_ns()))
    out.sort(key=lambda r: r[1])
    return out


def cupti_kernels_by_name(fn: Callable[[], object], iters: int, device,
                          flush: Optional[Callable[[], object]] = None) -> Dict[str, List[float]]:
    """Device durations (µs) of every kernel launched by ``iters`` calls of ``fn``,
    grouped by kernel name; kernels that ``flush`` launches are left out by name."""
    out: Dict[str, List[float]] = {}
    for name, t0, t1 in _kernel_records(fn, iters, device, flush):
        out.setdefault(name, []).append((t1 - t0) / 1e3)
    return out


def cupti_kernels_and_spans(fn: Callable[[], object], iters: int, device,
                            flush: Optional[Callable[[], object]] = None,
                            name_part: str = "gdn_"):
    """``cupti_kernels_by_name``'s durations plus, for calls that launch several kernels
    whose names contain ``name_part`` (each once per call), the span of each call from its
    first kernel's start to its last kernel's end, in µs.  Summing the kernels' durations
    would count twice the time in which a call's kernels overlap (a programmatic
    dependent launched during its predecessor's tail); the span does not.  The spans are
    None when the records do not split into whole calls."""
    recs = _kernel_records(fn, iters, device, flush)
    by_name: Dict[str, List[float]] = {}
    for name, t0, t1 in recs:
        by_name.setdefault(name, []).append((t1 - t0) / 1e3)
    return by_name, call_spans_us(recs, name_part)


def call_spans_us(recs: List[Tuple[str, int, int]], name_part: str = "gdn_"
                  ) -> Optional[List[float]]:
    """Per-call spans (µs) of (name, start ns, end ns) records in start order, for calls
    that launch each kernel whose name contains ``name_part`` exactly once: consecutive
    groups of as many records as there are such names, each group one call.  None when
    the records do not split into whole calls (a dropped or extra record)."""
    mine = [r for r in recs if name_part in r[0]]
    k = len({r[0] for r in mine})
    if k == 0 or len(mine) % k != 0:
        return None
    groups = [mine[i:i + k] for i in range(0, len(mine), k)]
    if not all(len({r[0] for r in g}) == k for g in groups):
        return None
    return [(max(r[2] for r in g) - min(r[1] for r in g)) / 1e3 for g in groups]
