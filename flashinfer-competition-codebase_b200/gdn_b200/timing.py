"""Device-time measurement used by the benchmark and the comparison tests.

Kernel durations come from CUPTI activity records through torch.profiler — the
GPU-side start/end of each launch, without host launch overhead — which is the
method the reference quotes its microsecond numbers with
(flashinfer.testing.bench_gpu_time(enable_cupti=True, cold_l2_cache=True),
scripts/bench_fi_timing.py:43-48).  A cold L2 is made the same way: a buffer
larger than the 126 MB L2 is zeroed before every launch.
"""

from __future__ import annotations

from typing import Callable, Dict, List, Optional

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


def cupti_kernels_by_name(fn: Callable[[], object], iters: int, device,
                          flush: Optional[Callable[[], object]] = None) -> Dict[str, List[float]]:
    """Device durations (µs) of every kernel launched by ``iters`` calls of ``fn``,
    grouped by kernel name; kernels that ``flush`` launches (it runs before every
    call, inside the profiled region) are left out by name."""
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
    out: Dict[str, List[float]] = {}
    for e in prof.profiler.kineto_results.events():
        if not str(e.device_type()).endswith("CUDA") or e.name() in flush_names:
            continue
        if flush is not None and FLUSH_KERNEL_TAG in e.name():
            continue
        if "Memcpy" in e.name() or "Memset" in e.name():
            continue
        out.setdefault(e.name(), []).append(e.duration_ns() / 1e3)
    return out
