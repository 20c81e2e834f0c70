"""Our decode kernel against the reference's own CUDA decode kernels on the same GPU.

``oracle/build_ref.sh`` compiles the reference's solution/cuda/kernel.cu (TVM-FFI
exports ``kernel_cuda`` = v1, kernel.cu:216-254, and ``kernel_cuda_v4``,
:405-443) from the reference checkout into ``oracle/_ref/libref_kernel.so``.
These tests run both on identical inputs — a GPU-side parity reference next to
the CPU oracle — and skip when that library or tvm_ffi is absent.

With ``GDN_REF_TIMING_OUT=<path>`` set, ``test_timing_report`` also writes CUPTI
medians of the three kernels at B = 1 (L2 flushed / warm), 64 and 256 to
``<path>`` as JSON (a measurement, not an assertion).
"""

import json
import os
import statistics

import pytest
import torch

from gdn_b200 import ops, synthetic
from gdn_b200.timing import cupti_kernel_durations_us, l2_flush_buffer

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref_kernel.so")
SCALE = 128 ** -0.5


@pytest.fixture(scope="module")
def ref_mod():
    tvm_ffi = pytest.importorskip("tvm_ffi")
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_kernel.so not built (oracle/build_ref.sh)")
    return tvm_ffi.load_module(REF_LIB)


def _ours(g, out, new_state):
    ops.kernel_cuda_b200(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, SCALE, out,
                         new_state)


def _ref(ref_mod, sym, g, out, new_state):
    getattr(ref_mod, sym)(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, SCALE, out,
                          new_state)


@pytest.mark.parametrize("sym", ["kernel_cuda", "kernel_cuda_v4"])
@pytest.mark.parametrize("B", [1, 8, 64])
def test_matches_reference_cuda_kernels(ref_mod, sym, B):
    g = synthetic.make_inputs(B=B, seed=300 + B).to("cuda")
    o1 = torch.empty((B, 1, 32, 128), dtype=torch.bfloat16, device="cuda")
    o2 = torch.empty_like(o1)
    s1 = torch.empty_like(g.state)
    s2 = torch.empty_like(g.state)
    _ours(g, o1, s1)
    _ref(ref_mod, sym, g, o2, s2)
    torch.cuda.synchronize()
    torch.testing.assert_close(o1.float(), o2.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(s1, s2, atol=1e-3, rtol=1e-3)


def test_timing_report(ref_mod):
    path = os.environ.get("GDN_REF_TIMING_OUT")
    if not path:
        pytest.skip("set GDN_REF_TIMING_OUT to record the timing comparison")
    dev = torch.device("cuda")
    flush = l2_flush_buffer(dev)
    kernels = {"b200": ("gdn_step_kernel", None), "reference cuda-v1": ("gdn_decode_kernel",
               "kernel_cuda"), "reference cuda-v4": ("gdn_decode_v4_kernel", "kernel_cuda_v4")}
    report = []
    for B, cold in ((1, True), (1, False), (8, True), (64, False), (256, False)):
        g = synthetic.make_inputs(B=B, seed=400 + B, device=dev)
        out = torch.empty((B, 1, 32, 128), dtype=torch.bfloat16, device=dev)
        row = {"B": B, "l2": "flushed" if cold else ("warm" if B < 64 else "inputs > L2")}
        for label, (kname, sym) in kernels.items():
            if sym is None:
                fn = lambda: _ours(g, out, g.state)  # noqa: E731
            else:
                fn = lambda sym=sym: _ref(ref_mod, sym, g, out, g.state)  # noqa: E731
            for _ in range(5):
                fn()
            iters = 200 if B <= 8 else 50
            d = cupti_kernel_durations_us(fn, iters, dev, name=kname,
                                          flush=flush.bitwise_not_ if cold else None)
            med = statistics.median(d)
            row[label] = {"median_us": round(med, 3),
                          "GBps": round(synthetic.bytes_per_call(B) / med / 1e3, 1)}
        report.append(row)
        del g, out
    with open(path, "w") as f:
        json.dump(report, f, indent=1)
