"""The decode step behind the reference's native boundary: the TVM-FFI function
``kernel_cuda_b200`` in libgdn_b200_tvm.so, with the signature of the reference's
``kernel_cuda`` export (solution/cuda/kernel.cu:216-254), called the way
solution/cuda/binding.py:35-41 calls it (torch tensors straight into the FFI
function, destination-passing)."""

import os

import pytest
import torch

tvm_ffi = pytest.importorskip("tvm_ffi")

from gdn_b200 import build, synthetic  # noqa: E402
from oracle import gdn_ref  # noqa: E402


@pytest.fixture(scope="module")
def tvm_mod():
    path = build.build_tvm_ffi()
    assert path is not None and os.path.exists(path)
    return tvm_ffi.load_module(path)


def test_module_exports_kernel(tvm_mod):
    fn = getattr(tvm_mod, "kernel_cuda_b200")
    assert callable(fn)


@pytest.mark.gpu
@pytest.mark.parametrize("heads", [(4, 8), (16, 32)])
def test_tvm_ffi_call_matches_oracle(tvm_mod, heads):
    H, HV = heads
    inp = synthetic.make_inputs(B=3, H=H, HV=HV, seed=61)
    want_out, want_state = gdn_ref.decode(*inp.args())
    g = inp.to("cuda")
    out = torch.empty((3, 1, HV, 128), dtype=torch.bfloat16, device="cuda")
    new_state = torch.empty_like(g.state)
    tvm_mod.kernel_cuda_b200(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, 0.0, out,
                             new_state)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), want_out.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(new_state.cpu(), want_state, atol=1e-3, rtol=1e-3)
    assert torch.equal(g.state.cpu(), inp.state)       # disjoint new_state: input untouched


@pytest.mark.gpu
def test_tvm_ffi_rejects_bad_dtype(tvm_mod):
    g = synthetic.make_inputs(B=1, seed=62).to("cuda")
    out = torch.empty((1, 1, 32, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(Exception, match="output"):
        tvm_mod.kernel_cuda_b200(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, 0.0, out,
                                 g.state)
