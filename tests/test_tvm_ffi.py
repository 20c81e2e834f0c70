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


def _parameters(source: str, function: str):
    """(type, name) pairs of a C++ function definition's parameter list."""
    import re

    m = re.search(rf"\bvoid\s+{function}\s*\((.*?)\)\s*\{{", source, flags=re.S)
    assert m, function
    params = []
    for p in m.group(1).split(","):
        p = " ".join(p.replace("tvm::ffi::", "").split())
        typ, name = p.rsplit(" ", 1)
        params.append((typ, name))
    return params


def test_export_has_the_reference_signature():
    """kernel_cuda_b200 takes exactly the reference's KernelCuda parameters (types,
    order, names; solution/cuda/kernel.cu:216-227), so flashinfer-bench's
    TVMFFIBuilder calls it like kernel_cuda.  Reads the reference checkout, when
    present, as text."""
    import __graft_entry__

    ref_root = __graft_entry__.reference_root()
    if ref_root is None:
        pytest.skip("reference checkout not present (GDN_REFERENCE_ROOT)")
    ref = os.path.join(ref_root, "solution", "cuda", "kernel.cu")
    ours = os.path.join(os.path.dirname(build.__file__), os.pardir, "csrc", "tvm_ffi_entry.cu")
    theirs = _parameters(open(ref).read(), "KernelCuda")
    mine = _parameters(open(ours).read(), "KernelCudaB200")
    assert len(theirs) == 11
    assert mine == theirs
    assert "TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel_cuda_b200, KernelCudaB200)" in open(ours).read()
