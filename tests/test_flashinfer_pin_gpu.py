"""This repository's decode kernels against FlashInfer's, on the same GPU and the
same inputs: the fp32 k-last decode that the reference's kernel_fi_baseline calls
(solution/triton/kernel.py:124-147), its multi-token path, and the bf16-state
backend (flashinfer/gdn_decode.py:255-261) that ``gdn_decode_bf16_state`` stands in
for.  The bf16 comparison pins the bf16-state semantics (fp32 arithmetic, the state
rounded to bf16 when stored) against the kernel it replaces, beyond this
repository's own oracle.

FlashInfer is library code installed in the image; these tests skip where it
cannot be imported.  Tolerances are the path's: bf16 outputs within
atol = rtol = 1e-2, fp32 states within atol = rtol = 1e-3, and bf16 states within
one bf16 rounding step (rtol = 2^-7) plus atol = 1e-3.
"""

import pytest
import torch

import gdn_b200
from gdn_b200 import synthetic

pytestmark = pytest.mark.gpu

OUT_TOL = dict(atol=1e-2, rtol=1e-2)
STATE_TOL = dict(atol=1e-3, rtol=1e-3)
BF16_STATE_TOL = dict(atol=1e-3, rtol=2.0 ** -7)


@pytest.fixture(scope="module")
def fi():
    return pytest.importorskip("flashinfer.gdn_decode")


def _l2normed(inp):
    """Unit-norm keys keep multi-step states bounded (|1 - beta |k|^2| <= 1)."""
    k = inp.k.float()
    inp.k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    return inp


@pytest.mark.parametrize("B", [1, 8, 33])
def test_fp32_decode_matches_flashinfer(fi, B):
    inp = synthetic.make_inputs(B=B, seed=800 + B, device="cuda")
    mine, theirs = inp.clone(), inp.clone()
    out_m = torch.empty((B, 1, 32, 128), dtype=torch.bfloat16, device="cuda")
    out_t = torch.empty_like(out_m)
    gdn_b200.kernel_cuda_b200(*mine.args(), out_m, mine.state)
    fi.gated_delta_rule_decode_pretranspose(
        theirs.q, theirs.k, theirs.v, theirs.state, theirs.A_log, theirs.a, theirs.dt_bias,
        theirs.b, scale=theirs.scale, output=out_t, use_qk_l2norm=False)
    torch.cuda.synchronize()
    torch.testing.assert_close(out_m.float(), out_t.float(), **OUT_TOL)
    torch.testing.assert_close(mine.state, theirs.state, **STATE_TOL)


@pytest.mark.parametrize("T", [2, 4])
def test_fp32_mtp_matches_flashinfer(fi, T):
    B = 6
    inp = _l2normed(synthetic.make_inputs(B=B, T=T, seed=820 + T, device="cuda"))
    mine, theirs = inp.clone(), inp.clone()
    idx = torch.arange(B, dtype=torch.int32, device="cuda")
    inter_m = torch.empty((B, T, 32, 128, 128), device="cuda")
    inter_t = torch.empty_like(inter_m)
    out_m, _ = gdn_b200.gated_delta_rule_mtp(
        mine.q, mine.k, mine.v, mine.state, idx, mine.A_log, mine.a, mine.dt_bias, mine.b,
        mine.scale, None, inter_m, disable_state_update=False, use_qk_l2norm=False)
    out_t, _ = fi.gated_delta_rule_mtp(
        theirs.q, theirs.k, theirs.v, theirs.state, idx, theirs.A_log, theirs.a,
        theirs.dt_bias, theirs.b, scale=theirs.scale, intermediate_states_buffer=inter_t,
        disable_state_update=False, use_qk_l2norm=False)
    torch.cuda.synchronize()
    torch.testing.assert_close(out_m.float(), out_t.float(), **OUT_TOL)
    torch.testing.assert_close(mine.state, theirs.state, **STATE_TOL)
    torch.testing.assert_close(inter_m, inter_t, **STATE_TOL)


@pytest.mark.parametrize("B,T,l2", [(1, 1, False), (16, 1, False), (16, 1, True), (8, 2, False)])
def test_bf16_state_matches_flashinfer_bf16_backend(fi, B, T, l2):
    inp = _l2normed(synthetic.make_inputs(B=B, T=T, seed=840 + B + T, device="cuda"))
    inp.state = inp.state.to(torch.bfloat16)
    mine, theirs = inp.clone(), inp.clone()
    out_m = gdn_b200.decode_bf16_state(mine.q, mine.k, mine.v, mine.state, mine.A_log, mine.a,
                                       mine.dt_bias, mine.b, mine.scale, use_qk_l2norm=l2)
    out_t, _ = fi.gated_delta_rule_decode_pretranspose(
        theirs.q, theirs.k, theirs.v, theirs.state, theirs.A_log, theirs.a, theirs.dt_bias,
        theirs.b, scale=theirs.scale, use_qk_l2norm=l2)
    torch.cuda.synchronize()
    torch.testing.assert_close(out_m.float(), out_t.float(), **OUT_TOL)
    torch.testing.assert_close(mine.state.float(), theirs.state.float(), **BF16_STATE_TOL)
    same = (mine.state.view(torch.int16) == theirs.state.view(torch.int16)).float().mean().item()
    print(f"bf16 state B={B} T={T} l2={l2}: {same:.6f} of elements bit-identical")
