"""GPU parity of the decode step fused with the decode layer's gated RMSNorm
(``gdn_decode_gated_norm``) against the oracle: the reference's decode step
(oracle.gdn_ref.decode, kernel.py:95-114) followed by Qwen3-Next's gated RMSNorm
(oracle.gdn_ref.gated_rmsnorm, transformers models/qwen3_next/modeling_qwen3_next.py:73-82).

Tolerances: bf16 outputs within atol = rtol = 1e-2, fp32 states within 1e-3.
"""

import pytest
import torch

import gdn_b200
from gdn_b200 import synthetic
from oracle import gdn_ref

pytestmark = pytest.mark.gpu

OUT_TOL = dict(atol=1e-2, rtol=1e-2)
STATE_TOL = dict(atol=1e-3, rtol=1e-3)


def gate_inputs(B, HV=32, seed=0):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, 1, HV, 128, generator=gen).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    return z, w


@pytest.mark.parametrize("B,H,HV,l2", [(1, 16, 32, True), (5, 16, 32, False), (3, 4, 8, True),
                                        (64, 16, 32, True)])
def test_fused_gated_norm_matches_decode_then_norm(B, H, HV, l2):
    inp = synthetic.make_inputs(B=B, H=H, HV=HV, seed=60 + B)
    z, w = gate_inputs(B, HV, seed=B)
    want_o, want_s = gdn_ref.decode(*inp.args(), use_qk_l2norm=l2)
    want = gdn_ref.gated_rmsnorm(want_o, z, w, 1e-6)
    g = inp.to("cuda")
    out = gdn_b200.gdn_decode_gated_norm(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b,
                                         z.cuda(), w.cuda(), scale=g.scale, eps=1e-6,
                                         use_qk_l2norm=l2)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), want.float(), **OUT_TOL)
    torch.testing.assert_close(g.state.cpu(), want_s, **STATE_TOL)


def test_fused_equals_unfused_kernels_on_the_gpu():
    """The fused epilogue against this library's plain decode kernel followed by the
    norm written in PyTorch on the GPU, same inputs: the state is bit-identical (same
    arithmetic), the normalised outputs agree within one bf16 rounding step."""
    B = 8
    inp = synthetic.make_inputs(B=B, seed=71)
    z, w = gate_inputs(B, seed=71)
    a, b = inp.to("cuda"), inp.to("cuda")
    fused = gdn_b200.gdn_decode_gated_norm(a.q, a.k, a.v, a.state, a.A_log, a.a, a.dt_bias, a.b,
                                           z.cuda(), w.cuda(), scale=a.scale,
                                           use_qk_l2norm=True)
    o, _ = gdn_b200.gated_delta_rule_decode_pretranspose(
        b.q, b.k, b.v, b.state, b.A_log, b.a, b.dt_bias, b.b, scale=b.scale, use_qk_l2norm=True)
    unfused = gdn_ref.gated_rmsnorm(o, z.cuda(), w.cuda(), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(a.state, b.state)
    torch.testing.assert_close(fused.float(), unfused.float(), rtol=2 ** -7, atol=1e-3)
