"""A second, independent pin of the oracle: the naive PyTorch recurrence of the
flash-linear-attention package (fla 0.5.1, installed in the image;
fla/ops/gated_delta_rule/naive.py ``naive_recurrent_gated_delta_rule``), which the
reference's Triton decode kernel was taken from (solution/triton/kernel.py:200-203).

fla keeps the state K-first ([B, H, K, V]), has no GVA (q/k are given per v-head),
takes the decay as its logarithm (h <- h * exp(g)) and applies ``scale`` to q
before the recurrence.  The test converts between the conventions and compares
the oracle's multi-token loop (``decode_mtp``) with it on the same inputs.  The
module is loaded from its file, so nothing of fla's Triton side is imported.
"""

import importlib.util
import os

import pytest
import torch
import torch.nn.functional as F

from gdn_b200 import synthetic
from oracle import gdn_ref


def _fla_naive():
    spec = importlib.util.find_spec("fla")
    if spec is None or spec.origin is None:
        pytest.skip("fla not installed")
    path = os.path.join(os.path.dirname(spec.origin), "ops", "gated_delta_rule", "naive.py")
    if not os.path.exists(path):
        pytest.skip("fla/ops/gated_delta_rule/naive.py not present")
    s = importlib.util.spec_from_file_location("_fla_gdr_naive", path)
    mod = importlib.util.module_from_spec(s)
    s.loader.exec_module(mod)
    return mod.naive_recurrent_gated_delta_rule


def _unit_rows(x: torch.Tensor) -> torch.Tensor:
    x = x.float()
    return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)


def _via_fla(naive, inp):
    """fla's recurrence on the oracle's inputs: (outputs [B,T,HV,V] fp32,
    final state [B,HV,V,K] fp32)."""
    B, T, H, K = inp.q.shape
    HV = inp.v.shape[2]
    rep = HV // H
    q = inp.q.float().repeat_interleave(rep, dim=2)
    k = inp.k.float().repeat_interleave(rep, dim=2)
    log_g = -torch.exp(inp.A_log.float()) * F.softplus(inp.a.float() + inp.dt_bias.float())
    beta = torch.sigmoid(inp.b.float())
    h0 = inp.state.float().transpose(-1, -2).contiguous()          # [B,HV,K,V]
    o, hT = naive(q, k, inp.v.float(), beta, log_g, scale=inp.scale, initial_state=h0,
                  output_final_state=True)
    return o, hT.transpose(-1, -2).contiguous()


@pytest.mark.parametrize("T,H,HV", [(1, 4, 8), (4, 4, 8), (3, 16, 32)])
def test_oracle_matches_fla_naive_unit_keys(T, H, HV):
    naive = _fla_naive()
    inp = synthetic.make_inputs(B=2, T=T, H=H, HV=HV, seed=40 + T)
    inp.q, inp.k = _unit_rows(inp.q), _unit_rows(inp.k)
    out, pool, inter = gdn_ref.decode_mtp(inp.q, inp.k, inp.v, inp.state, None, inp.A_log,
                                          inp.a, inp.dt_bias, inp.b, inp.scale)
    o_fla, s_fla = _via_fla(naive, inp)
    torch.testing.assert_close(pool, s_fla, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(inter[:, -1], s_fla, atol=1e-5, rtol=1e-5)
    # the oracle rounds its outputs to bf16 (kernel.py:117)
    torch.testing.assert_close(out.float(), o_fla.to(torch.bfloat16).float(), atol=1e-2,
                               rtol=1e-2)
    assert (out.float() - o_fla).abs().max() <= 2 ** -7 * o_fla.abs().max() + 1e-3


def test_oracle_matches_fla_naive_raw_keys_two_tokens():
    """Raw N(0,1) keys (|k|^2 ~ 128): the state grows by ~|1 - beta |k|^2| per token,
    so fp32 rounding differences grow with it; compare relative to the magnitude."""
    naive = _fla_naive()
    inp = synthetic.make_inputs(B=2, T=2, H=4, HV=8, seed=47)
    _, pool, _ = gdn_ref.decode_mtp(inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a,
                                    inp.dt_bias, inp.b, inp.scale)
    _, s_fla = _via_fla(naive, inp)
    scale = s_fla.abs().max()
    assert (pool - s_fla).abs().max() <= 1e-5 * scale
