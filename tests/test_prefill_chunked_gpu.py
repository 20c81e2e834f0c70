"""GPU parity of the chunked tensor-core prefill (``gdn_prefill_chunked``: tcgen05
products with the state in tensor memory, inputs by TMA) against the reference's
varlen prefill loop (golden fixtures from kernel_prefill_reference,
solution/triton/prefill_kernel.py:85-183), the oracle's restatement of it and this
library's token-loop kernel.

The chunked form reorders the arithmetic (64-token blocks, split-bf16 and tf32
products with fp32 accumulation), so results agree within tolerances, not bit for bit:
bf16 outputs within atol = rtol = 1e-2 and fp32 states within atol = rtol = 1e-3, the
path's tolerances.  Long sequences use unit-norm q/k, as a model's q/k producer gives
them (raw N(0, 1) keys grow the state by up to |1 - beta*|k|^2| per token).
"""

import pytest
import torch

import golden_io
import gdn_b200
from gdn_b200 import synthetic
from oracle import gdn_ref

pytestmark = pytest.mark.gpu

OUT_TOL = dict(atol=1e-2, rtol=1e-2)
STATE_TOL = dict(atol=1e-3, rtol=1e-3)
DEV = "cuda"


def run_chunked(d, in_place=False):
    g = {n: (t.to(DEV) if isinstance(t, torch.Tensor) else t) for n, t in d.items()}
    total, HV = g["v"].shape[0], g["v"].shape[1]
    N = g["cu_seqlens"].numel() - 1
    out = torch.full((total, HV, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    ns = g["state"] if in_place else torch.full((N, HV, 128, 128), float("nan"), device=DEV)
    status = gdn_b200.prefill_chunked(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                      g["dt_bias"], g["b"], g["cu_seqlens"], g["scale"], out, ns)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, ns


def check_oracle(d, in_place=False):
    want_o, want_s = gdn_ref.prefill_varlen(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                            d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"])
    out, ns = run_chunked(d, in_place)
    torch.testing.assert_close(out.float().cpu(), want_o.float(), **OUT_TOL)
    torch.testing.assert_close(ns.cpu(), want_s, **STATE_TOL)


@pytest.mark.parametrize("lengths", [[64], [1], [63], [65], [130, 7, 0, 200], [128, 64, 1]])
def test_ragged_sequences_match_oracle(lengths):
    check_oracle(synthetic.make_prefill_inputs(lengths, seed=sum(lengths)))


def test_contest_heads_no_initial_state_and_in_place():
    check_oracle(synthetic.make_prefill_inputs([6, 70], H=4, HV=8, seed=2, with_state=False))
    check_oracle(synthetic.make_prefill_inputs([100], seed=3), in_place=True)


def test_long_sequence_1024_tokens():
    check_oracle(synthetic.make_prefill_inputs([1024], seed=5))


@pytest.mark.parametrize("name", ["prefill_qk4v8_ragged", "prefill_qk4v8_ragged_nostate"])
def test_golden_ragged(name):
    meta, inp, gold = golden_io.load(name)
    d = dict(q=inp.q[0], k=inp.k[0], v=inp.v[0], state=inp.state if meta["initial_state"] else None,
             A_log=inp.A_log, a=inp.a[0], dt_bias=inp.dt_bias, b=inp.b[0],
             cu_seqlens=torch.tensor(meta["cu_seqlens"], dtype=torch.int32), scale=inp.scale)
    out, ns = run_chunked(d)
    torch.testing.assert_close(out.float().cpu(), gold["output"].float(), **OUT_TOL)
    torch.testing.assert_close(ns.cpu(), gold["new_state"], **STATE_TOL)


def test_matches_the_token_loop_on_a_batch_of_prompts():
    """8 prompts of 512 tokens at 16/32 heads: chunked against this library's token loop
    (gdn_prefill_tuned, the register-resident kernel) on the GPU."""
    d = synthetic.make_prefill_inputs([512] * 8, seed=8, device=DEV)
    out, ns = run_chunked(d)
    ref_o = torch.empty_like(out)
    ref_s = torch.empty_like(ns)
    gdn_b200.prefill_tuned(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                           d["b"], d["cu_seqlens"], d["scale"], ref_o, ref_s)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ref_o.float(), **OUT_TOL)
    torch.testing.assert_close(ns, ref_s, **STATE_TOL)


def test_dispatch_of_the_default_entry_matches_the_oracle():
    """gdn_prefill picks the chunked kernel for sequences of 32 tokens or more on average
    and the token loop below; both agree with the oracle."""
    for lengths in ([80, 40], [5, 9, 2]):
        d = synthetic.make_prefill_inputs(lengths, seed=len(lengths))
        want_o, want_s = gdn_ref.prefill_varlen(d["q"], d["k"], d["v"], d["state"], d["A_log"],
                                                d["a"], d["dt_bias"], d["b"], d["cu_seqlens"],
                                                d["scale"])
        g = {n: (t.to(DEV) if isinstance(t, torch.Tensor) else t) for n, t in d.items()}
        o, s = gdn_b200.gdn_prefill(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                    g["dt_bias"], g["b"], g["cu_seqlens"], g["scale"])
        torch.cuda.synchronize()
        torch.testing.assert_close(o.float().cpu(), want_o.float(), **OUT_TOL)
        torch.testing.assert_close(s.cpu(), want_s, **STATE_TOL)


def test_offsets_outside_the_tokens_are_clamped():
    d = synthetic.make_prefill_inputs([80], seed=7)
    d["cu_seqlens"] = torch.tensor([0, 70, 60, 1000], dtype=torch.int32)
    d["state"] = torch.cat([d["state"]] * 3)
    _, ns = run_chunked(d)
    for s, (t0, t1) in enumerate([(0, 70), (70, 70), (60, 80)]):
        sl = slice(t0, t1)
        _, want_s = gdn_ref.prefill_varlen(d["q"][sl], d["k"][sl], d["v"][sl], d["state"][s:s + 1],
                                           d["A_log"], d["a"][sl], d["dt_bias"], d["b"][sl],
                                           torch.tensor([0, t1 - t0], dtype=torch.int32),
                                           d["scale"])
        torch.testing.assert_close(ns[s].cpu(), want_s[0], **STATE_TOL)
    assert torch.all(ns[1] == 0)
