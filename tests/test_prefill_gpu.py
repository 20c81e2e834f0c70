"""GPU parity of the variable-length prefill (``gdn_prefill`` / ``kernel_prefill_b200``)
against the reference's varlen prefill loop (golden fixtures made from
kernel_prefill_reference, solution/triton/prefill_kernel.py:85-183) and the oracle's
restatement of it, ``oracle.gdn_ref.prefill_varlen``.

Tolerances: bf16 outputs within atol = rtol = 1e-2, fp32 states within
atol = rtol = 1e-3.  Long sequences use unit-norm keys, as a model's q/k producer
gives them; raw N(0,1) keys grow the state by up to |1 - beta*|k|^2| per token.
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


def flat_inputs(lengths, H=16, HV=32, seed=0, unit_keys=True, with_state=True):
    """Token-major prefill inputs for sequences of the given lengths (CPU)."""
    return synthetic.make_prefill_inputs(lengths, H=H, HV=HV, seed=seed, unit_qk=unit_keys,
                                         with_state=with_state)


def to_dev(d):
    return {n: (t.to(DEV) if isinstance(t, torch.Tensor) else t) for n, t in d.items()}


def check(d, l2=False, in_place=False):
    want_o, want_s = gdn_ref.prefill_varlen(d["q"], d["k"], d["v"], d["state"], d["A_log"],
                                            d["a"], d["dt_bias"], d["b"], d["cu_seqlens"],
                                            d["scale"], use_qk_l2norm=l2)
    g = to_dev(d)
    total, HV = g["v"].shape[0], g["v"].shape[1]
    N = g["cu_seqlens"].numel() - 1
    out = torch.full((total, HV, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    if in_place:
        new_state = g["state"]
    else:
        new_state = torch.full((N, HV, 128, 128), float("nan"), device=DEV)
    before = None if g["state"] is None else g["state"].clone()
    gdn_b200.kernel_prefill_b200(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                 g["dt_bias"], g["b"], g["cu_seqlens"], g["scale"], out,
                                 new_state, use_qk_l2norm=l2)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), want_o.float(), **OUT_TOL)
    torch.testing.assert_close(new_state.cpu(), want_s, **STATE_TOL)
    if before is not None and not in_place:
        assert torch.equal(g["state"], before)           # the initial state is read only
    return out, new_state


@pytest.mark.parametrize("name", ["prefill_qk4v8_ragged", "prefill_qk4v8_ragged_nostate",
                                  "mtp_prefill_qk4v8_b2_t4"])
def test_golden_prefill(name):
    meta, inp, gold = golden_io.load(name)
    if "cu_seqlens" in meta:
        cu = torch.tensor(meta["cu_seqlens"], dtype=torch.int32)
        q, k, v, a, b = inp.q[0], inp.k[0], inp.v[0], inp.a[0], inp.b[0]
        state = inp.state if meta["initial_state"] else None
    else:
        B, T = meta["B"], meta["T"]
        cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int32)
        q, k, v, a, b = (x.reshape(B * T, *x.shape[2:]) for x in (inp.q, inp.k, inp.v, inp.a,
                                                                  inp.b))
        state = inp.state
    g = to_dev(dict(q=q, k=k, v=v, state=state, A_log=inp.A_log, a=a, dt_bias=inp.dt_bias, b=b,
                    cu=cu))
    out, new_state = gdn_b200.gdn_prefill(g["q"], g["k"], g["v"], g["state"], g["A_log"],
                                          g["a"], g["dt_bias"], g["b"], g["cu"], inp.scale)
    torch.cuda.synchronize()
    want_out = gold["output"].reshape(out.shape)
    torch.testing.assert_close(out.float().cpu(), want_out.float(), **OUT_TOL)
    torch.testing.assert_close(new_state.cpu(), gold["new_state"], **STATE_TOL)


@pytest.mark.parametrize("lengths", [[1], [6], [1, 17, 0, 64, 5], [0, 0, 3], [128, 2]])
@pytest.mark.parametrize("in_place", [False, True])
def test_ragged_sequences_match_oracle(lengths, in_place):
    check(flat_inputs(lengths, seed=sum(lengths)), in_place=in_place)


def test_no_initial_state_and_qk_l2norm():
    d = flat_inputs([9, 0, 4], seed=3, unit_keys=False, with_state=False)
    check(d, l2=True)


def test_contest_head_config_and_int64_offsets():
    d = flat_inputs([5, 11], H=4, HV=8, seed=4)
    d["cu_seqlens"] = d["cu_seqlens"].long()
    check(d)


def test_long_sequence_sampled_heads():
    """One 1024-token sequence, 16/32 heads (the state runs through 1024 dependent
    updates); all outputs and the final state against the oracle."""
    check(flat_inputs([1024], seed=5))


@pytest.mark.parametrize("shape", [(8, 1, 1), (8, 2, 1), (8, 4, 1), (8, 1, 4), (16, 1, 1)])
def test_every_built_work_split_matches_the_default(shape):
    """Splits with the default 8 lanes per row reduce in the same order: bit-identical.
    16 lanes per row add the partial sums in another order: within the tolerances."""
    d = to_dev(flat_inputs([7, 33, 1], seed=6))
    total, N = d["v"].shape[0], d["cu_seqlens"].numel() - 1
    ref_o, ref_s = gdn_b200.gdn_prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                        d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"])
    out = torch.empty_like(ref_o)
    ns = torch.empty_like(ref_s)
    gdn_b200.prefill_tuned(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                           d["b"], d["cu_seqlens"], d["scale"], out, ns, *shape)
    torch.cuda.synchronize()
    if shape[0] == 8:
        assert torch.equal(out, ref_o) and torch.equal(ns, ref_s)
    else:
        torch.testing.assert_close(out.float(), ref_o.float(), **OUT_TOL)
        torch.testing.assert_close(ns, ref_s, **STATE_TOL)


def test_offsets_outside_the_tokens_are_clamped():
    """Malformed cu_seqlens (decreasing, beyond the token count) cannot address memory
    outside the inputs: bounds clamp to [0, total], a sequence whose end precedes its
    start is empty (zero final state)."""
    d = flat_inputs([8], seed=7)
    d["cu_seqlens"] = torch.tensor([0, 5, 3, 100], dtype=torch.int32)
    d["state"] = torch.cat([d["state"]] * 3)
    g = to_dev(d)
    out = torch.zeros((8, 32, 128), dtype=torch.bfloat16, device=DEV)
    ns = torch.full((3, 32, 128, 128), float("nan"), device=DEV)
    gdn_b200.kernel_prefill_b200(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                 g["dt_bias"], g["b"], g["cu_seqlens"], g["scale"], out, ns)
    torch.cuda.synchronize()
    for s, (t0, t1) in enumerate([(0, 5), (5, 5), (3, 8)]):
        cu = torch.tensor([0, t1 - t0], dtype=torch.int32)
        sl = slice(t0, t1)
        _, want_s = gdn_ref.prefill_varlen(d["q"][sl], d["k"][sl], d["v"][sl], d["state"][s:s + 1],
                                           d["A_log"], d["a"][sl], d["dt_bias"], d["b"][sl], cu,
                                           d["scale"])
        torch.testing.assert_close(ns[s].cpu(), want_s[0], **STATE_TOL)
    assert torch.all(ns[1] == 0)
