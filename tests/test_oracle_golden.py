"""The CPU oracle against the golden vectors produced by the reference itself.

This pins ``oracle/gdn_ref.py`` to the reference's ``kernel_pt_reference`` and
``kernel_prefill_reference`` before any GPU result is compared with the oracle.
Both the loop form (the one the CPU baseline times) and the batched form are
checked.  The oracle runs the same fp32 CPU arithmetic as the reference, so the
bounds here are tight: fp32 states to 1e-5 relative and bf16 outputs to one
bf16 rounding step.
"""

import pytest
import torch

import golden_io
from oracle import gdn_ref


def assert_bf16_close(got, want):
    # bf16 has 8 significant bits: one rounding step is 2**-8 relative.
    torch.testing.assert_close(got.float(), want.float(), rtol=2 ** -7, atol=1e-5)


def assert_state_close(got, want):
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["decode_qk4v8_b1", "decode_qk4v8_b2_edge", "decode_h16hv32_b1"])
@pytest.mark.parametrize("form", ["loop", "batched"])
def test_decode_matches_reference(name, form):
    meta, inp, gold = golden_io.load(name)
    fn = gdn_ref.decode_loop if form == "loop" else gdn_ref.decode
    out, state = fn(*inp.args())
    assert out.dtype == torch.bfloat16 and out.shape == gold["output"].shape
    assert_bf16_close(out, gold["output"])
    assert_state_close(state, gold["new_state"])


def test_edge_fixture_reaches_softplus_threshold():
    meta, inp, _ = golden_io.load("decode_qk4v8_b2_edge")
    x = inp.a.float() + inp.dt_bias
    assert (x > 20).any() and (x < -20).any()
    assert inp.scale == 0.0


def test_mtp_matches_reference():
    meta, inp, gold = golden_io.load("mtp_qk4v8_b1_t3")
    out, pool, inter = gdn_ref.decode_mtp(inp.q, inp.k, inp.v, inp.state, None, inp.A_log,
                                          inp.a, inp.dt_bias, inp.b, inp.scale)
    assert_bf16_close(out, gold["output"])
    assert_state_close(inter, gold["intermediates"])
    assert_state_close(pool, gold["intermediates"][:, -1])
    # the prefill reference's sequential loop lands on the same final state
    torch.testing.assert_close(pool, gold["prefill_state"], rtol=1e-4, atol=1e-4)


def test_mtp_matches_prefill_reference_two_sequences():
    """Two sequences of 4 tokens through the reference's varlen prefill loop
    (prefill_kernel.py:85-183 with cu_seqlens [0, 4, 8])."""
    meta, inp, gold = golden_io.load("mtp_prefill_qk4v8_b2_t4")
    out, pool, _ = gdn_ref.decode_mtp(inp.q, inp.k, inp.v, inp.state, None, inp.A_log,
                                      inp.a, inp.dt_bias, inp.b, inp.scale,
                                      keep_intermediates=False)
    assert_bf16_close(out, gold["output"])
    torch.testing.assert_close(pool, gold["new_state"], rtol=1e-4, atol=1e-4)


def test_mtp_disable_state_update_keeps_pool():
    meta, inp, gold = golden_io.load("mtp_qk4v8_b1_t3")
    out, pool, inter = gdn_ref.decode_mtp(inp.q, inp.k, inp.v, inp.state, None, inp.A_log,
                                          inp.a, inp.dt_bias, inp.b, inp.scale,
                                          disable_state_update=True)
    assert torch.equal(pool, inp.state)
    assert_state_close(inter, gold["intermediates"])


def test_pooled_matches_reference():
    meta, inp, gold = golden_io.load("pooled_qk4v8_p5_b3")
    idx = inp.state_indices
    out, pool = gdn_ref.decode_pooled(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log, inp.a,
                                      inp.dt_bias, inp.b, inp.scale)
    assert_bf16_close(out, gold["output"])
    pad = (idx < 0).nonzero().flatten()
    assert len(pad) == 1 and torch.all(out[pad].float() == 0)
    slots = gold["slots"].long()
    assert_state_close(pool[slots], gold["slot_states"])
    untouched = [s for s in range(pool.shape[0]) if s not in slots.tolist()]
    assert torch.equal(pool[untouched], inp.state[untouched])


def test_grouped_heads_equal_full_heads():
    """Running 16/32 heads at once equals four independent 4/8-head groups: the
    basis on which the 16/32 fixture was made with the 4/8-asserting reference."""
    inp = golden_io.make_inputs(B=2, H=16, HV=32, seed=7)
    out, state = gdn_ref.decode(*inp.args())
    for g in range(4):
        qs, vs = slice(4 * g, 4 * g + 4), slice(8 * g, 8 * g + 8)
        o, s = gdn_ref.decode(inp.q[:, :, qs], inp.k[:, :, qs], inp.v[:, :, vs], inp.state[:, vs],
                              inp.A_log[vs], inp.a[:, :, vs], inp.dt_bias[vs], inp.b[:, :, vs],
                              inp.scale)
        assert_bf16_close(o, out[:, :, vs])
        assert_state_close(s, state[:, vs])


def test_l2norm_equals_prenormalised_inputs():
    inp = golden_io.make_inputs(B=2, H=4, HV=8, seed=11)
    out_n, st_n = gdn_ref.decode(*inp.args(), use_qk_l2norm=True)
    qn = gdn_ref.l2norm(inp.q).to(torch.float32)
    kn = gdn_ref.l2norm(inp.k).to(torch.float32)
    S = inp.state.clone()
    g, beta = gdn_ref.gates(inp.A_log, inp.a, inp.dt_bias, inp.b)
    o, S = gdn_ref._step_batched(qn[:, 0].repeat_interleave(2, 1), kn[:, 0].repeat_interleave(2, 1),
                                 inp.v[:, 0].float(), g[:, 0], beta[:, 0], S, inp.scale)
    assert_state_close(st_n, S)
    assert_bf16_close(out_n, o.unsqueeze(1).to(torch.bfloat16))


@pytest.mark.parametrize("name", ["prefill_qk4v8_ragged", "prefill_qk4v8_ragged_nostate"])
def test_prefill_varlen_matches_reference_ragged(name):
    """Ragged sequences (lengths 6, 0, 7, 7) through the reference's varlen prefill loop
    (prefill_kernel.py:85-183): every token's output and each sequence's final state,
    the empty sequence's final state being zero; with and without an initial state."""
    meta, inp, gold = golden_io.load(name)
    cu = torch.tensor(meta["cu_seqlens"], dtype=torch.int32)
    o, s = gdn_ref.prefill_varlen(inp.q[0], inp.k[0], inp.v[0],
                                  inp.state if meta["initial_state"] else None, inp.A_log,
                                  inp.a[0], inp.dt_bias, inp.b[0], cu, inp.scale)
    assert_bf16_close(o, gold["output"])
    torch.testing.assert_close(s, gold["new_state"], rtol=1e-4, atol=1e-4)
    assert torch.all(s[1] == 0)


def test_prefill_varlen_matches_reference_two_sequences():
    meta, inp, gold = golden_io.load("mtp_prefill_qk4v8_b2_t4")
    B, T = meta["B"], meta["T"]
    flat = lambda x: x.reshape(B * T, *x.shape[2:])    # noqa: E731
    cu = torch.tensor([0, T, 2 * T], dtype=torch.int32)
    o, s = gdn_ref.prefill_varlen(flat(inp.q), flat(inp.k), flat(inp.v), inp.state, inp.A_log,
                                  flat(inp.a), inp.dt_bias, flat(inp.b), cu, inp.scale)
    assert_bf16_close(o.reshape(B, T, *o.shape[1:]), gold["output"])
    torch.testing.assert_close(s, gold["new_state"], rtol=1e-4, atol=1e-4)
