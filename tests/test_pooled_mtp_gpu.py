"""GPU parity of the pooled-state (continuous batching) and multi-token
(speculative verify) variants against the oracle and the golden vectors.

Tolerances: bf16 output within atol = rtol = 1e-2, fp32 state within
atol = rtol = 1e-3 (relative: un-normalised keys grow the state by ~|k|^2 per
token, so multi-token states reach magnitudes in the hundreds).
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


def close_out(got, want):
    torch.testing.assert_close(got.float().cpu(), want.float(), **OUT_TOL)


def close_state(got, want):
    torch.testing.assert_close(got.cpu(), want, **STATE_TOL)


# ---- pooled ------------------------------------------------------------------

def pooled_call(inp, idx, oidx=None, l2=False, bad=None):
    g = inp.to(DEV)
    B, HV = g.v.shape[0], g.v.shape[2]
    out = torch.full((B, 1, HV, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    gdn_b200.gated_delta_rule_decode_pretranspose(
        g.q, g.k, g.v, None, g.A_log, g.a, g.dt_bias, g.b, scale=g.scale, output=out,
        use_qk_l2norm=l2, initial_state=g.state, initial_state_indices=idx.to(DEV),
        output_state_indices=None if oidx is None else oidx.to(DEV), bad_index_count=bad)
    torch.cuda.synchronize()
    return out, g.state


def test_golden_pooled():
    meta, inp, gold = golden_io.load("pooled_qk4v8_p5_b3")
    out, pool = pooled_call(inp, inp.state_indices)
    close_out(out, gold["output"])
    slots = gold["slots"].long()
    close_state(pool[slots.to(DEV)], gold["slot_states"])
    untouched = [s for s in range(5) if s not in slots.tolist()]
    assert torch.equal(pool[untouched].cpu(), inp.state[untouched])


@pytest.mark.parametrize("l2", [False, True])
def test_pool_permutation_with_padding(l2):
    """The benchmark's pooled configuration, scaled down: B=32 of 96 slots, one -1."""
    inp = synthetic.make_inputs(B=32, slots=96, seed=31)
    idx = synthetic.make_pool_indices(32, 96, seed=31, n_pad=1)
    want_out, want_pool = gdn_ref.decode_pooled(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log,
                                                inp.a, inp.dt_bias, inp.b, inp.scale,
                                                use_qk_l2norm=l2)
    out, pool = pooled_call(inp, idx, l2=l2)
    close_out(out, want_out)
    assert torch.all(out[(idx < 0).to(DEV)].float() == 0)
    live = idx[idx >= 0].long()
    close_state(pool[live.to(DEV)], want_pool[live])
    dead = torch.ones(96, dtype=torch.bool)
    dead[live] = False
    assert torch.equal(pool[dead.to(DEV)].cpu(), inp.state[dead])


def test_pool_int64_indices():
    inp = synthetic.make_inputs(B=6, slots=10, seed=32)
    idx = torch.tensor([9, 0, -1, 4, 7, 2], dtype=torch.int64)
    want_out, want_pool = gdn_ref.decode_pooled(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log,
                                                inp.a, inp.dt_bias, inp.b, inp.scale)
    out, pool = pooled_call(inp, idx)
    close_out(out, want_out)
    close_state(pool, want_pool)


def test_output_state_indices_and_null_slot():
    inp = synthetic.make_inputs(B=4, slots=12, seed=33)
    idx = torch.tensor([3, 5, 7, -1], dtype=torch.int32)
    oidx = torch.tensor([8, -1, 10, 11], dtype=torch.int32)   # -1 writes to slot 0
    want_out, want_pool = gdn_ref.decode_pooled(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log,
                                                inp.a, inp.dt_bias, inp.b, inp.scale,
                                                output_state_indices=oidx)
    out, pool = pooled_call(inp, idx, oidx)
    close_out(out, want_out)
    close_state(pool, want_pool)
    assert torch.equal(pool[3].cpu(), inp.state[3])          # read slots keep their values
    assert torch.equal(pool[11].cpu(), inp.state[11])        # entry 3 was padding: no write


def test_out_of_range_indices_are_skipped_and_counted():
    inp = synthetic.make_inputs(B=4, slots=6, seed=34)
    idx = torch.tensor([1, 6, 2, 100], dtype=torch.int32)    # 6 and 100 are out of range
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    want_out, want_pool = gdn_ref.decode_pooled(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log,
                                                inp.a, inp.dt_bias, inp.b, inp.scale)
    out, pool = pooled_call(inp, idx, bad=bad)
    close_out(out, want_out)
    close_state(pool, want_pool)
    assert int(bad.item()) == 2


def test_all_padding():
    inp = synthetic.make_inputs(B=3, slots=4, seed=35)
    idx = torch.full((3,), -1, dtype=torch.int32)
    out, pool = pooled_call(inp, idx)
    assert torch.all(out.float() == 0)
    assert torch.equal(pool.cpu(), inp.state)


def test_pool_without_pool_arguments_uses_state_in_place():
    inp = synthetic.make_inputs(B=3, seed=36)
    want = gdn_ref.decode(*inp.args(), use_qk_l2norm=True)   # FlashInfer's default: l2norm on
    g = inp.to(DEV)
    out, st = gdn_b200.gated_delta_rule_decode_pretranspose(*g.args())
    assert st.data_ptr() == g.state.data_ptr()
    close_out(out, want[0])
    close_state(st, want[1])


# ---- multi-token -------------------------------------------------------------

def mtp_call(inp, idx=None, inter=True, disable=False, l2=False, cache_steps=None):
    g = inp.to(DEV)
    B, T, HV = g.v.shape[0], g.v.shape[1], g.v.shape[2]
    buf = None
    if inter:
        buf = torch.zeros((B, cache_steps or T, HV, 128, 128), device=DEV)
    out, pool = gdn_b200.gated_delta_rule_mtp(
        g.q, g.k, g.v, g.state, None if idx is None else idx.to(DEV), g.A_log, g.a, g.dt_bias,
        g.b, scale=g.scale, intermediate_states_buffer=buf, disable_state_update=disable,
        use_qk_l2norm=l2)
    torch.cuda.synchronize()
    return out, pool, buf


def test_golden_mtp():
    meta, inp, gold = golden_io.load("mtp_qk4v8_b1_t3")
    out, pool, inter = mtp_call(inp)
    close_out(out, gold["output"])
    close_state(inter, gold["intermediates"])
    close_state(pool, gold["intermediates"][:, -1])


def test_golden_prefill_two_sequences():
    """The reference's varlen prefill loop on two 4-token sequences (golden fixture)."""
    meta, inp, gold = golden_io.load("mtp_prefill_qk4v8_b2_t4")
    out, pool, _ = mtp_call(inp, inter=False)
    close_out(out, gold["output"])
    close_state(pool, gold["new_state"])


@pytest.mark.parametrize("T", [2, 4])
def test_mtp_vs_oracle(T):
    """The benchmark's multi-token configuration, scaled down to B=8."""
    inp = synthetic.make_inputs(B=8, T=T, seed=40 + T)
    want_out, want_pool, want_inter = gdn_ref.decode_mtp(
        inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale)
    out, pool, inter = mtp_call(inp)
    close_out(out, want_out)
    close_state(inter, want_inter)
    close_state(pool, want_pool)


def test_mtp_disable_state_update_and_longer_cache():
    inp = synthetic.make_inputs(B=4, T=3, seed=50)
    want_out, _, want_inter = gdn_ref.decode_mtp(
        inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale)
    out, pool, inter = mtp_call(inp, disable=True, cache_steps=5)
    close_out(out, want_out)
    assert torch.equal(pool.cpu(), inp.state)
    close_state(inter[:, :3], want_inter)
    assert torch.all(inter[:, 3:] == 0)


def test_mtp_with_indices_padding_and_l2norm():
    inp = synthetic.make_inputs(B=5, T=2, slots=9, seed=51)
    idx = torch.tensor([8, -1, 0, 4, 2], dtype=torch.int32)
    want_out, want_pool, want_inter = gdn_ref.decode_mtp(
        inp.q, inp.k, inp.v, inp.state, idx, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
        use_qk_l2norm=True)
    out, pool, inter = mtp_call(inp, idx=idx, l2=True)
    close_out(out, want_out)
    close_state(pool, want_pool)
    close_state(inter, want_inter)


def test_mtp_without_intermediates_t1_matches_decode():
    inp = synthetic.make_inputs(B=3, T=1, seed=52)
    want = gdn_ref.decode(*inp.args())
    out, pool, _ = mtp_call(inp, inter=False)
    close_out(out, want[0])
    close_state(pool, want[1])


@pytest.mark.parametrize("T", [2, 4])
def test_mtp_full_heads_b64_sampled(T):
    """B=64, T in {2, 4} at full head count (the benchmark shape); oracle on 4 entries."""
    inp = synthetic.make_inputs(B=64, T=T, seed=53)
    out, pool, inter = mtp_call(inp)
    sel = torch.tensor([0, 17, 42, 63])
    sub_out, sub_pool, sub_inter = gdn_ref.decode_mtp(
        inp.q[sel], inp.k[sel], inp.v[sel], inp.state[sel], None, inp.A_log, inp.a[sel],
        inp.dt_bias, inp.b[sel], inp.scale)
    s = sel.to(DEV)
    close_out(out[s], sub_out)
    close_state(pool[s], sub_pool)
    close_state(inter[s], sub_inter)


def test_baseline_pool_full_size():
    """The benchmark's pooled configuration at full size: a 1024-slot fp32 pool
    (2 GiB, so slot offsets pass 2^31 bytes), B = 256 entries drawn as a random
    permutation with one -1.  Eight sampled live entries match the oracle, every
    slot no entry reads stays bit-identical, and the -1 entry's output is zero."""
    P, B = 1024, 256
    inp = synthetic.make_inputs(B=B, slots=P, seed=77, device=DEV)
    idx = synthetic.make_pool_indices(B, P, seed=77, n_pad=1, device=DEV)
    idx_l = idx.cpu().long()
    live = [i for i in range(B) if idx_l[i] >= 0]
    pad = [i for i in range(B) if idx_l[i] < 0]
    assert len(pad) == 1 and len(live) == B - 1 and max(idx_l.tolist()) >= 1000
    sample = torch.tensor([live[j] for j in (0, 31, 64, 100, 128, 170, 222, len(live) - 1)])
    sel = sample.to(DEV)
    want_out, want_states = gdn_ref.decode(
        inp.q[sel].cpu(), inp.k[sel].cpu(), inp.v[sel].cpu(), inp.state[idx[sel].long()].cpu(),
        inp.A_log.cpu(), inp.a[sel].cpu(), inp.dt_bias.cpu(), inp.b[sel].cpu(), inp.scale)
    before = inp.state.clone()
    out = torch.full((B, 1, 32, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    gdn_b200.gated_delta_rule_decode_pretranspose(
        inp.q, inp.k, inp.v, None, inp.A_log, inp.a, inp.dt_bias, inp.b, scale=inp.scale,
        output=out, use_qk_l2norm=False, initial_state=inp.state, initial_state_indices=idx,
        bad_index_count=bad)
    torch.cuda.synchronize()
    close_out(out[sel], want_out)
    close_state(inp.state[idx[sel].long()], want_states)
    touched = torch.zeros(P, dtype=torch.bool, device=DEV)
    touched[idx[idx >= 0].long()] = True
    untouched = (~touched).nonzero().flatten()
    assert untouched.numel() == P - (B - 1)
    for chunk in untouched.split(128):
        assert torch.equal(inp.state[chunk], before[chunk])
    assert torch.all(out[pad[0]] == 0)
    assert int(bad.item()) == 0
