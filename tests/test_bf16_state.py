"""The bf16-state variant: oracle semantics and argument checks on the CPU, parity
of the CUDA path against the oracle on the GPU.

FlashInfer's bf16-state backend (flashinfer/gdn_decode.py:255-261) stores the
recurrent state in bf16 and computes in fp32.  The oracle widens the state,
runs the fp32 steps of the fp32 oracle (itself pinned to the reference's golden
vectors) and rounds every stored state to bf16.  Tolerances on the GPU: outputs
atol = rtol = 1e-2 as elsewhere; bf16 states atol = rtol = 1e-2, i.e. one bf16
rounding step (2^-8 relative) plus an fp32 difference that flips a rounding.
"""


import pytest
import torch

import gdn_b200
from gdn_b200 import _lib, synthetic
from oracle import gdn_ref

OUT_TOL = dict(atol=1e-2, rtol=1e-2)
BF16_STATE_TOL = dict(atol=1e-2, rtol=1e-2)
P = 1 << 20


def bf16_inputs(B, T=1, slots=None, seed=0, H=16, HV=32):
    inp = synthetic.make_inputs(B=B, T=T, H=H, HV=HV, slots=slots, seed=seed)
    inp.state = inp.state.to(torch.bfloat16)
    return inp


# ---- CPU -------------------------------------------------------------------

def test_oracle_t1_is_the_fp32_step_rounded():
    inp = bf16_inputs(B=3, seed=1)
    out, pool, _ = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, None, inp.A_log,
                                             inp.a, inp.dt_bias, inp.b, inp.scale)
    want_out, want_state = gdn_ref.decode(inp.q, inp.k, inp.v, inp.state.float(), inp.A_log,
                                          inp.a, inp.dt_bias, inp.b, inp.scale)
    assert pool.dtype == torch.bfloat16
    torch.testing.assert_close(out.float(), want_out.float(), rtol=2 ** -7, atol=1e-5)
    assert torch.equal(pool, want_state.to(torch.bfloat16))


def test_oracle_slots_padding_and_write_redirect():
    inp = bf16_inputs(B=3, slots=6, seed=2)
    idx = torch.tensor([4, -1, 1], dtype=torch.int32)
    oidx = torch.tensor([5, 2, -1], dtype=torch.int32)
    out, pool, _ = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log,
                                             inp.a, inp.dt_bias, inp.b, inp.scale,
                                             output_state_indices=oidx)
    assert torch.all(out[1].float() == 0)
    for s in (1, 2, 3, 4):                                   # read slots and untouched slots
        assert torch.equal(pool[s], inp.state[s])
    assert not torch.equal(pool[5], inp.state[5]) and not torch.equal(pool[0], inp.state[0])


def test_bf16_entry_rejects_before_launch():
    f = _lib.load().gdn_decode_bf16_state
    base = dict(q=P, k=P, v=P, pool=P, pool_size=4, idx=None, oidx=None, A_log=P, a=P,
                dt_bias=P, b=P, scale=0.0, output=P, inter=None, cache_steps=0, disable=0, B=2,
                T=1, H=16, HV=32, K=128, V=128, l2=0, bad=None, stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    assert call(q=P + 8) == _lib.GDN_ERR_ALIGN           # bf16 q/k chunks are 16 bytes
    assert call(oidx=P) == _lib.GDN_ERR_ARG              # write slots need read slots
    assert call(pool_size=1) == _lib.GDN_ERR_SHAPE       # no indices: pool must hold B
    assert call(inter=P, cache_steps=1, T=2) == _lib.GDN_ERR_SHAPE
    assert call(pool=None) == _lib.GDN_ERR_NULL
    assert call(B=0, q=None) == _lib.GDN_OK              # empty batch: nothing to do


# ---- GPU -------------------------------------------------------------------

def run_gpu(inp, idx=None, oidx=None, T=1, inter=False, disable=False, l2=False):
    g = inp.to("cuda")
    B, HV = g.v.shape[0], g.v.shape[2]
    buf = torch.zeros((B, T, HV, 128, 128), dtype=torch.bfloat16, device="cuda") if inter else None
    out = gdn_b200.decode_bf16_state(
        g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, scale=g.scale,
        state_indices=None if idx is None else idx.to("cuda"),
        output_state_indices=None if oidx is None else oidx.to("cuda"),
        intermediate_states_buffer=buf, disable_state_update=disable, use_qk_l2norm=l2)
    torch.cuda.synchronize()
    return out, g.state, buf


def check(got, want):
    out, pool, inter = got
    w_out, w_pool, w_inter = want
    torch.testing.assert_close(out.float().cpu(), w_out.float(), **OUT_TOL)
    torch.testing.assert_close(pool.float().cpu(), w_pool.float(), **BF16_STATE_TOL)
    if w_inter is not None:
        torch.testing.assert_close(inter.float().cpu(), w_inter.float(), **BF16_STATE_TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 8, 64])
def test_gpu_t1_matches_oracle(B):
    inp = bf16_inputs(B=B, seed=10 + B)
    want = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a,
                                     inp.dt_bias, inp.b, inp.scale)
    check(run_gpu(inp), want)


@pytest.mark.gpu
@pytest.mark.parametrize("l2", [False, True])
def test_gpu_pool_padding_and_output_slots(l2):
    inp = bf16_inputs(B=8, slots=20, seed=30)
    idx = torch.tensor([19, 3, -1, 7, 0, 11, 25, 5], dtype=torch.int32)      # 25: out of range
    oidx = torch.tensor([1, 2, 4, 6, -1, 12, 13, 14], dtype=torch.int32)
    want = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, idx, inp.A_log, inp.a,
                                     inp.dt_bias, inp.b, inp.scale, output_state_indices=oidx,
                                     use_qk_l2norm=l2)
    check(run_gpu(inp, idx=idx, oidx=oidx, l2=l2), want)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [2, 4])
def test_gpu_multi_token_with_intermediates(T):
    inp = bf16_inputs(B=6, T=T, seed=40 + T)
    want = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a,
                                     inp.dt_bias, inp.b, inp.scale, keep_intermediates=True,
                                     use_qk_l2norm=True)
    check(run_gpu(inp, T=T, inter=True, l2=True), want)


@pytest.mark.gpu
def test_gpu_multi_token_disable_state_update_raw_keys():
    inp = bf16_inputs(B=4, T=3, seed=50)
    want = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a,
                                     inp.dt_bias, inp.b, inp.scale, keep_intermediates=True,
                                     disable_state_update=True)
    got = run_gpu(inp, T=3, inter=True, disable=True)
    assert torch.equal(got[1].cpu(), inp.state)
    check(got, want)


@pytest.mark.gpu
def test_gpu_pretranspose_dispatches_on_state_dtype():
    inp = bf16_inputs(B=5, seed=60)
    want = gdn_ref.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, None, inp.A_log, inp.a,
                                     inp.dt_bias, inp.b, inp.scale, use_qk_l2norm=True)
    g = inp.to("cuda")
    out, st = gdn_b200.gated_delta_rule_decode_pretranspose(*g.args())   # FlashInfer default: l2norm
    torch.cuda.synchronize()
    assert st.data_ptr() == g.state.data_ptr() and st.dtype == torch.bfloat16
    check((out, st, None), want)


@pytest.mark.gpu
def test_gpu_full_size_b256_sampled():
    inp = bf16_inputs(B=256, seed=70)
    out, pool, _ = run_gpu(inp)
    sel = torch.tensor([0, 9, 128, 255])
    want = gdn_ref.decode_bf16_state(inp.q[sel], inp.k[sel], inp.v[sel], inp.state[sel], None,
                                     inp.A_log, inp.a[sel], inp.dt_bias, inp.b[sel], inp.scale)
    s = sel.to("cuda")
    check((out[s], pool[s], None), want)
