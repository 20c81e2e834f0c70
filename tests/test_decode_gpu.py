"""GPU parity of the T=1 decode step against the oracle and the reference's
golden vectors, through the C ABI (via the gdn_b200 Python API).

Tolerances (the path's contract): bf16 output within atol = rtol = 1e-2,
fp32 state within atol = rtol = 1e-3.
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


def check(out, state, want_out, want_state):
    torch.testing.assert_close(out.float().cpu(), want_out.float(), **OUT_TOL)
    torch.testing.assert_close(state.cpu(), want_state, **STATE_TOL)


def run_dps(inp, new_state=None, l2=False):
    g = inp.to(DEV)
    B, HV = g.v.shape[0], g.v.shape[2]
    out = torch.full((B, 1, HV, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    dst = g.state if new_state is None else new_state
    gdn_b200.kernel_cuda_b200(*g.args(), out, dst, use_qk_l2norm=l2)
    torch.cuda.synchronize()
    return out, dst, g


@pytest.mark.parametrize("name", ["decode_qk4v8_b1", "decode_qk4v8_b2_edge", "decode_h16hv32_b1"])
def test_golden_decode(name):
    meta, inp, gold = golden_io.load(name)
    out, state, _ = run_dps(inp)
    check(out, state, gold["output"], gold["new_state"])


@pytest.mark.parametrize("B", [1, 2, 8, 33, 64])
def test_batch_sweep_vs_oracle(B):
    inp = synthetic.make_inputs(B=B, seed=100 + B)
    want = gdn_ref.decode(*inp.args())
    out, state, _ = run_dps(inp)
    check(out, state, *want)


def test_value_returning_form_updates_in_place():
    inp = synthetic.make_inputs(B=4, seed=1)
    want = gdn_ref.decode(*inp.args())
    g = inp.to(DEV)
    ptr = g.state.data_ptr()
    out, new_state = gdn_b200.gdn_decode(*g.args())
    assert new_state.data_ptr() == ptr and out.shape == (4, 1, 32, 128)
    check(out, new_state, *want)


def test_disjoint_new_state_leaves_state_untouched():
    inp = synthetic.make_inputs(B=3, seed=2)
    want = gdn_ref.decode(*inp.args())
    dst = torch.full_like(inp.state, float("nan"), device=DEV)
    out, new_state, g = run_dps(inp, new_state=dst)
    check(out, new_state, *want)
    assert torch.equal(g.state.cpu(), inp.state)


def test_zero_initial_state():
    inp = synthetic.make_inputs(B=2, seed=3)
    want = gdn_ref.decode(*inp.args()[:3], None, *inp.args()[4:])
    g = inp.to(DEV)
    out, state = gdn_b200.gdn_decode(g.q, g.k, g.v, None, g.A_log, g.a, g.dt_bias, g.b, g.scale)
    check(out, state, *want)


@pytest.mark.parametrize("heads", [(4, 8), (8, 32), (32, 32), (2, 16)])
def test_head_configurations(heads):
    H, HV = heads
    inp = synthetic.make_inputs(B=3, H=H, HV=HV, seed=H * 100 + HV)
    want = gdn_ref.decode(*inp.args())
    out, state, _ = run_dps(inp)
    check(out, state, *want)


def test_qk_l2norm():
    inp = synthetic.make_inputs(B=5, seed=9)
    want = gdn_ref.decode(*inp.args(), use_qk_l2norm=True)
    out, state, _ = run_dps(inp, l2=True)
    check(out, state, *want)


def test_explicit_scale_and_default_scale():
    inp = synthetic.make_inputs(B=2, seed=4)
    inp.scale = 0.3
    want = gdn_ref.decode(*inp.args())
    out, state, _ = run_dps(inp)
    check(out, state, *want)
    inp.scale = 0.0
    want = gdn_ref.decode(*inp.args())
    out, state, _ = run_dps(inp)
    check(out, state, *want)


def test_empty_batch_is_a_no_op():
    inp = synthetic.make_inputs(B=0, seed=0)
    g = inp.to(DEV)
    out = torch.empty((0, 1, 32, 128), dtype=torch.bfloat16, device=DEV)
    gdn_b200.kernel_cuda_b200(*g.args(), out, g.state)
    torch.cuda.synchronize()


@pytest.mark.parametrize("lpr", [8, 16, 32])
@pytest.mark.parametrize("rg", [1, 2, 4])
@pytest.mark.parametrize("warps", [1, 2, 4, 8])
def test_every_launch_shape(lpr, rg, warps):
    inp = synthetic.make_inputs(B=3, seed=lpr + rg + warps)
    want = gdn_ref.decode(*inp.args())
    g = inp.to(DEV)
    out = torch.empty((3, 1, 32, 128), dtype=torch.bfloat16, device=DEV)
    gdn_b200.decode_tuned(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, g.scale, out,
                          lanes_per_row=lpr, rows_per_lane=rg, warps_per_cta=warps)
    check(out, g.state, *want)


def test_full_size_b256_sampled_heads():
    """BASELINE batch 256 on the device; the oracle checks a sample of 8 entries
    (all 32 heads each) and every output element is finite."""
    torch.manual_seed(0)
    inp = synthetic.make_inputs(B=256, seed=0)
    g = inp.to(DEV)
    out = torch.empty((256, 1, 32, 128), dtype=torch.bfloat16, device=DEV)
    gdn_b200.kernel_cuda_b200(*g.args(), out, g.state)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    sel = torch.tensor([0, 1, 77, 128, 200, 253, 254, 255])
    sub = synthetic.GdnInputs(inp.q[sel], inp.k[sel], inp.v[sel], inp.state[sel], inp.A_log,
                              inp.a[sel], inp.dt_bias, inp.b[sel], inp.scale)
    want = gdn_ref.decode(*sub.args())
    check(out[sel.to(DEV)], g.state[sel.to(DEV)], *want)


@pytest.mark.parametrize("l2", [True, False])
def test_repeated_steps_track_oracle(l2):
    """Several decode steps in a row on the same state (a decode loop).

    With L2-normalised q/k (the model's setting) the state stays bounded and the
    fixed tolerances hold over 8 steps.  With raw N(0,1) keys (|k|^2 ~ 128) each
    step scales the state along k by about |1 - beta |k|^2|, amplifying fp32
    rounding by the same factor, so 3 steps are checked with tolerances scaled
    to the largest state and output magnitude."""
    steps = 8 if l2 else 3
    inp = synthetic.make_inputs(B=4, seed=21)
    g = inp.to(DEV)
    S = inp.state.clone()
    outs, want_outs = [], []
    for step in range(steps):
        nxt = synthetic.make_inputs(B=4, seed=1000 + step)
        o_ref, S = gdn_ref.decode(nxt.q, nxt.k, nxt.v, S, inp.A_log, nxt.a, inp.dt_bias, nxt.b,
                                  inp.scale, use_qk_l2norm=l2)
        gn = nxt.to(DEV)
        out, _ = gdn_b200.gdn_decode(gn.q, gn.k, gn.v, g.state, g.A_log, gn.a, g.dt_bias, gn.b,
                                     g.scale, use_qk_l2norm=l2)
        outs.append(out.float().cpu())
        want_outs.append(o_ref.float())
    if l2:
        for o, w in zip(outs, want_outs):
            torch.testing.assert_close(o, w, **OUT_TOL)
        torch.testing.assert_close(g.state.cpu(), S, **STATE_TOL)
    else:
        for o, w in zip(outs, want_outs):
            torch.testing.assert_close(o, w, rtol=1e-2, atol=1e-2 * float(w.abs().max()))
        torch.testing.assert_close(g.state.cpu(), S, rtol=1e-3, atol=1e-3 * float(S.abs().max()))


def test_bad_arguments_raise_on_gpu():
    inp = synthetic.make_inputs(B=2, seed=5).to(DEV)
    out = torch.empty((2, 1, 32, 128), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        gdn_b200.kernel_cuda_b200(*inp.args(), out[:, :, :16], inp.state)
    with pytest.raises(ValueError, match="contiguous"):
        gdn_b200.kernel_cuda_b200(*inp.args(), out, inp.state.transpose(-1, -2))
    # a state that overlaps new_state without being it is refused by the library
    big = torch.zeros((3, 32, 128, 128), device=DEV)
    with pytest.raises(gdn_b200.GdnError, match="overlap"):
        gdn_b200.kernel_cuda_b200(inp.q, inp.k, inp.v, big[:2], inp.A_log, inp.a, inp.dt_bias,
                                  inp.b, inp.scale, out, big[1:])
