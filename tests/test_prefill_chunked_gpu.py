"""GPU parity of the chunked tensor-core prefill against the reference's varlen prefill
loop, for both implementations: ``gdn_prefill_chunked`` (one launch: tcgen05 products
with the state in tensor memory, inputs by TMA) and ``gdn_prefill_wy`` (two launches:
all chunks' state-independent products at once into a workspace, then each sequence's
state chain).  References: the reference's varlen prefill loop (golden fixtures from kernel_prefill_reference,
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


@pytest.fixture(params=["chunked", "wy"])
def impl(request):
    return request.param


def run_chunked(d, impl, in_place=False):
    g = {n: (t.to(DEV) if isinstance(t, torch.Tensor) else t) for n, t in d.items()}
    total, HV = g["v"].shape[0], g["v"].shape[1]
    N = g["cu_seqlens"].numel() - 1
    out = torch.full((total, HV, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    ns = g["state"] if in_place else torch.full((N, HV, 128, 128), float("nan"), device=DEV)
    fn = gdn_b200.prefill_chunked if impl == "chunked" else gdn_b200.prefill_wy
    status = fn(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                g["cu_seqlens"], g["scale"], out, ns)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, ns


def check_oracle(d, impl, in_place=False):
    want_o, want_s = gdn_ref.prefill_varlen(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                            d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"])
    out, ns = run_chunked(d, impl, in_place)
    torch.testing.assert_close(out.float().cpu(), want_o.float(), **OUT_TOL)
    torch.testing.assert_close(ns.cpu(), want_s, **STATE_TOL)


@pytest.mark.parametrize("lengths", [[64], [1], [63], [65], [130, 7, 0, 200], [128, 64, 1]])
def test_ragged_sequences_match_oracle(lengths, impl):
    check_oracle(synthetic.make_prefill_inputs(lengths, seed=sum(lengths)), impl)


def test_contest_heads_no_initial_state_and_in_place(impl):
    check_oracle(synthetic.make_prefill_inputs([6, 70], H=4, HV=8, seed=2, with_state=False), impl)
    check_oracle(synthetic.make_prefill_inputs([100], seed=3), impl, in_place=True)


def test_long_sequence_1024_tokens(impl):
    check_oracle(synthetic.make_prefill_inputs([1024], seed=5), impl)


@pytest.mark.parametrize("name", ["prefill_qk4v8_ragged", "prefill_qk4v8_ragged_nostate"])
def test_golden_ragged(name, impl):
    meta, inp, gold = golden_io.load(name)
    d = dict(q=inp.q[0], k=inp.k[0], v=inp.v[0], state=inp.state if meta["initial_state"] else None,
             A_log=inp.A_log, a=inp.a[0], dt_bias=inp.dt_bias, b=inp.b[0],
             cu_seqlens=torch.tensor(meta["cu_seqlens"], dtype=torch.int32), scale=inp.scale)
    out, ns = run_chunked(d, impl)
    torch.testing.assert_close(out.float().cpu(), gold["output"].float(), **OUT_TOL)
    torch.testing.assert_close(ns.cpu(), gold["new_state"], **STATE_TOL)


def test_matches_the_token_loop_on_a_batch_of_prompts(impl):
    """8 prompts of 512 tokens at 16/32 heads: chunked against this library's token loop
    (gdn_prefill_tuned, the register-resident kernel) on the GPU."""
    d = synthetic.make_prefill_inputs([512] * 8, seed=8, device=DEV)
    out, ns = run_chunked(d, impl)
    ref_o = torch.empty_like(out)
    ref_s = torch.empty_like(ns)
    gdn_b200.prefill_tuned(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                           d["b"], d["cu_seqlens"], d["scale"], ref_o, ref_s)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ref_o.float(), **OUT_TOL)
    torch.testing.assert_close(ns, ref_s, **STATE_TOL)


def test_dispatch_of_the_default_entry_matches_the_oracle():
    """gdn_prefill picks the two-launch chunked form for sequences of 256 tokens or more
    on average, the one-launch form from 32 tokens, the token loop below; all agree with
    the oracle."""
    for lengths in ([300, 260], [80, 40], [5, 9, 2]):
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


def test_offsets_outside_the_tokens_are_clamped(impl):
    d = synthetic.make_prefill_inputs([80], seed=7)
    d["cu_seqlens"] = torch.tensor([0, 70, 60, 1000], dtype=torch.int32)
    d["state"] = torch.cat([d["state"]] * 3)
    _, ns = run_chunked(d, impl)
    for s, (t0, t1) in enumerate([(0, 70), (70, 70), (60, 80)]):
        sl = slice(t0, t1)
        _, want_s = gdn_ref.prefill_varlen(d["q"][sl], d["k"][sl], d["v"][sl], d["state"][s:s + 1],
                                           d["A_log"], d["a"][sl], d["dt_bias"], d["b"][sl],
                                           torch.tensor([0, t1 - t0], dtype=torch.int32),
                                           d["scale"])
        torch.testing.assert_close(ns[s].cpu(), want_s[0], **STATE_TOL)
    assert torch.all(ns[1] == 0)


def test_two_launch_form_matches_the_single_launch_form():
    """The two chunked implementations on one batch of ragged prompts (16/32 heads): the
    same products in a different order of launches agree closely."""
    d = synthetic.make_prefill_inputs([700, 64, 3, 129], seed=21, device=DEV)
    o1, s1 = run_chunked(d, "chunked")
    o2, s2 = run_chunked(d, "wy")
    torch.testing.assert_close(o2.float(), o1.float(), atol=4e-3, rtol=4e-3)
    torch.testing.assert_close(s2, s1, atol=2e-4, rtol=2e-4)


def test_overlapping_offsets_stay_inside_the_workspace():
    """Offsets that make sequences overlap (tokens 0-200 and 10-300) may give two chunks
    the same workspace record (their results are then unspecified), but every access
    stays inside the workspace: a guard region after it keeps its pattern."""
    d = synthetic.make_prefill_inputs([300], seed=9, device=DEV)
    d["cu_seqlens"] = torch.tensor([0, 200, 10, 300], dtype=torch.int32, device=DEV)
    d["state"] = torch.cat([d["state"]] * 3)
    N, total, HV = 3, 300, 32
    need = gdn_b200._lib.prefill_workspace_bytes(N, total, HV)
    buf = torch.full((need + 65536,), 0xA5, dtype=torch.uint8, device=DEV)
    out = torch.empty((total, HV, 128), dtype=torch.bfloat16, device=DEV)
    ns = torch.empty((N, HV, 128, 128), device=DEV)
    status = gdn_b200.prefill_wy(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                                 d["dt_bias"], d["b"], d["cu_seqlens"], d["scale"], out, ns,
                                 workspace=buf[:need])
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.all(buf[need:] == 0xA5)
    assert torch.all(ns[1] == 0)


def test_c_entry_allocates_its_workspace_stream_ordered():
    """The C entry gdn_prefill (no workspace argument) allocates the two-launch form's
    workspace with cudaMallocAsync on the call's stream and frees it after the launches:
    two calls in a row agree with the oracle."""
    import ctypes
    from gdn_b200 import _lib
    from gdn_b200.ops import _stream_handle

    d = synthetic.make_prefill_inputs([400, 300], seed=31)
    want_o, want_s = gdn_ref.prefill_varlen(d["q"], d["k"], d["v"], d["state"], d["A_log"],
                                            d["a"], d["dt_bias"], d["b"], d["cu_seqlens"],
                                            d["scale"])
    g = {n: (t.to(DEV) if isinstance(t, torch.Tensor) else t) for n, t in d.items()}
    cu = g["cu_seqlens"].to(torch.int32)
    lib = _lib.load()
    for _ in range(2):
        out = torch.full((700, 32, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        ns = torch.full((2, 32, 128, 128), float("nan"), device=DEV)
        rc = lib.gdn_prefill(g["q"].data_ptr(), g["k"].data_ptr(), g["v"].data_ptr(),
                             g["state"].data_ptr(), g["A_log"].data_ptr(), g["a"].data_ptr(),
                             g["dt_bias"].data_ptr(), g["b"].data_ptr(), cu.data_ptr(),
                             ctypes.c_double(float(g["scale"])), out.data_ptr(), ns.data_ptr(),
                             2, 700, 16, 32, 128, 128, 0, _stream_handle(torch.device(DEV)))
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), want_o.float(), **OUT_TOL)
        torch.testing.assert_close(ns.cpu(), want_s, **STATE_TOL)
