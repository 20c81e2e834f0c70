"""Host-side logic of the Python API on the CPU: argument checks (which run
before any library call), the synthetic input recipe and the byte model."""

import math

import pytest
import torch

import gdn_b200
from gdn_b200 import ops, synthetic


def small(B=2, T=1, H=4, HV=8):
    return synthetic.make_inputs(B=B, T=T, H=H, HV=HV, seed=3)


def test_cpu_tensors_are_refused_no_fallback():
    inp = small()
    out = torch.empty(2, 1, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA tensor"):
        gdn_b200.kernel_cuda_b200(*inp.args(), out, inp.state)
    with pytest.raises(ValueError, match="CUDA tensor"):
        gdn_b200.gdn_decode(*inp.args())


def test_shape_and_dtype_checks():
    inp = small()
    with pytest.raises(TypeError, match="state must be torch.float32"):
        ops._check(inp.state.half(), "state", torch.float32)
    with pytest.raises(ValueError, match="head dims"):
        ops._check_step_inputs(inp.q[..., :64], inp.k[..., :64], inp.v, inp.A_log, inp.a,
                               inp.dt_bias, inp.b)
    with pytest.raises(ValueError, match="multiple"):
        ops._check_step_inputs(inp.q[:, :, :3], inp.k[:, :, :3], inp.v, inp.A_log, inp.a,
                               inp.dt_bias, inp.b)
    with pytest.raises(ValueError, match="expected T == 1"):
        t2 = small(T=2)
        ops._check_step_inputs(t2.q, t2.k, t2.v, t2.A_log, t2.a, t2.dt_bias, t2.b, T_expected=1)


def test_pool_argument_rules():
    inp = small()
    args = inp.args()[:8]
    f = gdn_b200.gated_delta_rule_decode_pretranspose
    with pytest.raises(ValueError, match="together"):
        f(*args, initial_state=inp.state)
    with pytest.raises(ValueError, match="pool mode"):
        f(*args, output_state_indices=torch.zeros(2, dtype=torch.int32))
    with pytest.raises(ValueError, match="either state"):
        f(*args[:3], None, *args[4:8])
    with pytest.raises(ValueError, match="shape"):
        ops._index_tensor(torch.zeros(3, dtype=torch.int32), "idx", 2, torch.device("cpu"), 4)
    with pytest.raises(TypeError, match="int32 or int64"):
        ops._index_tensor(torch.zeros(2), "idx", 2, torch.device("cpu"), 4)
    idx = ops._index_tensor(torch.tensor([3, -1]), "idx", 2, torch.device("cpu"), 4)
    assert idx.dtype == torch.int32 and idx.tolist() == [3, -1]


def test_int64_indices_cannot_wrap_onto_a_valid_slot():
    """2**32 + 1 would wrap to slot 1 if narrowed to int32; it must stay out of
    range (>= pool: skipped and counted by the kernel), and a large negative value
    must stay negative (the -1 conventions)."""
    big = torch.tensor([2**32 + 1, -(2**40), 2**31, 3, -1, 7], dtype=torch.int64)
    idx = ops._index_tensor(big, "idx", 6, torch.device("cpu"), 4)
    assert idx.dtype == torch.int32
    assert idx.tolist() == [4, -1, 4, 3, -1, 4]
    same = ops._index_tensor(torch.tensor([0, 3], dtype=torch.int32), "idx", 2,
                             torch.device("cpu"), 4)
    assert same.tolist() == [0, 3]


def test_prefill_offsets_int32_pass_through_int64_clamped(monkeypatch):
    """int32 sequence offsets reach the kernels as they are (the kernels clamp each
    sequence's bounds into [0, total] themselves, so no extra launch is spent); int64
    offsets are clamped into [0, total] before narrowing, so that 2**32 + 3 cannot wrap
    onto token 3.  (The per-tensor check, which refuses CPU tensors, is stubbed: only the
    offsets logic is under test here.)"""
    monkeypatch.setattr(ops, "_check", lambda *a, **k: None)
    x = synthetic.make_prefill_inputs([3, 5])
    args = (x["q"], x["k"], x["v"], x["A_log"], x["a"], x["dt_bias"], x["b"])
    cu32 = torch.tensor([0, 3, 8], dtype=torch.int32)
    total, H, HV, K, V, N, cu, _ = ops._check_prefill_inputs(*args, cu32)
    assert (total, H, HV, N) == (8, 16, 32, 2)
    assert cu.data_ptr() == cu32.data_ptr()            # the caller's tensor, untouched
    cu64 = torch.tensor([-5, 2**32 + 3, 8], dtype=torch.int64)
    *_, cu, _ = ops._check_prefill_inputs(*args, cu64)
    assert cu.dtype == torch.int32 and cu.tolist() == [0, 8, 8]


def test_call_spans_from_overlapping_kernels():
    """A call whose second kernel starts during its first one's tail is timed from the
    first start to the last end (2 + 8 = 10 us summed, 9 us spanned); a dropped record
    leaves no whole calls and gives None; other kernels (the L2 flush) are ignored."""
    from gdn_b200.timing import call_spans_us

    us = 1000
    recs = [("gdn_a", 0, 2 * us), ("flush", 2 * us, 3 * us), ("gdn_b", 1 * us, 9 * us),
            ("gdn_a", 20 * us, 22 * us), ("gdn_b", 21 * us, 25 * us)]
    recs.sort(key=lambda r: r[1])
    assert call_spans_us(recs) == [9.0, 5.0]
    assert call_spans_us(recs[:-1]) is None
    assert call_spans_us([("gdn_x", 0, 3 * us)]) == [3.0]
    assert call_spans_us([("other", 0, 1)]) is None


def test_scale_default():
    assert ops._resolve_scale(None, 128) == 1 / math.sqrt(128)
    assert ops._resolve_scale(0.0, 128) == 1 / math.sqrt(128)
    assert ops._resolve_scale(0.5, 128) == 0.5


def test_synthetic_inputs_are_seeded_and_distributed():
    a = synthetic.make_inputs(B=4, seed=5)
    b = synthetic.make_inputs(B=4, seed=5)
    for x, y in zip(a.args()[:8], b.args()[:8]):
        assert torch.equal(x, y)
    assert a.q.shape == (4, 1, 16, 128) and a.v.shape == (4, 1, 32, 128)
    assert a.state.shape == (4, 32, 128, 128) and a.state.dtype == torch.float32
    assert a.q.dtype == torch.bfloat16 and a.a.shape == (4, 1, 32)
    assert -2.0 <= float(a.A_log.min()) and float(a.A_log.max()) <= 1.0
    assert abs(float(a.state.std()) - 0.1) < 0.01
    assert a.scale == 1 / math.sqrt(128)


def test_pool_indices_are_distinct_with_padding():
    idx = synthetic.make_pool_indices(256, 1024, seed=0, n_pad=1)
    assert idx.dtype == torch.int32 and idx.shape == (256,)
    live = idx[idx >= 0]
    assert (idx == -1).sum() == 1 and len(set(live.tolist())) == 255
    assert int(live.max()) < 1024


def test_byte_model():
    # 131,844 bytes per (batch, v-head) update + 256 bytes of A_log/dt_bias per call
    for B in (1, 8, 256):
        assert synthetic.bytes_per_call(B) == 4_219_008 * B + 256
    assert synthetic.bytes_per_call(256) == 1_080_066_304


def test_registry_mirrors_reference_shape():
    fns = gdn_b200.load_algo_functions()
    assert set(fns) == set(gdn_b200.ALGO_ENTRY_POINTS)
    assert gdn_b200.ALGO_NO_DPS <= set(fns)


def _flashinfer_parameters(name):
    """Parameter names and default expressions of a function in the installed
    flashinfer/gdn_decode.py, read from its source (importing it needs a GPU)."""
    import ast
    import importlib.util

    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        pytest.skip("flashinfer not installed")
    import os

    path = os.path.join(list(spec.submodule_search_locations)[0], "gdn_decode.py")
    if not os.path.exists(path):
        pytest.skip("flashinfer/gdn_decode.py not present")
    tree = ast.parse(open(path).read())
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            args = node.args.posonlyargs + node.args.args
            defaults = [None] * (len(args) - len(node.args.defaults)) + [
                ast.unparse(d) for d in node.args.defaults]
            return [(a.arg, d) for a, d in zip(args, defaults)]
    pytest.skip(f"{name} not found in the installed flashinfer")


@pytest.mark.parametrize("name", ["gated_delta_rule_decode_pretranspose", "gated_delta_rule_mtp"])
def test_flashinfer_entry_points_keep_flashinfer_parameters(name):
    """A caller switching `from flashinfer.gdn_decode import ...` to gdn_b200 passes
    the same positional and keyword arguments: FlashInfer's parameter list
    (names, order, defaults) is a prefix of ours; ours only adds optional ones.
    gated_delta_rule_mtp's disable_state_update defaults to None here (FlashInfer:
    None as well, treated as True with a warning)."""
    import inspect

    theirs = _flashinfer_parameters(name)
    ours = list(inspect.signature(getattr(ops, name)).parameters.values())
    assert [p.name for p in ours[:len(theirs)]] == [n for n, _ in theirs]
    for p, (n, default) in zip(ours, theirs):
        if default is None:
            assert p.default is inspect.Parameter.empty, n
        else:
            assert repr(p.default) == default, (n, p.default, default)
    for p in ours[len(theirs):]:
        assert p.default is not inspect.Parameter.empty, p.name
