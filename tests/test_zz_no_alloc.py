"""The allocation-free tensor-parallel step, ``gdn_decode_tp_static``.

Some callers cannot allocate device memory where they run a decode step: a
serving runtime that reserves all of HBM for its own pool at start-up, code that
runs while a CUDA graph is being captured, a plain-C host without an allocator.
``gdn_decode_tp`` needs one piece of scratch besides the caller's inputs,
outputs and signal words — its barrier epoch counter — and this variant keeps
that counter in a fixed array inside the library (64 channels), so the caller
allocates nothing for it.

The GPU test runs one rank (world = 1, so one GPU is enough) through the C ABI
and compares two consecutive calls with those of ``gdn_decode_tp``, which takes
its counter from the caller: the outputs and states must be bit-identical, and
each call must advance both counters by exactly one.  It holds whether it runs alone in a fresh process
or after the other tests: with a single rank the barrier only waits for this
rank's own signal, so whatever the channel's counter already holds, each call
advances it by one.
"""

import ctypes

import pytest
import torch

from gdn_b200 import _lib, synthetic

P = ctypes.c_void_p
CHANNEL = 7


def test_static_variant_rejects_channels_beyond_its_scratch():
    lib = _lib.load()
    f = lib.gdn_decode_tp_static
    one = (P * 1)(1 << 20)
    for channel in (-1, 64, 1000):
        rc = f(1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 0.0, one,
               one, 1 << 20, 0, channel, 0, 1, 1, 16, 32, 128, 128, 0, None)
        assert rc == _lib.GDN_ERR_LIMIT
    assert "0..63" in _lib.strerror(_lib.GDN_ERR_LIMIT)


@pytest.mark.gpu
def test_static_scratch_variant_matches_caller_scratch_entry():
    inp = synthetic.make_inputs(B=5, seed=123)
    a, b = inp.to("cuda"), inp.to("cuda")          # same inputs, separate states
    B, _, H, K = a.q.shape
    HV = a.v.shape[2]
    outs_a = [torch.zeros((B, 1, HV, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    outs_b = [torch.zeros_like(outs_a[0]) for _ in range(2)]
    sig_a = torch.zeros(8, dtype=torch.int32, device="cuda")
    sig_b = torch.zeros(8, dtype=torch.int32, device="cuda")
    epoch_a = torch.zeros(1, dtype=torch.int32, device="cuda")
    status_a = torch.zeros(1, dtype=torch.int32, device="cuda")
    status_b = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    seen = []
    for step in range(2):                          # two calls in a row, alternating buffers
        oa, ob = outs_a[step & 1], outs_b[step & 1]
        _lib.call("gdn_decode_tp", a.q.data_ptr(), a.k.data_ptr(), a.v.data_ptr(),
                  a.state.data_ptr(), a.A_log.data_ptr(), a.a.data_ptr(), a.dt_bias.data_ptr(),
                  a.b.data_ptr(), a.scale, (P * 1)(oa.data_ptr()), (P * 1)(sig_a.data_ptr()),
                  epoch_a.data_ptr(), status_a.data_ptr(), 0, 0, 1, B, H, HV, K, 128, 0, stream)
        _lib.call("gdn_decode_tp_static", b.q.data_ptr(), b.k.data_ptr(), b.v.data_ptr(),
                  b.state.data_ptr(), b.A_log.data_ptr(), b.a.data_ptr(), b.dt_bias.data_ptr(),
                  b.b.data_ptr(), b.scale, (P * 1)(ob.data_ptr()), (P * 1)(sig_b.data_ptr()),
                  status_b.data_ptr(), 0, CHANNEL, 0, 1, B, H, HV, K, 128, 0, stream)
        torch.cuda.synchronize()
        # the same kernel on the same inputs: bit-identical outputs and states (a slip
        # in argument forwarding, e.g. a swapped flag or scale, would show here)
        assert torch.equal(ob, oa)
        assert torch.equal(b.state, a.state)
        seen.append(int(sig_b[0].item()))
        assert int(epoch_a.item()) == step + 1
    assert int(status_a.item()) == 0 and int(status_b.item()) == 0
    assert seen[0] >= 1 and seen[1] == seen[0] + 1   # the channel counter advanced once per call
    assert int(epoch_a.item()) == 2
