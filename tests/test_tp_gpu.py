"""Tensor-parallel decode on GPUs: the head-interleave kernel, the single-rank
path, and (with two or more GPUs) NCCL ranks that split the v-heads and
all-gather the outputs, checked against the single-GPU result."""

import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

import ctypes

import gdn_b200
from gdn_b200 import _lib, synthetic

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashinfer-competition-codebase_b200")


@pytest.mark.parametrize("world,rows,hvl", [(2, 3, 16), (4, 256, 8), (8, 5, 4), (1, 7, 32)])
def test_interleave_kernel_matches_permute(world, rows, hvl):
    g = torch.randn(world, rows, hvl, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty(rows, world * hvl, 128, dtype=torch.bfloat16, device="cuda")
    gdn_b200.interleave_heads(g, out)
    want = g.permute(1, 0, 2, 3).reshape(rows, world * hvl, 128)
    assert torch.equal(out, want)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, results, collective="peer", steps=2):
    for p in (PKG, ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from gdn_b200 import synthetic as syn
        from gdn_b200.tp import TPDecode

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        inp = syn.make_inputs(B=12, seed=90)                     # same full inputs on every rank
        tp = TPDecode(H=16, HV=32, max_batch=16, device=dev, collective=collective)
        local = [t.to(dev) for t in tp.shard.shard_inputs(inp.q, inp.k, inp.v, inp.state,
                                                          inp.A_log, inp.a, inp.dt_bias, inp.b)]
        outs = []
        for _ in range(steps):                                   # steps on the local state
            outs.append(tp.step(*local, inp.scale).cpu())
        torch.cuda.synchronize(dev)
        if collective == "peer":
            tp.check()
        results[rank] = ("ok", outs, local[3].cpu(), tp.shard.hv0, tp.shard.hv1)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        results[rank] = ("error", repr(e), traceback.format_exc()[-600:])


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("collective", ["peer", "nccl"])
def test_tp_ranks_match_single_gpu(world, collective):
    """world ranks (one GPU each) split the 16/32 heads; every rank's gathered output
    and own state shard equal the single-GPU result on the same inputs."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    steps = 3
    inp = synthetic.make_inputs(B=12, seed=90)
    g = inp.to("cuda:0")
    want = []
    for _ in range(steps):
        o, state = gdn_b200.gdn_decode(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b,
                                       g.scale)
        want.append(o.cpu())
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        res = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, res, collective, steps))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
        for p in procs:
            if p.is_alive():
                p.kill()
        res = dict(res)
    for r in range(world):
        assert res[r][0] == "ok", res[r]
        _, outs, st, hv0, hv1 = res[r]
        for got, w in zip(outs, want):
            torch.testing.assert_close(got.float(), w.float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(st, state[:, hv0:hv1].cpu(), atol=1e-3, rtol=1e-3)


def _tp_call(g, out_ptrs, sig_ptrs, epoch, status, rank, world, timeout_us=0):
    P = ctypes.c_void_p
    B, _, H, K = g.q.shape
    HV = g.v.shape[2]
    _lib.call("gdn_decode_tp", g.q.data_ptr(), g.k.data_ptr(), g.v.data_ptr(), g.state.data_ptr(),
              g.A_log.data_ptr(), g.a.data_ptr(), g.dt_bias.data_ptr(), g.b.data_ptr(), g.scale,
              (P * world)(*out_ptrs), (P * world)(*sig_ptrs), epoch.data_ptr(),
              status.data_ptr(), timeout_us, rank, world, B, H, HV, K, 128, 0,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B", [1, 5, 64])
def test_fused_step_single_rank_matches_plain_kernel(B):
    """world = 1: scatter to the own buffer and a barrier with itself, over
    several epochs alternating two output buffers."""
    inp = synthetic.make_inputs(B=B, seed=95)
    g, h = inp.to("cuda"), inp.to("cuda")
    outs = [torch.full((B, 1, 32, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
            for _ in range(2)]
    sig = torch.zeros(8, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    for step in range(1, 4):
        out = outs[step & 1]
        _tp_call(g, [out.data_ptr()], [sig.data_ptr()], epoch, status, 0, 1)
        want, _ = gdn_b200.gdn_decode(*h.args())
        torch.cuda.synchronize()
        assert torch.equal(out, want) and torch.equal(g.state, h.state)
    assert int(status.item()) == 0 and int(sig[0].item()) == 3 and int(epoch.item()) == 3


@pytest.mark.parametrize("B", [1, 64])
def test_chained_steps_match_plain_steps(B):
    """world = 1: one gdn_decode_tp, then gdn_decode_tp_chained steps enqueued back to
    back (each decode kernel a programmatic dependent of the previous barrier, loading
    the state that the previous decode wrote) give the plain kernel's results exactly."""
    P = ctypes.c_void_p
    inp = synthetic.make_inputs(B=B, seed=98)
    g, h = inp.to("cuda"), inp.to("cuda")
    outs = [torch.zeros((B, 1, 32, 128), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    sig = torch.zeros(8, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for step in range(4):
        _lib.call("gdn_decode_tp_chained" if step else "gdn_decode_tp",
                  g.q.data_ptr(), g.k.data_ptr(), g.v.data_ptr(), g.state.data_ptr(),
                  g.A_log.data_ptr(), g.a.data_ptr(), g.dt_bias.data_ptr(), g.b.data_ptr(),
                  g.scale, (P * 1)(outs[step & 1].data_ptr()), (P * 1)(sig.data_ptr()),
                  epoch.data_ptr(), status.data_ptr(), 0, 0, 1, B, 16, 32, 128, 128, 0, stream)
    for _ in range(4):                     # the same steps with the plain kernel, afterwards
        want, _ = gdn_b200.gdn_decode(*h.args())
    torch.cuda.synchronize()
    assert torch.equal(outs[1], want) and torch.equal(g.state, h.state)
    assert int(status.item()) == 0 and int(epoch.item()) == 4


def test_fused_step_replays_from_cuda_graphs():
    """world = 1 through TPDecode.capture: the barrier's epoch lives on the device,
    so replayed graphs keep advancing it; outputs alternate between two buffers."""
    import torch.distributed as dist
    from gdn_b200.tp import TPDecode

    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()),
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda:0"))
    try:
        inp = synthetic.make_inputs(B=6, seed=97)
        g, h = inp.to("cuda"), inp.to("cuda")
        tp = TPDecode(H=16, HV=32, max_batch=8, device="cuda", collective="peer")
        steps = tp.capture(*g.args())
        for i in range(5):
            out = steps.replay()
            want, _ = gdn_b200.gdn_decode(*h.args())
            torch.cuda.synchronize()
            assert torch.equal(out, want) and torch.equal(g.state, h.state), i
        assert int(tp._epoch.item()) == 5 and int(tp.status.item()) == 0
        # four steps per graph, replayed twice, after the odd count above
        many = tp.capture(*g.args(), steps=4)
        for i in range(2):
            out = many.replay()
            for _ in range(4):
                want, _ = gdn_b200.gdn_decode(*h.args())
            torch.cuda.synchronize()
            assert torch.equal(out, want) and torch.equal(g.state, h.state), i
        assert int(tp._epoch.item()) == 13 and tp._steps == 13
        # hooks: an input copy from pinned host memory before each step and a copy of
        # each step's output after it, recorded into the same graph (steps unchained)
        q_host = g.q.cpu().pin_memory()
        got = [torch.empty_like(out) for _ in range(3)]
        hooked = tp.capture_sequence([g.args()] * 3,
                                     before=lambda i: g.q.copy_(q_host, non_blocking=True),
                                     after=lambda i, o: got[i].copy_(o))
        hooked.replay()
        wants = []
        for _ in range(3):
            want, _ = gdn_b200.gdn_decode(*h.args())
            wants.append(want.clone())
        torch.cuda.synchronize()
        for i in range(3):
            assert torch.equal(got[i], wants[i]), i
        assert torch.equal(g.state, h.state)
        assert int(tp._epoch.item()) == 16 and tp._steps == 16
        del steps, many, hooked
    finally:
        dist.destroy_process_group()


def test_fused_step_barrier_times_out_without_a_peer():
    """Failure detection without a GPU fault: world = 2 with no second rank, so the
    barrier word of rank 1 is never written.  The kernel gives up after the time
    limit, records it in the status word and returns; the GPU stays usable."""
    inp = synthetic.make_inputs(B=2, H=8, HV=16, seed=96)
    g = inp.to("cuda")
    out0 = torch.zeros((2, 1, 32, 128), dtype=torch.bfloat16, device="cuda")
    out1 = torch.zeros_like(out0)
    sig0 = torch.zeros(8, dtype=torch.int32, device="cuda")
    sig1 = torch.zeros(8, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    _tp_call(g, [out0.data_ptr(), out1.data_ptr()], [sig0.data_ptr(), sig1.data_ptr()],
             epoch, status, 0, 2, timeout_us=20000)
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert int(sig1[0].item()) == 1 and int(sig0[0].item()) == 1 and int(sig0[1].item()) == 0
    # rank 0's 16 heads reached both buffers; rank 1's half is untouched
    assert torch.equal(out0[:, :, :16], out1[:, :, :16]) and torch.all(out0[:, :, 16:] == 0)
    # the context is still healthy
    test_fused_step_single_rank_matches_plain_kernel(1)


def test_tp_world_one_is_the_plain_step():
    import torch.distributed as dist
    from gdn_b200.tp import TPDecode

    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda:0"))
    try:
        inp = synthetic.make_inputs(B=5, seed=91)
        g = inp.to("cuda")
        h = inp.to("cuda")
        tp = TPDecode(H=16, HV=32, max_batch=8, device="cuda")
        out = tp.step(*g.args())
        want, _ = gdn_b200.gdn_decode(*h.args())
        assert torch.equal(out, want) and torch.equal(g.state, h.state)
    finally:
        dist.destroy_process_group()
