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

import gdn_b200
from gdn_b200 import synthetic

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


def _rank(rank, world, port, results):
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
        tp = TPDecode(H=16, HV=32, max_batch=16, device=dev)
        local = [t.to(dev) for t in tp.shard.shard_inputs(inp.q, inp.k, inp.v, inp.state,
                                                          inp.A_log, inp.a, inp.dt_bias, inp.b)]
        outs = []
        for _ in range(2):                                       # two steps on the local state
            outs.append(tp.step(*local, inp.scale).cpu())
        torch.cuda.synchronize(dev)
        results[rank] = ("ok", outs[0], outs[1], local[3].cpu(), tp.shard.hv0, tp.shard.hv1)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        results[rank] = ("error", repr(e), traceback.format_exc()[-600:])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_two_ranks_match_single_gpu():
    world = 2
    inp = synthetic.make_inputs(B=12, seed=90)
    g = inp.to("cuda:0")
    o1, _ = gdn_b200.gdn_decode(*g.args())
    o2, state2 = gdn_b200.gdn_decode(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, g.scale)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        res = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, res)) for r in range(world)]
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
        _, a, b, st, hv0, hv1 = res[r]
        torch.testing.assert_close(a.float(), o1.float().cpu(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(b.float(), o2.float().cpu(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(st, state2[:, hv0:hv1].cpu(), atol=1e-3, rtol=1e-3)


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
