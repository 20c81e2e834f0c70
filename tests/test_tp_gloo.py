"""Tensor-parallel host logic on CPU ranks (gloo, world size 2 and 4).

Each rank runs the oracle on its head shard in place of the CUDA step and a
PyTorch permute in place of the interleave kernel; the test checks that the
shard boundaries, the all-gather layout and the head interleave reproduce the
single-rank result exactly, and that a rank that fails before the collective
makes the others fail with an error instead of hanging.
"""

import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashinfer-competition-codebase_b200")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for p in (PKG, ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)


def _oracle_step(q, k, v, state, A_log, a, dt_bias, b, scale, out):
    from oracle import gdn_ref

    o, s = gdn_ref.decode(q, k, v, state, A_log, a, dt_bias, b, scale)
    state.copy_(s)
    out.copy_(o)


def _torch_interleave(gathered, out):
    W, rows, hvl, V = gathered.shape
    out.copy_(gathered.permute(1, 0, 2, 3).reshape(rows, W * hvl, V))


def _worker(rank, world, port, mode, results):
    _setup_paths()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        from gdn_b200 import synthetic
        from gdn_b200.tp import TPDecode
        from oracle import gdn_ref

        inp = synthetic.make_inputs(B=3, H=16, HV=32, seed=77)
        tp = TPDecode(H=16, HV=32, max_batch=4, group=None, device="cpu",
                      local_step=_oracle_step, interleave=_torch_interleave)
        local = tp.shard.shard_inputs(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a,
                                      inp.dt_bias, inp.b)
        if mode == "fail" and rank == world - 1:
            raise RuntimeError("injected failure before the all-gather")
        out = tp.step(*local, inp.scale)
        want_out, want_state = gdn_ref.decode(*inp.args())
        ok = torch.equal(out.float(), want_out.float()) or torch.allclose(
            out.float(), want_out.float(), atol=1e-2, rtol=1e-2)
        st = local[3]
        ok_state = torch.allclose(st, want_state[:, tp.shard.hv0:tp.shard.hv1], atol=1e-5,
                                  rtol=1e-5)
        results[rank] = ("ok", bool(ok), bool(ok_state), tp.shard.hv0, tp.shard.hv1)
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which decides
        results[rank] = ("error", type(e).__name__, str(e)[:200], traceback.format_exc()[-400:])
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        return dict(results)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_decode_matches_single_rank(world):
    res = _run(world, "ok")
    assert sorted(res) == list(range(world))
    bounds = []
    for r in range(world):
        status, ok_out, ok_state, hv0, hv1 = res[r]
        assert status == "ok" and ok_out and ok_state, res[r]
        bounds.append((hv0, hv1))
    assert bounds == [(r * 32 // world, (r + 1) * 32 // world) for r in range(world)]


def test_rank_failure_surfaces_as_error_not_hang():
    res = _run(2, "fail")
    assert res[1][0] == "error" and "injected" in res[1][2]
    # the surviving rank's all-gather ends with an error (peer gone / timeout)
    assert res[0][0] == "error", res[0]


def test_head_shard_rules():
    _setup_paths()
    from gdn_b200.tp import HeadShard

    s = HeadShard(1, 4, 16, 32)
    assert (s.h0, s.h1, s.hv0, s.hv1) == (4, 8, 8, 16)
    # the v-heads of a shard read only the q/k heads of the same shard
    assert all(s.h0 <= hv // 2 < s.h1 for hv in range(s.hv0, s.hv1))
    with pytest.raises(ValueError):
        HeadShard(0, 3, 16, 32)
    with pytest.raises(ValueError):
        HeadShard(2, 2, 16, 32)


def test_captured_steps_follow_the_shared_step_parity():
    """CapturedSteps.replay picks the graph recorded for the output buffer the TP
    object's step count has reached, and advances that count by the steps it ran."""
    _setup_paths()
    from gdn_b200.tp import CapturedSteps

    class FakeGraph:
        def __init__(self, log, name):
            self.log, self.name = log, name

        def replay(self):
            self.log.append(self.name)

    class FakeTP:
        collective = "peer"
        _steps = 0

    log = []
    tp = FakeTP()
    three = CapturedSteps(tp, [FakeGraph(log, "3@even"), FakeGraph(log, "3@odd")],
                          ["out-even", "out-odd"], 3)
    two = CapturedSteps(tp, [FakeGraph(log, "2@even"), FakeGraph(log, "2@odd")],
                        ["o2-even", "o2-odd"], 2)
    assert three.replay() == "out-even" and tp._steps == 3
    assert three.replay() == "out-odd" and tp._steps == 6
    assert two.replay() == "o2-even" and tp._steps == 8      # mixing captures keeps the count
    tp._steps += 1                                              # an eager step in between
    assert two.replay() == "o2-odd" and tp._steps == 11
    assert log == ["3@even", "3@odd", "2@even", "2@odd"]
