"""Tensor-parallel GDN decode: v-heads split across the GPUs of one node.

Every (batch entry, v-head) update is independent, so rank r of W owns a
contiguous block of HV/W v-heads together with the H/W q/k heads they read
(v-head hv reads q/k head hv // (HV/H), so a contiguous split keeps each
pair on one rank), the matching slices of A_log, dt_bias, a and b, and its
own state [B, HV/W, V, K].  The state update needs no communication; the one
exchange is the output, which every rank needs in full ([B, 1, HV, V]).

Two ways to do that exchange:

* ``collective="peer"`` (default on GPUs): the decode kernel of each rank
  stores each output row straight into every rank's output buffer over NVLink
  while the other rows are still being computed, then a one-CTA kernel makes
  the ranks meet at a bounded barrier on signal words (``gdn_decode_tp``).  The buffers are torch symmetric memory with NVLink
  multicast disabled (plain peer pointers only); outputs alternate between two
  buffers by step parity, so a fast rank's next step cannot overwrite rows a slow
  rank is still reading, provided each rank consumes a step's output before it
  enqueues its next step (see ``TPDecode.step``).
* ``collective="nccl"``: the local kernel writes [B, 1, HV/W, V], NCCL
  all-gathers it into a rank-major buffer [W, B, HV/W, V], and the library's
  head-interleave kernel reorders it.  This is the baseline, and the path the
  CPU (gloo) tests exercise with stand-in per-rank steps.

The reference runs on one GPU only; this layer has no counterpart there.  The
head split corresponds to the contest definition itself, which is Qwen3-Next's
16/32 heads split four ways (4 q/k, 8 v-heads per rank).
"""

from __future__ import annotations

import ctypes
import os
from typing import Callable, Optional

import torch
import torch.distributed as dist


class HeadShard:
    """The contiguous head range of one rank."""

    def __init__(self, rank: int, world: int, H: int, HV: int):
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"bad rank {rank} of world {world}")
        if H % world or HV % world:
            raise ValueError(f"H={H} and HV={HV} must both be divisible by the world size {world}")
        self.rank, self.world, self.H, self.HV = rank, world, H, HV
        self.h_local = H // world
        self.hv_local = HV // world
        self.h0, self.h1 = rank * self.h_local, (rank + 1) * self.h_local
        self.hv0, self.hv1 = rank * self.hv_local, (rank + 1) * self.hv_local

    def qk(self, x: torch.Tensor) -> torch.Tensor:
        """[B, T, H, K] -> this rank's [B, T, H/W, K]."""
        return x[:, :, self.h0:self.h1].contiguous()

    def per_vhead(self, x: torch.Tensor) -> torch.Tensor:
        """v [B,T,HV,V] or a/b [B,T,HV] -> this rank's v-heads."""
        return x[:, :, self.hv0:self.hv1].contiguous()

    def params(self, x: torch.Tensor) -> torch.Tensor:
        """A_log / dt_bias [HV] -> [HV/W]."""
        return x[self.hv0:self.hv1].contiguous()

    def state(self, s: torch.Tensor) -> torch.Tensor:
        """[S, HV, V, K] -> [S, HV/W, V, K]."""
        return s[:, self.hv0:self.hv1].contiguous()

    def shard_inputs(self, q, k, v, state, A_log, a, dt_bias, b):
        return (self.qk(q), self.qk(k), self.per_vhead(v), self.state(state), self.params(A_log),
                self.per_vhead(a), self.params(dt_bias), self.per_vhead(b))


def _cuda_local_step(q, k, v, state, A_log, a, dt_bias, b, scale, out):
    from .ops import kernel_cuda_b200

    kernel_cuda_b200(q, k, v, state, A_log, a, dt_bias, b, scale, out, state)


def _cuda_interleave(gathered, out):
    from .ops import interleave_heads

    interleave_heads(gathered, out)


class TPDecode:
    """One decode step per call on this rank's head shard, outputs exchanged.

    Buffers are allocated once for ``max_batch`` entries and reused.  With
    ``collective="nccl"``, ``local_step(q, k, v, state, A_log, a, dt_bias, b,
    scale, out)`` and ``interleave(gathered, out)`` default to the CUDA kernels;
    tests on CPU ranks pass stand-ins.
    """

    def __init__(self, H: int, HV: int, max_batch: int, V: int = 128,
                 group: Optional[dist.ProcessGroup] = None, device=None,
                 local_step: Optional[Callable] = None, interleave: Optional[Callable] = None,
                 collective: Optional[str] = None, timeout_us: int = 1_000_000,
                 chain: bool = True):
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.shard = HeadShard(rank, world, H, HV)
        self.V = V
        self.max_batch = max_batch
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        if collective is None:
            collective = "peer" if (self.device.type == "cuda" and local_step is None) else "nccl"
        if collective not in ("peer", "nccl"):
            raise ValueError(f"collective must be 'peer' or 'nccl', got {collective!r}")
        self.collective = collective
        self.timeout_us = int(timeout_us)
        # captured sequences launch each step after the first as a programmatic
        # dependent of the previous step's barrier (gdn_decode_tp_chained)
        self.chain = bool(chain)
        self._steps = 0              # host count of peer steps: output buffer parity
        n = max_batch * self.shard.hv_local * V
        if collective == "nccl":
            self._local = torch.empty(n, dtype=torch.bfloat16, device=self.device)
            self._gathered = torch.empty(world * n, dtype=torch.bfloat16, device=self.device)
            self.local_step = local_step or _cuda_local_step
            self.interleave = interleave or _cuda_interleave
        else:
            if local_step is not None or interleave is not None:
                raise ValueError("stand-in steps apply to collective='nccl' only")
            self._init_peer()

    # -- peer-memory exchange --------------------------------------------------
    def _init_peer(self):
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem

        W = self.shard.world
        self._out_bytes = self.max_batch * self.shard.HV * self.V * 2
        self._sig_off = 2 * self._out_bytes
        total = self._sig_off + 256
        group = self.group if self.group is not None else dist.group.WORLD
        self._buf = symm_mem.empty(total, dtype=torch.uint8, device=self.device)
        self._buf[self._sig_off:].zero_()
        self._hdl = symm_mem.rendezvous(self._buf, group)
        ptrs = [int(x) for x in self._hdl.buffer_ptrs]
        if len(ptrs) != W:
            raise RuntimeError(f"symmetric memory mapped {len(ptrs)} ranks, expected {W}")
        P = ctypes.c_void_p
        self._peer_out = [(P * W)(*[x + k * self._out_bytes for x in ptrs]) for k in (0, 1)]
        self._peer_sig = (P * W)(*[x + self._sig_off for x in ptrs])
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._epoch = torch.zeros(1, dtype=torch.int32, device=self.device)  # device counter
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def _peer_step(self, q, k, v, state, A_log, a, dt_bias, b, scale, B, events, parity=None,
                   chained=False):
        from . import _lib
        from .ops import _check, _check_step_inputs, _resolve_scale

        Bq, T, Hl, HVl, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b, T_expected=1)
        if Hl != self.shard.h_local or HVl != self.shard.hv_local:
            raise ValueError("inputs are not this rank's head shard")
        _check(state, "state", torch.float32, (B, HVl, V, K), dev)
        if parity is None:
            parity = self._steps & 1
            self._steps += 1
        e0, e1 = events if events is not None else (None, None)
        if e0 is not None:
            e0.record()
        with torch.cuda.device(dev):
            _lib.call(
                "gdn_decode_tp_chained" if chained else "gdn_decode_tp",
                q.data_ptr(), k.data_ptr(), v.data_ptr(), state.data_ptr(),
                A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
                _resolve_scale(scale, K), self._peer_out[parity], self._peer_sig,
                self._epoch.data_ptr(), self.status.data_ptr(), self.timeout_us,
                self.shard.rank, self.shard.world, B, Hl, HVl, K, V, 0,
                torch.cuda.current_stream(dev).cuda_stream)
        if e1 is not None:
            e1.record()
        return self._peer_view(B, parity)

    def _peer_view(self, B, parity):
        start = parity * self._out_bytes
        nbytes = B * self.shard.HV * self.V * 2
        return self._buf[start:start + nbytes].view(torch.bfloat16).view(B, 1, self.shard.HV, self.V)

    @torch.no_grad()
    def capture(self, q, k, v, state, A_log, a, dt_bias, b, scale,
                steps: int = 1) -> "CapturedSteps":
        """Record ``steps`` consecutive steps on these (fixed) input tensors as CUDA
        graphs; see ``capture_sequence``."""
        return self.capture_sequence([(q, k, v, state, A_log, a, dt_bias, b, scale)] * steps)

    @torch.no_grad()
    def capture_sequence(self, step_args, before: Optional[Callable[[int], None]] = None,
                         after: Optional[Callable[[int, torch.Tensor], None]] = None
                         ) -> "CapturedSteps":
        """Record one step per entry of ``step_args`` (tuples of the ``step``
        arguments, e.g. one per model layer with that layer's state) as CUDA graphs.

        Replaying runs the steps on whatever the tensors hold at that time, with no
        host work besides one graph launch (several steps per graph amortise it, as a
        model's decode graph does over its layers).  The peer exchange alternates two
        output buffers, so one graph is recorded per starting buffer and each replay
        picks the one that continues this object's step count (captures and eager
        steps can be mixed).  Every rank must replay the same number of steps.
        Nothing runs while capturing.

        ``before(i)`` and ``after(i, out)``, when given, are called while step i is
        captured, right before it and right after it, on the capturing stream (current
        stream): they record work into the same graph, e.g. staging the step's inputs
        from pinned host memory and reading its output ``out`` back.  ``out`` follows
        the rule of ``step``: work that reads it must be ordered on the capturing
        stream before the next step (a copy there, which a side stream may then read).
        Steps captured with hooks are not chained (the hooks' work sits between one
        step's barrier and the next step)."""
        step_args = list(step_args)
        if not step_args:
            raise ValueError("nothing to capture")
        hooked = before is not None or after is not None
        graphs, outs = [], []
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        for start in (0, 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i, args in enumerate(step_args):
                    parity = (start + i) & 1
                    if before is not None:
                        before(i)
                    if self.collective == "peer":
                        # steps after the first follow the previous step's barrier kernel
                        # directly: their decode kernels start loading state while it waits
                        out = self._peer_step(*args, args[0].shape[0], None, parity=parity,
                                              chained=self.chain and i > 0 and not hooked)
                    else:
                        out = self.step(*args)
                    if after is not None:
                        after(i, out)
            graphs.append(g)
            outs.append(out)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        return CapturedSteps(self, graphs, outs, len(step_args))

    def check(self) -> None:
        """Raise if a cross-rank wait of the peer exchange has timed out (syncs)."""
        if self.collective == "peer" and int(self.status.item()) != 0:
            raise RuntimeError("gdn_decode_tp: a rank did not reach the output barrier in time")

    @torch.no_grad()
    def step(self, q, k, v, state, A_log, a, dt_bias, b, scale, out=None,
             kernel_events=None) -> torch.Tensor:
        """Inputs are this rank's shards (``HeadShard.shard_inputs``); the local
        state is updated in place.  Returns the full output [B, 1, HV, V]: with
        ``collective="peer"`` and ``out=None`` that is a view of an internal
        buffer, valid only until the next step (or replay) is enqueued on this
        rank: consume it first (enqueue the work that reads it on the same stream),
        or pass ``out`` to get a copy.  The two peer buffers alternate, and another
        rank's step after next writes this buffer as soon as this rank's next
        barrier has signalled, so a read enqueued after the next step may race with
        that write.  ``kernel_events`` = (start, end) CUDA events recorded around the
        decode launch (for ``"peer"`` the launch includes the exchange)."""
        B = q.shape[0]
        if B > self.max_batch:
            raise ValueError(f"batch {B} exceeds max_batch {self.max_batch}")
        if self.collective == "peer":
            res = self._peer_step(q, k, v, state, A_log, a, dt_bias, b, scale, B, kernel_events)
            if out is not None:
                out.copy_(res)
                return out
            return res
        W, hvl, V = self.shard.world, self.shard.hv_local, self.V
        if out is None:
            out = torch.empty((B, 1, self.shard.HV, V), dtype=torch.bfloat16, device=self.device)
        e0, e1 = kernel_events if kernel_events is not None else (None, None)
        if W == 1:
            local = out
        else:
            local = self._local[:B * hvl * V].view(B, 1, hvl, V)
        if e0 is not None:
            e0.record()
        self.local_step(q, k, v, state, A_log, a, dt_bias, b, scale, local)
        if e1 is not None:
            e1.record()
        if W == 1:
            return out
        n = B * hvl * V
        gathered = self._gathered[:W * n]
        dist.all_gather_into_tensor(gathered, self._local[:n], group=self.group)
        self.interleave(gathered.view(W, B, hvl, V), out.view(B, self.shard.HV, V))
        return out


class CapturedSteps:
    """Recorded TP steps (see ``TPDecode.capture``)."""

    def __init__(self, tp: TPDecode, graphs, outs, steps: int):
        self.tp, self.graphs, self.outs, self.steps = tp, graphs, outs, steps
        self.count = 0

    def replay(self) -> torch.Tensor:
        """Run the recorded steps once; returns the last step's output
        [B, 1, HV, V], valid only until the next step or replay is enqueued on this
        rank (the same rule as ``TPDecode.step``): consume or copy it before that."""
        i = self.tp._steps & 1
        self.graphs[i].replay()
        self.count += 1
        self.tp._steps += self.steps
        return self.outs[i]
