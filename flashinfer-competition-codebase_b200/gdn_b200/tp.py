"""Tensor-parallel GDN decode: v-heads split across the GPUs of one node.

Every (batch entry, v-head) update is independent, so rank r of W owns a
contiguous block of HV/W v-heads together with the H/W q/k heads they read
(v-head hv reads q/k head hv // (HV/H), so a contiguous split keeps each
pair on one rank), the matching slices of A_log, dt_bias, a and b, and its
own state [B, HV/W, V, K].  The state update needs no communication.  The
one exchange is the output: each rank's bf16 [B, T, HV/W, V] is all-gathered
over NVLink by NCCL into a rank-major buffer [W, B*T, HV/W, V], which the
library's head-interleave kernel turns into [B, T, HV, V].

The reference runs on one GPU only; this layer has no counterpart there.  The
head split corresponds to the contest definition itself, which is Qwen3-Next's
16/32 heads split four ways (4 q/k, 8 v-heads per rank).

Collectives go through ``torch.distributed`` on the given group (NCCL on
GPUs, gloo in the CPU tests, where the per-rank step and the interleave are
supplied by the test).
"""

from __future__ import annotations

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
    """One decode step per call on this rank's head shard, outputs all-gathered.

    Buffers for the local output and the gathered outputs are allocated once
    for ``max_batch`` entries and reused.  ``local_step(q, k, v, state, A_log,
    a, dt_bias, b, scale, out)`` and ``interleave(gathered, out)`` default to
    the CUDA kernels; tests on CPU ranks pass stand-ins.
    """

    def __init__(self, H: int, HV: int, max_batch: int, V: int = 128,
                 group: Optional[dist.ProcessGroup] = None, device=None,
                 local_step: Optional[Callable] = None, interleave: Optional[Callable] = None):
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.shard = HeadShard(rank, world, H, HV)
        self.V = V
        self.max_batch = max_batch
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        n = max_batch * self.shard.hv_local * V
        self._local = torch.empty(n, dtype=torch.bfloat16, device=self.device)
        self._gathered = torch.empty(world * n, dtype=torch.bfloat16, device=self.device)
        self.local_step = local_step or _cuda_local_step
        self.interleave = interleave or _cuda_interleave

    @torch.no_grad()
    def step(self, q, k, v, state, A_log, a, dt_bias, b, scale, out=None,
             kernel_events=None) -> torch.Tensor:
        """Inputs are this rank's shards (``HeadShard.shard_inputs``); the local
        state is updated in place.  Returns the full output [B, 1, HV, V].
        ``kernel_events`` = (start, end) CUDA events recorded around the local
        decode launch, for timing it apart from the all-gather."""
        B = q.shape[0]
        if B > self.max_batch:
            raise ValueError(f"batch {B} exceeds max_batch {self.max_batch}")
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
