"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the contest's workload dataset is not available,
so these stand in for it):

    q, k, v  bf16 ~ N(0, 1)          state  fp32 ~ N(0, 1) * 0.1
    A_log    fp32 ~ U(-2, 1)         a, b   bf16 ~ N(0, 1)
    dt_bias  fp32 ~ N(0, 0.5)        scale  = 1/sqrt(128)

Qwen3-Next head counts by default: 16 q/k heads, 32 v-heads, K = V = 128.
Tensors are drawn in a fixed order from one ``torch.Generator`` so that a
seed pins every value; ``device="cuda"`` draws on the GPU (different values,
same distributions) for sizes where a CPU draw would be slow.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class GdnInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: torch.Tensor
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    scale: float
    state_indices: Optional[torch.Tensor] = None

    def to(self, device) -> "GdnInputs":
        f = lambda t: None if t is None else t.to(device)  # noqa: E731
        return GdnInputs(f(self.q), f(self.k), f(self.v), f(self.state), f(self.A_log), f(self.a),
                         f(self.dt_bias), f(self.b), self.scale, f(self.state_indices))

    def clone(self) -> "GdnInputs":
        f = lambda t: None if t is None else t.clone()  # noqa: E731
        return GdnInputs(f(self.q), f(self.k), f(self.v), f(self.state), f(self.A_log), f(self.a),
                         f(self.dt_bias), f(self.b), self.scale, f(self.state_indices))

    def args(self):
        """Positional arguments of the reference signature (q, k, v, state, A_log, a, dt_bias, b, scale)."""
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias, self.b,
                self.scale)


def make_inputs(B: int, T: int = 1, H: int = 16, HV: int = 32, K: int = 128, V: int = 128,
                seed: int = 0, slots: Optional[int] = None, device="cpu",
                state_std: float = 0.1) -> GdnInputs:
    """Draw one batch of decode inputs; ``slots`` sizes the state (default B)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    S = B if slots is None else slots

    def randn(*shape):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32)

    q = randn(B, T, H, K).to(torch.bfloat16)
    k = randn(B, T, H, K).to(torch.bfloat16)
    v = randn(B, T, HV, V).to(torch.bfloat16)
    state = randn(S, HV, V, K).mul_(state_std)
    A_log = torch.rand(HV, generator=gen, device=device, dtype=torch.float32).mul_(3.0).sub_(2.0)
    a = randn(B, T, HV).to(torch.bfloat16)
    dt_bias = randn(HV).mul_(0.5)
    b = randn(B, T, HV).to(torch.bfloat16)
    return GdnInputs(q, k, v, state, A_log, a, dt_bias, b, 1.0 / math.sqrt(K))


def make_pool_indices(B: int, pool: int, seed: int = 0, n_pad: int = 1,
                      device="cpu") -> torch.Tensor:
    """B distinct slots drawn as a random permutation of the pool; the first
    ``n_pad`` entries (after a seeded shuffle of positions) are set to -1."""
    gen = torch.Generator(device="cpu").manual_seed(seed + 1)
    idx = torch.randperm(pool, generator=gen)[:B].to(torch.int32)
    if n_pad > 0:
        pos = torch.randperm(B, generator=gen)[:n_pad]
        idx[pos] = -1
    return idx.to(device)


def bytes_per_call(B: int, T: int = 1, H: int = 16, HV: int = 32, K: int = 128, V: int = 128,
                   active: Optional[int] = None, intermediates: bool = False,
                   write_final: bool = True, state_elem_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one call: state read once and written once per
    active entry (plus one write per token when intermediates are kept), and
    every input and output element once.  For T=1, an fp32 state and the
    Qwen3-Next shapes this is 4,219,008 * B + 256 bytes (state_elem_bytes=2 for a
    bf16 state)."""
    n = B if active is None else active
    state = HV * V * K * state_elem_bytes
    traffic = n * state * (1 + (1 if write_final else 0) + (T if intermediates else 0))
    qk = 2 * B * T * H * K * 2
    vv = B * T * HV * V * 2
    ab = 2 * B * T * HV * 2
    out = B * T * HV * V * 2
    params = 2 * HV * 4
    return traffic + qk + vv + ab + out + params


def make_prefill_inputs(lengths, H: int = 16, HV: int = 32, seed: int = 0, device="cpu",
                        unit_qk: bool = True, with_state: bool = True) -> dict:
    """Token-major variable-length prefill inputs for sequences of the given lengths:
    q, k [total, H, 128], v [total, HV, 128], a, b [total, HV], state
    [len(lengths), HV, 128, 128] (or None), cu_seqlens int32 [len(lengths) + 1].  The
    distributions are make_inputs'; ``unit_qk`` scales q and k to unit norm, as a
    model's q/k producer does (long sequences of raw N(0, 1) keys make the state grow
    by up to |1 - beta*|k|^2| per token)."""
    total = int(sum(lengths))
    inp = make_inputs(B=1, T=max(total, 1), H=H, HV=HV, seed=seed, slots=len(lengths),
                      device=device)
    q, k, v, a, b = (x[0, :total].contiguous() for x in (inp.q, inp.k, inp.v, inp.a, inp.b))
    if unit_qk:
        q = (q.float() / q.float().norm(dim=-1, keepdim=True)).to(torch.bfloat16)
        k = (k.float() / k.float().norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    offsets = [0]
    for n in lengths:
        offsets.append(offsets[-1] + int(n))
    cu = torch.tensor(offsets, dtype=torch.int32, device=device)
    return dict(q=q, k=k, v=v, state=inp.state if with_state else None, A_log=inp.A_log, a=a,
                dt_bias=inp.dt_bias, b=b, cu_seqlens=cu, scale=inp.scale)


def prefill_bytes(lengths, H: int = 16, HV: int = 32, K: int = 128, V: int = 128,
                  with_state: bool = True) -> int:
    """Algorithmic HBM bytes of one prefill call: each sequence's state read once (when
    given) and written once, every token's q, k, v, a, b read and output written once."""
    total = int(sum(lengths))
    n = len(lengths)
    state = n * HV * V * K * 4 * (2 if with_state else 1)
    per_token = 2 * H * K * 2 + HV * V * 2 + 2 * HV * 2 + HV * V * 2
    return state + total * per_token + 2 * HV * 4
