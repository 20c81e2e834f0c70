"""TEST INFRASTRUCTURE — CPU oracle for the GDN decode path.  Not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
``--impl reference`` legs use this module, and only as the checker or as the
timed CPU restatement of the reference.  The product path (``gdn_b200``) never
imports it.

It restates, in PyTorch fp32 on the CPU, the reference's oracle
``kernel_pt_reference`` (solution/triton/kernel.py:22-118) and the per-token
loop of ``kernel_prefill_reference`` (solution/triton/prefill_kernel.py:85-183),
without their 4/8-head asserts (kernel.py:63-67) so that it covers the 16/32
heads of the benchmark directly, plus the pool semantics of FlashInfer's fp32
decode (flashinfer/gdn_decode.py:166-195, gdn_kernels/gdn_decode_pretranspose.py:136-160)
and the multi-token semantics of its MTP API (flashinfer/gdn_decode.py:557-616).

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own
``kernel_pt_reference`` and ``kernel_prefill_reference`` (imported from the
reference checkout) on seeded inputs and stores their outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against
them.  ``tests/test_oracle_fla_naive.py`` also checks it against an independent
implementation, flash-linear-attention's naive recurrence (fla 0.5.1,
fla/ops/gated_delta_rule/naive.py), the package the reference's Triton kernel
came from.

Per (batch, v-head) with the state viewed as S[K, V] (transpose of the k-last
storage [V, K]), following kernel.py:73-114:
    g     = exp(-exp(A_log) * softplus(a + dt_bias))        kernel.py:73-74
    beta  = sigmoid(b)                                      kernel.py:75
    old   = g * S                                           kernel.py:101
    old_v = k @ old                                         kernel.py:102
    new_v = beta * v + (1 - beta) * old_v                   kernel.py:103
    S     = old - k^T old_v + k^T new_v                     kernel.py:104-106
    o     = scale * q @ S                                   kernel.py:108
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def resolve_scale(scale, K: int) -> float:
    """kernel.py:69-70: None or 0 selects 1/sqrt(K)."""
    if scale is None or float(scale) == 0.0:
        return 1.0 / math.sqrt(K)
    return float(scale)


def gates(A_log, a, dt_bias, b):
    """(g, beta) in fp32, kernel.py:73-75 (F.softplus keeps its threshold of 20)."""
    x = a.float() + dt_bias.float()
    g = torch.exp(-torch.exp(A_log.float()) * F.softplus(x))
    beta = torch.sigmoid(b.float())
    return g, beta


def l2norm(x: torch.Tensor) -> torch.Tensor:
    """x * rsqrt(sum(x^2) + 1e-6) over the last axis (flashinfer/gdn_kernels/
    gdn_decode_pretranspose.py:253-254); the reference path never normalises."""
    x = x.float()
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + 1e-6)


@torch.no_grad()
def decode_loop(q, k, v, state, A_log, a, dt_bias, b, scale):
    """Per-head Python loop in the reference's own form (kernel.py:57-118), any
    head counts with HV % H == 0.  This is the CPU implementation the
    benchmark's reference arm times.  Returns (output [B,1,HV,V] bf16, new_state)."""
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    assert T == 1
    scale = resolve_scale(scale, K)
    g, beta = gates(A_log, a, dt_bias, b)
    qf = q.squeeze(1).float().repeat_interleave(HV // H, dim=1)
    kf = k.squeeze(1).float().repeat_interleave(HV // H, dim=1)
    vf = v.squeeze(1).float()
    g = g.squeeze(1)
    beta = beta.squeeze(1)
    S_in = state.float() if state is not None else torch.zeros(B, HV, V, K)
    new_state = torch.zeros_like(S_in)
    out = torch.zeros(B, HV, V, dtype=torch.float32)
    for bi in range(B):
        for h in range(HV):
            S = S_in[bi, h].clone().transpose(-1, -2)  # [K, V]
            old = g[bi, h] * S
            old_v = kf[bi, h] @ old
            new_v = beta[bi, h] * vf[bi, h] + (1 - beta[bi, h]) * old_v
            S = old - kf[bi, h].unsqueeze(1) @ old_v.unsqueeze(0) \
                + kf[bi, h].unsqueeze(1) @ new_v.unsqueeze(0)
            out[bi, h] = scale * (qf[bi, h] @ S)
            new_state[bi, h] = S.transpose(-1, -2)
    return out.unsqueeze(1).to(torch.bfloat16), new_state


@torch.no_grad()
def _step_batched(qf, kf, vf, g, beta, S_vk, scale):
    """One token for all (batch, head) pairs at once.  qf/kf/vf [N,HV,K] fp32,
    g/beta [N,HV], S_vk [N,HV,V,K] fp32 (k-last).  Returns (o [N,HV,V], S_vk)."""
    S = S_vk.transpose(-1, -2)                                    # [N,HV,K,V]
    old = g[..., None, None] * S
    old_v = torch.einsum("nhk,nhkv->nhv", kf, old)
    new_v = beta[..., None] * vf + (1 - beta[..., None]) * old_v
    S = old - kf[..., :, None] * old_v[..., None, :] + kf[..., :, None] * new_v[..., None, :]
    o = scale * torch.einsum("nhk,nhkv->nhv", qf, S)
    return o, S.transpose(-1, -2).contiguous()


def _expand_qk(x, HV, use_l2):
    xf = l2norm(x) if use_l2 else x.float()
    return xf.repeat_interleave(HV // x.shape[-2], dim=-2)


@torch.no_grad()
def decode(q, k, v, state, A_log, a, dt_bias, b, scale, use_qk_l2norm: bool = False):
    """Batched restatement of kernel_pt_reference for T=1 (same step order as
    decode_loop, heads batched with einsum).  Returns (output bf16, new_state fp32)."""
    B, T, H, K = q.shape
    HV = v.shape[2]
    assert T == 1
    scale = resolve_scale(scale, K)
    g, beta = gates(A_log, a, dt_bias, b)
    qf = _expand_qk(q[:, 0], HV, use_qk_l2norm)
    kf = _expand_qk(k[:, 0], HV, use_qk_l2norm)
    S = state.float() if state is not None else torch.zeros(B, HV, v.shape[3], K)
    o, S = _step_batched(qf, kf, v[:, 0].float(), g[:, 0], beta[:, 0], S, scale)
    return o.unsqueeze(1).to(torch.bfloat16), S


@torch.no_grad()
def decode_pooled(q, k, v, pool, state_indices, A_log, a, dt_bias, b, scale,
                  output_state_indices: Optional[torch.Tensor] = None,
                  use_qk_l2norm: bool = False):
    """Pool semantics of the fp32 FlashInfer decode (gdn_decode_pretranspose.py:136-160):
    entry i reads slot idx[i]; idx < 0 (or >= pool size) skips it with a zero
    output row; the update is written to out_idx[i] (default idx[i]), a negative
    write index meaning slot 0 and an out-of-range one dropping the write.
    Returns (output [B,1,HV,V] bf16, new_pool)."""
    B = q.shape[0]
    P, HV, V, K = pool.shape
    idx = state_indices.long().tolist()
    oidx = idx if output_state_indices is None else output_state_indices.long().tolist()
    active = [i for i in range(B) if 0 <= idx[i] < P]
    new_pool = pool.clone()
    output = torch.zeros(B, 1, HV, V, dtype=torch.bfloat16)
    if not active:
        return output, new_pool
    sel = torch.tensor(active)
    o, S = decode(q[sel], k[sel], v[sel], pool[torch.tensor([idx[i] for i in active])],
                  A_log, a[sel], dt_bias, b[sel], scale, use_qk_l2norm)
    output[sel] = o
    for j, i in enumerate(active):
        w = oidx[i] if oidx[i] >= 0 else 0
        if w < P:
            new_pool[w] = S[j]
    return output, new_pool


@torch.no_grad()
def decode_mtp(q, k, v, pool, state_indices, A_log, a, dt_bias, b, scale,
               keep_intermediates: bool = True, disable_state_update: bool = False,
               use_qk_l2norm: bool = False):
    """T sequential tokens per entry, the per-token loop of kernel_prefill_reference
    (prefill_kernel.py:162-181) with the MTP API's slots and intermediate states.
    Returns (output [B,T,HV,V] bf16, new_pool, intermediates [B,T,HV,V,K] or None);
    intermediates of skipped entries are zeros."""
    B, T, H, K = q.shape
    P, HV, V, _ = pool.shape
    scale = resolve_scale(scale, K)
    idx = list(range(B)) if state_indices is None else state_indices.long().tolist()
    active = [i for i in range(B) if 0 <= idx[i] < P]
    new_pool = pool.clone()
    output = torch.zeros(B, T, HV, V, dtype=torch.bfloat16)
    inter = torch.zeros(B, T, HV, V, K) if keep_intermediates else None
    if not active:
        return output, new_pool, inter
    sel = torch.tensor(active)
    slots = torch.tensor([idx[i] for i in active])
    g, beta = gates(A_log, a[sel], dt_bias, b[sel])                # [n,T,HV]
    S = pool[slots].float()
    for t in range(T):
        qf = _expand_qk(q[sel, t], HV, use_qk_l2norm)
        kf = _expand_qk(k[sel, t], HV, use_qk_l2norm)
        o, S = _step_batched(qf, kf, v[sel, t].float(), g[:, t], beta[:, t], S, scale)
        output[sel, t] = o.to(torch.bfloat16)
        if inter is not None:
            inter[sel, t] = S
    if not disable_state_update:
        new_pool[slots] = S
    return output, new_pool, inter


@torch.no_grad()
def decode_bf16_state(q, k, v, pool, state_indices, A_log, a, dt_bias, b, scale,
                      output_state_indices: Optional[torch.Tensor] = None,
                      keep_intermediates: bool = False, disable_state_update: bool = False,
                      use_qk_l2norm: bool = False):
    """A state stored in bf16 (FlashInfer's bf16-state backend, flashinfer/gdn_decode.py:255-261):
    the state is widened to fp32, the T tokens run with the fp32 steps of decode_mtp, and
    every state that is stored (intermediates, final) is rounded to bf16 (nearest even).
    Slots follow decode_pooled: a read index < 0 or >= pool size skips the entry with
    zero outputs; the final state goes to output_state_indices[i] (default: the read
    slot), a negative write index meaning slot 0, an out-of-range one dropping it.
    Returns (output [B,T,HV,V] bf16, new_pool bf16, intermediates bf16 or None)."""
    B, T = q.shape[0], q.shape[1]
    P = pool.shape[0]
    idx = list(range(B)) if state_indices is None else state_indices.long().tolist()
    oidx = idx if output_state_indices is None else output_state_indices.long().tolist()
    out, _, inter = decode_mtp(q, k, v, pool.float(), state_indices, A_log, a, dt_bias, b, scale,
                               keep_intermediates=True, disable_state_update=True,
                               use_qk_l2norm=use_qk_l2norm)
    new_pool = pool.clone()
    if not disable_state_update:
        for i in range(B):
            if 0 <= idx[i] < P:
                w = oidx[i] if oidx[i] >= 0 else 0
                if w < P:
                    new_pool[w] = inter[i, T - 1].to(torch.bfloat16)
    return out, new_pool, (inter.to(torch.bfloat16) if keep_intermediates else None)


@torch.no_grad()
def prefill_varlen(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
                   use_qk_l2norm: bool = False):
    """Variable-length prefill, kernel_prefill_reference (prefill_kernel.py:85-183)
    without its 4/8-head asserts: q, k [total, H, K], v [total, HV, V], a, b
    [total, HV], state [num_seqs, HV, V, K] or None (zeros), cu_seqlens
    [num_seqs + 1].  Sequence s runs its tokens cu[s]..cu[s+1]-1 in order from
    state[s] (the decode step of kernel.py:95-114 per token, prefill_kernel.py:162-181).
    A sequence with no tokens gets a zero final state, as the reference's
    zero-initialised new_state (prefill_kernel.py:145-147, :156-157) leaves it.
    Returns (output [total, HV, V] bf16, new_state [num_seqs, HV, V, K] fp32)."""
    total, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    scale = resolve_scale(scale, K)
    cu = [int(x) for x in cu_seqlens.tolist()]
    N = len(cu) - 1
    g, beta = gates(A_log, a, dt_bias, b)                      # [total, HV]
    output = torch.zeros(total, HV, V, dtype=torch.bfloat16)
    new_state = torch.zeros(N, HV, V, K)
    for s in range(N):
        t0, t1 = cu[s], cu[s + 1]
        if t1 <= t0:
            continue
        S = (state[s].float().clone() if state is not None else torch.zeros(HV, V, K))[None]
        for t in range(t0, t1):
            qf = _expand_qk(q[t:t + 1], HV, use_qk_l2norm)
            kf = _expand_qk(k[t:t + 1], HV, use_qk_l2norm)
            o, S = _step_batched(qf, kf, v[t:t + 1].float(), g[t:t + 1], beta[t:t + 1], S, scale)
            output[t] = o[0].to(torch.bfloat16)
        new_state[s] = S[0]
    return output, new_state


@torch.no_grad()
def gated_rmsnorm(o, z, weight, eps: float = 1e-6):
    """The decode layer's gated RMSNorm of the step output, in the order of
    Qwen3-Next's ``Qwen3NextRMSNormGated.forward`` (transformers
    models/qwen3_next/modeling_qwen3_next.py:73-82): o and z bf16 [..., V], weight
    bf16 [V]; fp32 normalisation, rounded to bf16, times the bf16 weight (a bf16
    product), times silu(z) in fp32, rounded to bf16."""
    x = o.float()
    var = x.pow(2).mean(-1, keepdim=True)
    x = x * torch.rsqrt(var + eps)
    x = weight * x.to(torch.bfloat16)
    x = x * F.silu(z.float())
    return x.to(torch.bfloat16)
