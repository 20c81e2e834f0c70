"""PyTorch-facing entry points of the B200 GDN decode path.

Each function validates its tensors on the host, then makes one call into
libgdn_b200.so on the tensors' current CUDA stream.  There is no CPU or
PyTorch fallback: a missing library or a non-CUDA tensor raises.

Entry points and the reference interfaces they stand in for:

* ``kernel_cuda_b200`` — destination-passing decode step, same signature as
  the reference's ``kernel_cuda`` / ``kernel_cuda_v4`` (solution/cuda/binding.py:35-60)
  and ``kernel_fla_recurrent`` (solution/triton/kernel.py:150-197).
* ``gdn_decode`` — value-returning form ``(q, k, v, state, A_log, a, dt_bias, b,
  scale) -> (output, new_state)`` of ``kernel_pt_reference``
  (solution/triton/kernel.py:22-118).  The state is updated in place and
  returned as ``new_state``.
* ``gated_delta_rule_decode_pretranspose`` — FlashInfer's fp32 k-last decode API
  (flashinfer/gdn_decode.py:118), which the reference's ``kernel_fi_baseline``
  calls (solution/triton/kernel.py:124-147), including the state-pool path
  (``initial_state`` + ``initial_state_indices`` + ``output_state_indices``).
* ``gated_delta_rule_mtp`` — FlashInfer's multi-token decode API
  (flashinfer/gdn_decode.py:557) for speculative verification, T >= 1.
* ``gdn_decode_gated_norm`` — the decode step fused with the decode layer's gated
  RMSNorm of its output (Qwen3-Next's layer, transformers
  models/qwen3_next/modeling_qwen3_next.py:73-82, :693-697).
* ``kernel_prefill_b200`` / ``gdn_prefill`` — variable-length prefill, the
  reference's DPS prefill entries (solution/triton/prefill_kernel.py:11-83) and the
  value form of ``kernel_prefill_reference`` (:85-183).
"""

from __future__ import annotations

import math
import warnings
from typing import Optional, Tuple

import torch

from . import _lib

_BF16 = torch.bfloat16
_F32 = torch.float32
HEAD_DIM = 128


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check(t, name: str, dtype: torch.dtype, shape=None, device=None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _resolve_scale(scale, K: int) -> float:
    # solution/triton/kernel.py:69-70: None or 0 selects 1/sqrt(K)
    if scale is None or float(scale) == 0.0:
        return 1.0 / math.sqrt(K)
    return float(scale)


def _index_tensor(idx: torch.Tensor, name: str, B: int, device, pool: int) -> torch.Tensor:
    """Slot indices as the contiguous int32 tensor the kernels read.

    int64 indices are clamped to [-1, pool] on the device before narrowing, so a
    value beyond the int32 range cannot wrap onto a valid slot: anything >= pool
    stays out of range (skipped and counted by the kernel) and anything negative
    stays negative (the -1 conventions).  No host synchronisation."""
    if not isinstance(idx, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if tuple(idx.shape) != (B,):
        raise ValueError(f"{name} must have shape ({B},), got {tuple(idx.shape)}")
    if idx.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"{name} must be int32 or int64, got {idx.dtype}")
    if idx.device != device:
        raise ValueError(f"{name} is on {idx.device}, expected {device}")
    if idx.dtype == torch.int64:
        idx = idx.clamp(min=-1, max=max(int(pool), 0))
    return idx.to(torch.int32).contiguous()


def _check_step_inputs(q, k, v, A_log, a, dt_bias, b, T_expected=None):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be 4-D [B, T, heads, dim]")
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if T_expected is not None and T != T_expected:
        raise ValueError(f"expected T == {T_expected}, got T == {T}")
    if K != HEAD_DIM or V != HEAD_DIM:
        raise ValueError(f"head dims must be K == V == {HEAD_DIM}, got K={K}, V={V}")
    if HV % H != 0:
        raise ValueError(f"num v-heads ({HV}) must be a multiple of num q/k heads ({H})")
    dev = q.device
    _check(q, "q", _BF16, (B, T, H, K), dev)
    _check(k, "k", _BF16, (B, T, H, K), dev)
    _check(v, "v", _BF16, (B, T, HV, V), dev)
    _check(A_log, "A_log", _F32, (HV,), dev)
    _check(dt_bias, "dt_bias", _F32, (HV,), dev)
    _check(a, "a", _BF16, (B, T, HV), dev)
    _check(b, "b", _BF16, (B, T, HV), dev)
    return B, T, H, HV, K, V, dev


@torch.no_grad()
def kernel_cuda_b200(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state,
                     use_qk_l2norm: bool = False) -> None:
    """Destination-passing GDN decode step (T=1) on the B200 kernel.

    Drop-in for the reference's ``kernel_cuda`` (solution/cuda/binding.py:35-41):
    q, k [B,1,H,128] bf16; v [B,1,HV,128] bf16; state [B,HV,128,128] fp32 (k-last);
    A_log, dt_bias [HV] fp32; a, b [B,1,HV] bf16; scale float (None/0 -> 1/sqrt(128));
    output [B,1,HV,128] bf16 and new_state [B,HV,128,128] fp32 are written.
    ``new_state`` may be ``state`` itself (in-place update) or a disjoint buffer.
    """
    B, T, H, HV, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b, T_expected=1)
    _check(state, "state", _F32, (B, HV, V, K), dev)
    _check(new_state, "new_state", _F32, (B, HV, V, K), dev)
    _check(output, "output", _BF16, (B, 1, HV, V), dev)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_decode",
            q.data_ptr(), k.data_ptr(), v.data_ptr(), state.data_ptr(), A_log.data_ptr(),
            a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), _resolve_scale(scale, K),
            output.data_ptr(), new_state.data_ptr(), B, H, HV, K, V, int(bool(use_qk_l2norm)),
            _stream_handle(dev),
        )


@torch.no_grad()
def gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale=None,
               use_qk_l2norm: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Value-returning GDN decode step: ``(output, new_state)``.

    Same arguments and results as ``kernel_pt_reference`` (solution/triton/kernel.py:22-118)
    for any head counts with HV % H == 0.  ``state`` is updated in place and returned
    as ``new_state``; ``state=None`` starts from a zero state (kernel.py:80-83).
    """
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if state is None:
        state = torch.zeros((B, HV, V, K), dtype=_F32, device=q.device)
    output = torch.empty((B, 1, HV, V), dtype=_BF16, device=q.device)
    kernel_cuda_b200(q, k, v, state, A_log, a, dt_bias, b, scale, output, state,
                     use_qk_l2norm=use_qk_l2norm)
    return output, state


@torch.no_grad()
def gated_delta_rule_decode_pretranspose(
    q, k, v, state, A_log, a, dt_bias, b, scale=None, output=None,
    use_qk_l2norm: bool = True, initial_state=None, initial_state_indices=None,
    output_state_indices=None, bad_index_count=None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """FlashInfer-compatible k-last decode (flashinfer/gdn_decode.py:118-261).

    Without a pool, ``state`` [B,HV,V,K] is updated in place.  With
    ``initial_state`` [pool,HV,V,K] and ``initial_state_indices`` [B], entry i
    reads slot ``initial_state_indices[i]`` and writes slot
    ``output_state_indices[i]`` (default: the same slot) of the pool in place.
    A negative read index skips the entry and writes a zero output row; a
    negative write index redirects the write to slot 0.  Out-of-range indices
    are skipped and, if ``bad_index_count`` (an int32 CUDA tensor of one
    element) is given, counted into it.  An fp32 state takes T == 1; a bf16 state
    (``decode_bf16_state``) takes T >= 1, like FlashInfer's bf16-state backend.
    Returns ``(output, state_or_pool)``.
    """
    use_pool = initial_state is not None
    if use_pool != (initial_state_indices is not None):
        raise ValueError("initial_state and initial_state_indices must be provided together")
    if output_state_indices is not None and not use_pool:
        raise ValueError("output_state_indices can only be used with initial_state (pool mode)")
    if not use_pool and state is None:
        raise ValueError("either state or initial_state must be provided")
    st = initial_state if use_pool else state
    if isinstance(st, torch.Tensor) and st.dtype == _BF16:
        # bf16 state: FlashInfer's bf16-state backend (flashinfer/gdn_decode.py:255-261),
        # T = 1 or several tokens
        output = decode_bf16_state(
            q, k, v, st, A_log, a, dt_bias, b, scale=scale, output=output,
            state_indices=initial_state_indices if use_pool else None,
            output_state_indices=output_state_indices, use_qk_l2norm=use_qk_l2norm,
            bad_index_count=bad_index_count)
        return output, st
    B, T, H, HV, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b)
    if T != 1:
        raise ValueError("the fp32-state decode takes T == 1; use gated_delta_rule_mtp for T > 1")
    if output is None:
        output = torch.empty((B, 1, HV, V), dtype=_BF16, device=dev)
    _check(output, "output", _BF16, (B, 1, HV, V), dev)
    if bad_index_count is not None:
        _check(bad_index_count, "bad_index_count", torch.int32, (1,), dev)
    sc = _resolve_scale(scale, K)
    if not use_pool:
        _check(state, "state", _F32, (B, HV, V, K), dev)
        kernel_cuda_b200(q, k, v, state, A_log, a, dt_bias, b, sc, output, state,
                         use_qk_l2norm=use_qk_l2norm)
        return output, state
    pool = initial_state.shape[0] if initial_state.dim() == 4 else -1
    _check(initial_state, "initial_state", _F32, (pool, HV, V, K), dev)
    idx_in = _index_tensor(initial_state_indices, "initial_state_indices", B, dev, pool)
    idx_out = (None if output_state_indices is None else
               _index_tensor(output_state_indices, "output_state_indices", B, dev, pool))
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_decode_pooled",
            q.data_ptr(), k.data_ptr(), v.data_ptr(), initial_state.data_ptr(), pool,
            idx_in.data_ptr(), _ptr(idx_out), A_log.data_ptr(), a.data_ptr(),
            dt_bias.data_ptr(), b.data_ptr(), sc, output.data_ptr(), B, H, HV, K, V,
            int(bool(use_qk_l2norm)), _ptr(bad_index_count), _stream_handle(dev),
        )
    return output, initial_state


@torch.no_grad()
def decode_bf16_state(q, k, v, state_pool, A_log, a, dt_bias, b, scale=None, output=None,
                      state_indices=None, output_state_indices=None,
                      intermediate_states_buffer=None, disable_state_update: bool = False,
                      use_qk_l2norm: bool = False, bad_index_count=None) -> torch.Tensor:
    """Decode with the state stored in bf16, T >= 1 tokens, updated in place.

    ``state_pool`` [pool, HV, V, K] bf16; entry i uses slot ``state_indices[i]``
    (``None``: slot i) and writes ``output_state_indices[i]`` (default: the read
    slot), with the index rules of the pooled fp32 path.  The math is fp32; the
    state is rounded to bf16 when stored.  ``intermediate_states_buffer``
    [>= B, cache_steps >= T, HV, V, K] bf16 receives the state after each token.
    Returns the output [B, T, HV, V] bf16.  C entry: ``gdn_decode_bf16_state``.
    """
    B, T, H, HV, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b)
    pool = state_pool.shape[0] if state_pool.dim() == 4 else -1
    _check(state_pool, "state_pool", _BF16, (pool, HV, V, K), dev)
    idx = None if state_indices is None else _index_tensor(state_indices, "state_indices", B, dev, pool)
    oidx = None
    if output_state_indices is not None:
        if idx is None:
            raise ValueError("output_state_indices needs state_indices")
        oidx = _index_tensor(output_state_indices, "output_state_indices", B, dev, pool)
    if idx is None and pool < B:
        raise ValueError(f"state_pool holds {pool} slots; without indices it needs >= B={B}")
    if output is None:
        output = torch.empty((B, T, HV, V), dtype=_BF16, device=dev)
    _check(output, "output", _BF16, (B, T, HV, V), dev)
    cache_steps = 0
    if intermediate_states_buffer is not None:
        ib = intermediate_states_buffer
        if ib.dim() != 5 or ib.shape[0] < B or ib.shape[1] < T or tuple(ib.shape[2:]) != (HV, V, K):
            raise ValueError(
                f"intermediate_states_buffer must be [>= {B}, >= {T}, {HV}, {V}, {K}], got {tuple(ib.shape)}")
        _check(ib, "intermediate_states_buffer", _BF16, None, dev)
        cache_steps = ib.shape[1]
    if bad_index_count is not None:
        _check(bad_index_count, "bad_index_count", torch.int32, (1,), dev)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_decode_bf16_state", q.data_ptr(), k.data_ptr(), v.data_ptr(),
            state_pool.data_ptr(), pool, _ptr(idx), _ptr(oidx), A_log.data_ptr(), a.data_ptr(),
            dt_bias.data_ptr(), b.data_ptr(), _resolve_scale(scale, K), output.data_ptr(),
            _ptr(intermediate_states_buffer), cache_steps, int(bool(disable_state_update)),
            B, T, H, HV, K, V, int(bool(use_qk_l2norm)), _ptr(bad_index_count),
            _stream_handle(dev))
    return output


_warned_mtp_default = False


@torch.no_grad()
def gated_delta_rule_mtp(
    q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale=None,
    output=None, intermediate_states_buffer=None, disable_state_update: Optional[bool] = None,
    use_qk_l2norm: bool = True, bad_index_count=None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """FlashInfer-compatible multi-token decode (flashinfer/gdn_decode.py:557-616).

    Runs T tokens sequentially per batch entry from slot
    ``initial_state_indices[i]`` of ``initial_state`` [pool,HV,V,K] (``None``
    means slot i).  ``intermediate_states_buffer`` [>=B, cache_steps>=T, HV, V, K]
    receives the state after every token, indexed by batch entry.  The final
    state is written back unless ``disable_state_update`` (``None`` means True,
    FlashInfer 0.6's default, with a one-time warning).
    """
    global _warned_mtp_default
    if disable_state_update is None:
        if not _warned_mtp_default:
            warnings.warn("gated_delta_rule_mtp(): disable_state_update defaults to True; "
                          "pass it explicitly", stacklevel=2)
            _warned_mtp_default = True
        disable_state_update = True
    B, T, H, HV, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b)
    pool = initial_state.shape[0] if initial_state.dim() == 4 else -1
    _check(initial_state, "initial_state", _F32, (pool, HV, V, K), dev)
    idx = None
    if initial_state_indices is not None:
        idx = _index_tensor(initial_state_indices, "initial_state_indices", B, dev, pool)
    elif pool < B:
        raise ValueError(f"initial_state holds {pool} slots; without indices it needs >= B={B}")
    if output is None:
        output = torch.empty((B, T, HV, V), dtype=_BF16, device=dev)
    _check(output, "output", _BF16, (B, T, HV, V), dev)
    cache_steps = 0
    if intermediate_states_buffer is not None:
        ib = intermediate_states_buffer
        if ib.dim() != 5 or ib.shape[0] < B or ib.shape[1] < T or tuple(ib.shape[2:]) != (HV, V, K):
            raise ValueError(
                f"intermediate_states_buffer must be [>= {B}, >= {T}, {HV}, {V}, {K}], got {tuple(ib.shape)}")
        _check(ib, "intermediate_states_buffer", _F32, None, dev)
        cache_steps = ib.shape[1]
    if bad_index_count is not None:
        _check(bad_index_count, "bad_index_count", torch.int32, (1,), dev)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_decode_mtp",
            q.data_ptr(), k.data_ptr(), v.data_ptr(), initial_state.data_ptr(), pool, _ptr(idx),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
            _resolve_scale(scale, K), output.data_ptr(), _ptr(intermediate_states_buffer),
            cache_steps, int(bool(disable_state_update)), B, T, H, HV, K, V,
            int(bool(use_qk_l2norm)), _ptr(bad_index_count), _stream_handle(dev),
        )
    return output, initial_state


@torch.no_grad()
def decode_tuned(q, k, v, state_pool, A_log, a, dt_bias, b, scale, output, state_indices=None,
                 lanes_per_row: int = 0, rows_per_lane: int = 0, warps_per_cta: int = 0,
                 use_qk_l2norm: bool = False) -> None:
    """In-place decode with an explicit launch shape (benchmark sweeps)."""
    B, T, H, HV, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b)
    pool = state_pool.shape[0]
    _check(state_pool, "state_pool", _F32, (pool, HV, V, K), dev)
    _check(output, "output", _BF16, (B, T, HV, V), dev)
    idx = None if state_indices is None else _index_tensor(state_indices, "state_indices", B, dev, pool)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_decode_tuned",
            q.data_ptr(), k.data_ptr(), v.data_ptr(), state_pool.data_ptr(), pool, _ptr(idx),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
            _resolve_scale(scale, K), output.data_ptr(), B, T, H, HV, K, V,
            int(bool(use_qk_l2norm)), lanes_per_row, rows_per_lane, warps_per_cta,
            _stream_handle(dev),
        )


@torch.no_grad()
def interleave_heads(gathered: torch.Tensor, output: torch.Tensor) -> torch.Tensor:
    """[W, rows, HVl, V] bf16 (a rank-major all-gather) -> output [rows, W*HVl, V]."""
    if gathered.dim() != 4:
        raise ValueError("gathered must be [world, rows, heads_per_rank, V]")
    W, rows, hvl, V = gathered.shape
    dev = gathered.device
    _check(gathered, "gathered", _BF16, None, dev)
    _check(output, "output", _BF16, None, dev)
    if output.numel() != gathered.numel() or output.shape[-1] != V:
        raise ValueError("output must hold rows * world * heads_per_rank * V elements")
    with torch.cuda.device(dev):
        _lib.call("gdn_interleave_heads", gathered.data_ptr(), output.data_ptr(), W, rows, hvl, V,
                  _stream_handle(dev))
    return output


@torch.no_grad()
def gdn_decode_gated_norm(q, k, v, state, A_log, a, dt_bias, b, z, norm_weight, scale=None,
                          eps: float = 1e-6, use_qk_l2norm: bool = True,
                          output=None) -> torch.Tensor:
    """Decode step (T=1, ``state`` [B,HV,128,128] fp32 updated in place) fused with the
    decode layer's gated RMSNorm of its output: returns
    ``bf16(bf16(norm_weight * bf16(o * rsqrt(mean(o^2) + eps))) * silu(z))`` per
    (batch entry, v-head), the computation of Qwen3-Next's ``Qwen3NextRMSNormGated``
    (transformers models/qwen3_next/modeling_qwen3_next.py:73-82) applied to the step
    output ``o`` as the layer does before its output projection (:693-697).  z
    [B,1,HV,128] bf16; norm_weight [128] bf16.  The model's decode layer normalises q
    and k in the kernel, hence ``use_qk_l2norm=True`` by default.  C entry:
    ``gdn_decode_gated_norm``."""
    B, T, H, HV, K, V, dev = _check_step_inputs(q, k, v, A_log, a, dt_bias, b, T_expected=1)
    _check(state, "state", _F32, (B, HV, V, K), dev)
    _check(z, "z", _BF16, (B, 1, HV, V), dev)
    _check(norm_weight, "norm_weight", _BF16, (V,), dev)
    if output is None:
        output = torch.empty((B, 1, HV, V), dtype=_BF16, device=dev)
    _check(output, "output", _BF16, (B, 1, HV, V), dev)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_decode_gated_norm", q.data_ptr(), k.data_ptr(), v.data_ptr(), state.data_ptr(),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
            _resolve_scale(scale, K), z.data_ptr(), norm_weight.data_ptr(), float(eps),
            output.data_ptr(), B, H, HV, K, V, int(bool(use_qk_l2norm)), _stream_handle(dev))
    return output


def _check_prefill_inputs(q, k, v, A_log, a, dt_bias, b, cu_seqlens):
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be 3-D [total_tokens, heads, dim]")
    total, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    if K != HEAD_DIM or V != HEAD_DIM:
        raise ValueError(f"head dims must be K == V == {HEAD_DIM}, got K={K}, V={V}")
    if HV % H != 0:
        raise ValueError(f"num v-heads ({HV}) must be a multiple of num q/k heads ({H})")
    dev = q.device
    _check(q, "q", _BF16, (total, H, K), dev)
    _check(k, "k", _BF16, (total, H, K), dev)
    _check(v, "v", _BF16, (total, HV, V), dev)
    _check(A_log, "A_log", _F32, (HV,), dev)
    _check(dt_bias, "dt_bias", _F32, (HV,), dev)
    _check(a, "a", _BF16, (total, HV), dev)
    _check(b, "b", _BF16, (total, HV), dev)
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
        raise ValueError("cu_seqlens must be a 1-D tensor [num_seqs + 1]")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
    if cu_seqlens.device != dev:
        raise ValueError(f"cu_seqlens is on {cu_seqlens.device}, expected {dev}")
    # Every prefill kernel clamps each sequence's bounds into [0, total] itself, so int32
    # offsets go to it as they are (no extra launch); int64 offsets are clamped into the
    # same range before narrowing (no host sync), so that none wraps into a valid one
    if cu_seqlens.dtype == torch.int32:
        cu = cu_seqlens.contiguous()
    else:
        cu = cu_seqlens.clamp(0, total).to(torch.int32).contiguous()
    return total, H, HV, K, V, cu.numel() - 1, cu, dev


@torch.no_grad()
def kernel_prefill_b200(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                        new_state, use_qk_l2norm: bool = False) -> None:
    """Destination-passing variable-length prefill on the B200 kernel.

    Drop-in for the reference's ``kernel_prefill_fla_chunk`` /
    ``kernel_prefill_fi_baseline`` (solution/triton/prefill_kernel.py:11-83) with the
    semantics of ``kernel_prefill_reference`` (:85-183): q, k [total, H, 128] bf16;
    v [total, HV, 128] bf16; state [num_seqs, HV, 128, 128] fp32 or None (zeros);
    a, b [total, HV] bf16; cu_seqlens [num_seqs + 1] int32/int64; output
    [total, HV, 128] bf16 and new_state [num_seqs, HV, 128, 128] fp32 are written
    (``new_state`` may be ``state``).  A sequence with no tokens ends with a zero state.
    """
    total, H, HV, K, V, N, cu, dev = _check_prefill_inputs(q, k, v, A_log, a, dt_bias, b,
                                                            cu_seqlens)
    if state is not None:
        _check(state, "state", _F32, (N, HV, V, K), dev)
    _check(new_state, "new_state", _F32, (N, HV, V, K), dev)
    _check(output, "output", _BF16, (total, HV, V), dev)
    # the two-launch chunked path (sequences of 256+ tokens on average, no q/k L2-norm)
    # takes its workspace from torch's caching allocator; the C entry decides the path
    ws = _prefill_workspace(N, total, HV, dev) if not use_qk_l2norm and total >= 256 * N else None
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_prefill_ws", q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(state),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
            _resolve_scale(scale, K), output.data_ptr(), new_state.data_ptr(), _ptr(ws),
            0 if ws is None else ws.numel(), N, total, H, HV, K, V, int(bool(use_qk_l2norm)),
            _stream_handle(dev))


def _prefill_workspace(N: int, total: int, HV: int, dev) -> Optional[torch.Tensor]:
    nbytes = _lib.prefill_workspace_bytes(N, total, HV)
    return torch.empty(nbytes, dtype=torch.uint8, device=dev) if nbytes > 0 else None


@torch.no_grad()
def gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None,
                use_qk_l2norm: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Value-returning variable-length prefill, ``kernel_prefill_reference``'s form
    (solution/triton/prefill_kernel.py:85-183): returns ``(output, new_state)``; the
    initial ``state`` (or None for zeros) is left unchanged."""
    total, _, HV, K, V, N, _, dev = _check_prefill_inputs(q, k, v, A_log, a, dt_bias, b,
                                                           cu_seqlens)
    output = torch.empty((total, HV, V), dtype=_BF16, device=dev)
    new_state = torch.empty((N, HV, V, K), dtype=_F32, device=dev)
    kernel_prefill_b200(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                        new_state, use_qk_l2norm=use_qk_l2norm)
    return output, new_state


@torch.no_grad()
def prefill_chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                    status=None) -> torch.Tensor:
    """``kernel_prefill_b200`` computed by 64-token chunks on the tensor cores (C entry
    ``gdn_prefill_chunked``).  Returns the int32 status tensor (1 if a wait for the
    tensor cores timed out)."""
    total, H, HV, K, V, N, cu, dev = _check_prefill_inputs(q, k, v, A_log, a, dt_bias, b,
                                                            cu_seqlens)
    if state is not None:
        _check(state, "state", _F32, (N, HV, V, K), dev)
    _check(new_state, "new_state", _F32, (N, HV, V, K), dev)
    _check(output, "output", _BF16, (total, HV, V), dev)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_prefill_chunked", q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(state),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
            _resolve_scale(scale, K), output.data_ptr(), new_state.data_ptr(), status.data_ptr(),
            N, total, H, HV, K, V, _stream_handle(dev))
    return status


@torch.no_grad()
def prefill_wy(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
               status=None, workspace=None) -> torch.Tensor:
    """``kernel_prefill_b200`` computed by 64-token chunks in two launches (C entry
    ``gdn_prefill_wy``): every chunk's state-independent products at once, then each
    sequence's state chain.  ``workspace`` (uint8, at least
    ``gdn_prefill_workspace_bytes`` long) is allocated when None.  Returns the int32
    status tensor (1 if a bounded wait timed out)."""
    total, H, HV, K, V, N, cu, dev = _check_prefill_inputs(q, k, v, A_log, a, dt_bias, b,
                                                            cu_seqlens)
    if state is not None:
        _check(state, "state", _F32, (N, HV, V, K), dev)
    _check(new_state, "new_state", _F32, (N, HV, V, K), dev)
    _check(output, "output", _BF16, (total, HV, V), dev)
    if workspace is None:
        workspace = _prefill_workspace(N, total, HV, dev)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_prefill_wy", q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(state),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
            _resolve_scale(scale, K), output.data_ptr(), new_state.data_ptr(), status.data_ptr(),
            _ptr(workspace), 0 if workspace is None else workspace.numel(), N, total, H, HV, K, V,
            _stream_handle(dev))
    return status


@torch.no_grad()
def prefill_tuned(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                  lanes_per_row: int = 0, rows_per_lane: int = 0, warps_per_cta: int = 0) -> None:
    """``kernel_prefill_b200`` with an explicit work split (benchmark sweeps)."""
    total, H, HV, K, V, N, cu, dev = _check_prefill_inputs(q, k, v, A_log, a, dt_bias, b,
                                                            cu_seqlens)
    with torch.cuda.device(dev):
        _lib.call(
            "gdn_prefill_tuned", q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(state),
            A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(), cu.data_ptr(),
            _resolve_scale(scale, K), output.data_ptr(), new_state.data_ptr(), N, total, H, HV,
            K, V, 0, lanes_per_row, rows_per_lane, warps_per_cta, _stream_handle(dev))


# Algorithm registry in the shape of the reference's scripts/shared.py:19-37.
ALGO_ENTRY_POINTS = {
    "cuda-b200": "gdn_b200.ops::kernel_cuda_b200",
    "b200-value": "gdn_b200.ops::gdn_decode",
    "prefill-b200": "gdn_b200.ops::kernel_prefill_b200",
    "prefill-b200-value": "gdn_b200.ops::gdn_prefill",
}
ALGO_NO_DPS = {"b200-value", "prefill-b200-value"}


def load_algo_functions() -> dict:
    return {"cuda-b200": kernel_cuda_b200, "b200-value": gdn_decode,
            "prefill-b200": kernel_prefill_b200, "prefill-b200-value": gdn_prefill}
