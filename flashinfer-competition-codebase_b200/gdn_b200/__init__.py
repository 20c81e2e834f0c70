"""gdn_b200 — Gated DeltaNet decode for NVIDIA B200 (sm_100a).

Host side of the hand-written CUDA decode step in ``csrc/gdn_decode.cu``,
reached through the C ABI of ``libgdn_b200.so`` (``include/gdn_b200.h``).
"""

from ._lib import GdnError, load as load_library  # noqa: F401
from .ops import (  # noqa: F401
    ALGO_ENTRY_POINTS,
    ALGO_NO_DPS,
    decode_bf16_state,
    decode_tuned,
    gated_delta_rule_decode_pretranspose,
    gated_delta_rule_mtp,
    gdn_decode,
    gdn_decode_gated_norm,
    gdn_prefill,
    interleave_heads,
    kernel_prefill_b200,
    prefill_chunked,
    prefill_wy,
    prefill_tuned,
    kernel_cuda_b200,
    load_algo_functions,
)

__all__ = [
    "GdnError",
    "load_library",
    "kernel_cuda_b200",
    "gdn_decode",
    "gdn_decode_gated_norm",
    "gdn_prefill",
    "kernel_prefill_b200",
    "prefill_chunked",
    "prefill_wy",
    "prefill_tuned",
    "gated_delta_rule_decode_pretranspose",
    "gated_delta_rule_mtp",
    "decode_bf16_state",
    "decode_tuned",
    "interleave_heads",
    "ALGO_ENTRY_POINTS",
    "ALGO_NO_DPS",
    "load_algo_functions",
]
