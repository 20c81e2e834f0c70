"""ctypes binding of libgdn_b200.so (the C ABI declared in include/gdn_b200.h).

Loading never falls back to another implementation: if the library is
missing, every entry point raises.  Pointers cross the boundary as integers
(``tensor.data_ptr()``), the stream as the raw ``cudaStream_t`` handle.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_P = ctypes.c_void_p
_I = ctypes.c_int
_D = ctypes.c_double
_U = ctypes.c_uint32
_Z = ctypes.c_size_t

# Every function declared in include/gdn_b200.h with its ctypes signature.
SIGNATURES = {
    "gdn_abi_version": (_I, []),
    "gdn_strerror": (ctypes.c_char_p, [_I]),
    "gdn_decode": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "gdn_decode_pooled": (
        _I,
        [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _D, _P, _I, _I, _I, _I, _I, _I, _P, _P],
    ),
    "gdn_decode_mtp": (
        _I,
        [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _D, _P, _P, _I, _I,
         _I, _I, _I, _I, _I, _I, _I, _P, _P],
    ),
    "gdn_decode_bf16_state": (
        _I,
        [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _D, _P, _P, _I, _I,
         _I, _I, _I, _I, _I, _I, _I, _P, _P],
    ),
    "gdn_decode_tuned": (
        _I,
        [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _D, _P,
         _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_decode_tp": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _P, _P, _U,
         _I, _I, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_decode_tp_chained": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _P, _P, _U,
         _I, _I, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_decode_tp_static": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _P, _U,
         _I, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_decode_gated_norm": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _D, _P, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_prefill": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_prefill_chunked": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    ),
    "gdn_prefill_ws": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _P, _Z, _I, _I, _I, _I, _I, _I, _I,
         _P],
    ),
    "gdn_prefill_workspace_bytes": (_Z, [_I, _I, _I]),
    "gdn_prefill_wy": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _P, _P, _Z, _I, _I, _I, _I, _I, _I,
         _P],
    ),
    "gdn_prefill_tuned": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _D, _P, _P, _I, _I, _I, _I, _I, _I, _I,
         _I, _I, _I, _P],
    ),
    "gdn_interleave_heads": (_I, [_P, _P, _I, _I, _I, _I, _P]),
}

ABI_VERSION = 1

GDN_OK = 0
GDN_ERR_NULL = -1
GDN_ERR_SHAPE = -2
GDN_ERR_ALIGN = -3
GDN_ERR_LAUNCH = -4
GDN_ERR_ALIAS = -5
GDN_ERR_ARG = -6
GDN_ERR_LIMIT = -7


class GdnError(RuntimeError):
    """A libgdn_b200 entry point returned a non-zero status."""

    def __init__(self, func: str, code: int, text: str):
        super().__init__(f"{func}: {text} (code {code})")
        self.func = func
        self.code = code


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once and attach the signatures; raise if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"libgdn_b200.so not found at {path}; build it with "
                "`python -m gdn_b200.build` (needs nvcc) before using gdn_b200"
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.gdn_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"libgdn_b200.so ABI {lib.gdn_abi_version()} != expected {ABI_VERSION}; rebuild it"
            )
        _lib = lib
        return lib


def strerror(code: int) -> str:
    return load().gdn_strerror(code).decode()


def prefill_workspace_bytes(num_seqs: int, total_tokens: int, HV: int) -> int:
    """Workspace bytes of the two-launch chunked prefill (``gdn_prefill_workspace_bytes``)."""
    return int(load().gdn_prefill_workspace_bytes(num_seqs, total_tokens, HV))


def call(name: str, *args) -> None:
    rc = getattr(load(), name)(*args)
    if rc != GDN_OK:
        raise GdnError(name, rc, strerror(rc))
