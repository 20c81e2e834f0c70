"""Drop-in replacement for the reference's solution/cuda/binding.py (its
``_get_mod()`` / ``kernel_cuda`` pair, binding.py:19-60), routed through
libgdn_b200.so's C ABI with ctypes.

Copy this file next to the reference's binding.py and register it in
scripts/shared.py (``ALGO_ENTRY_POINTS["cuda-b200"] = "binding_b200.py::kernel_cuda_b200"``).
Same arguments, same in-place convention: ``new_state`` may alias ``state``, as
``kernel_fi_baseline`` arranges with ``set_`` (solution/triton/kernel.py:132-134).
The library is found through GDN_B200_LIB, else on the loader path.
"""

import ctypes
import math
import os

import torch

_lib = ctypes.CDLL(os.environ.get("GDN_B200_LIB", "libgdn_b200.so"))
_P, _I, _D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
_lib.gdn_decode.restype = _I
_lib.gdn_decode.argtypes = [_P] * 8 + [_D, _P, _P] + [_I] * 6 + [_P]
_lib.gdn_strerror.restype = ctypes.c_char_p


@torch.no_grad()
def kernel_cuda_b200(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(q.shape[-1])
    B, _, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    rc = _lib.gdn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), state.data_ptr(),
                         A_log.data_ptr(), a.data_ptr(), dt_bias.data_ptr(), b.data_ptr(),
                         float(scale), output.data_ptr(), new_state.data_ptr(),
                         B, H, HV, K, V, 0, torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(_lib.gdn_strerror(rc).decode())
