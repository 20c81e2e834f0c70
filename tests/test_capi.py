"""The C-ABI library on the CPU: it loads, exports every function that
include/gdn_b200.h declares, and rejects bad arguments before touching CUDA.

Every call here fails argument validation, which returns before any CUDA API
call, so no GPU is needed (the pointers passed are never dereferenced).
"""

import ctypes
import os
import re

import pytest

from gdn_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "gdn_b200.h")

# a fake, 256-byte aligned address that is never dereferenced (calls fail validation first)
P = 1 << 20


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^GDN_API\s+[\w\s\*]+?\b(gdn_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_bound_functions():
    assert declared_functions() == sorted(_lib.SIGNATURES)


def test_every_declared_symbol_is_exported(gdn_lib):
    for name in declared_functions():
        assert hasattr(gdn_lib, name), name
        assert isinstance(getattr(gdn_lib, name), ctypes._CFuncPtr)


def test_only_declared_symbols_are_exported(gdn_lib):
    out = os.popen(f"nm -D --defined-only {gdn_lib._name}").read()
    exported = sorted(l.split()[-1] for l in out.splitlines() if " T " in l and "gdn_" in l)
    assert exported == declared_functions()


def test_library_has_no_cuda_runtime_dependency(gdn_lib):
    deps = os.popen(f"ldd {gdn_lib._name}").read()
    assert "libcudart" not in deps and "libtorch" not in deps


def test_abi_version_and_errors(gdn_lib):
    assert gdn_lib.gdn_abi_version() == _lib.ABI_VERSION
    codes = (_lib.GDN_OK, _lib.GDN_ERR_NULL, _lib.GDN_ERR_SHAPE, _lib.GDN_ERR_ALIGN,
             _lib.GDN_ERR_LAUNCH, _lib.GDN_ERR_ALIAS, _lib.GDN_ERR_ARG, _lib.GDN_ERR_LIMIT)
    assert codes == (0, -1, -2, -3, -4, -5, -6, -7)
    texts = [_lib.strerror(code) for code in codes]
    assert all(texts) and len(set(texts)) == len(texts)
    assert "unknown" in _lib.strerror(-99)


def test_python_error_codes_match_the_header():
    text = open(HEADER).read()
    defined = {m.group(1): int(m.group(2))
               for m in re.finditer(r"^#define\s+(GDN_(?:OK|ERR_\w+))\s+\(?(-?\d+)\)?", text,
                                    flags=re.M)}
    assert len(defined) == 8
    for name, value in defined.items():
        assert getattr(_lib, name) == value, name


def decode_args(**over):
    a = dict(q=P, k=P, v=P, state=P, A_log=P, a=P, dt_bias=P, b=P, scale=0.0, output=P,
             new_state=P, B=1, H=16, HV=32, K=128, V=128, l2=0, stream=None)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize("over,code", [
    (dict(q=None), _lib.GDN_ERR_NULL),
    (dict(state=None), _lib.GDN_ERR_NULL),
    (dict(output=None), _lib.GDN_ERR_NULL),
    (dict(new_state=None), _lib.GDN_ERR_NULL),
    (dict(K=64), _lib.GDN_ERR_SHAPE),
    (dict(V=256), _lib.GDN_ERR_SHAPE),
    (dict(HV=33), _lib.GDN_ERR_SHAPE),
    (dict(H=0), _lib.GDN_ERR_SHAPE),
    (dict(B=-1), _lib.GDN_ERR_SHAPE),
    (dict(B=1 << 20, HV=32), _lib.GDN_ERR_SHAPE),
    (dict(state=P + 4), _lib.GDN_ERR_ALIGN),
    (dict(new_state=P + 8), _lib.GDN_ERR_ALIGN),
    (dict(q=P + 2), _lib.GDN_ERR_ALIGN),
    (dict(v=P + 1), _lib.GDN_ERR_ALIGN),
    (dict(A_log=P + 2), _lib.GDN_ERR_ALIGN),
    (dict(new_state=P + 1024), _lib.GDN_ERR_ALIAS),
])
def test_decode_rejects_before_launch(gdn_lib, over, code):
    assert gdn_lib.gdn_decode(*decode_args(**over)) == code


def test_pooled_rejects(gdn_lib):
    f = gdn_lib.gdn_decode_pooled
    base = dict(q=P, k=P, v=P, pool=P, pool_size=4, idx=P, oidx=None, A_log=P, a=P, dt_bias=P,
                b=P, scale=0.0, output=P, B=2, H=4, HV=8, K=128, V=128, l2=0, bad=None,
                stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    assert call(idx=None) == _lib.GDN_ERR_NULL
    assert call(pool_size=0) == _lib.GDN_ERR_SHAPE
    assert call(idx=P + 2) == _lib.GDN_ERR_ALIGN
    assert call(bad=P + 1) == _lib.GDN_ERR_ALIGN


def test_mtp_rejects(gdn_lib):
    f = gdn_lib.gdn_decode_mtp
    base = dict(q=P, k=P, v=P, pool=P, pool_size=2, idx=None, A_log=P, a=P, dt_bias=P, b=P,
                scale=0.0, output=P, inter=P, cache_steps=4, disable=0, B=2, T=4, H=4, HV=8,
                K=128, V=128, l2=0, bad=None, stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    assert call(T=0) == _lib.GDN_ERR_SHAPE
    assert call(cache_steps=3) == _lib.GDN_ERR_SHAPE           # intermediates shorter than T
    assert call(pool_size=1) == _lib.GDN_ERR_SHAPE             # no indices: pool must hold B
    assert call(inter=P + 4) == _lib.GDN_ERR_ALIGN
    assert call(v=None) == _lib.GDN_ERR_NULL


def test_tuned_rejects_unknown_shape_without_launch(gdn_lib):
    f = gdn_lib.gdn_decode_tuned
    args = [P, P, P, P, 2, None, P, P, P, P, 0.0, P, 2, 1, 4, 8, 128, 128, 0, 12, 1, 1, None]
    assert f(*args) == _lib.GDN_ERR_SHAPE                       # 12 lanes per row
    args[19] = 8
    args[20] = 3
    assert f(*args) == _lib.GDN_ERR_SHAPE                       # 3 rows per lane


def test_interleave_rejects(gdn_lib):
    f = gdn_lib.gdn_interleave_heads
    assert f(None, P, 2, 4, 8, 128, None) == _lib.GDN_ERR_NULL
    assert f(P, P * 2, 0, 4, 8, 128, None) == _lib.GDN_ERR_SHAPE
    assert f(P, P * 2, 2, 4, 8, 126, None) == _lib.GDN_ERR_SHAPE
    assert f(P + 4, P * 2, 2, 4, 8, 128, None) == _lib.GDN_ERR_ALIGN
    assert f(P, P + 64, 2, 4, 8, 128, None) == _lib.GDN_ERR_ALIAS


def test_tp_rejects(gdn_lib):
    import ctypes
    f = gdn_lib.gdn_decode_tp
    arr = (ctypes.c_void_p * 2)(P, P)
    O = 1 << 30                                   # output buffers, disjoint from the state
    outs = (ctypes.c_void_p * 2)(O, O)
    base = dict(q=P, k=P, v=P, state=P, A_log=P, a=P, dt_bias=P, b=P, scale=0.0, outs=outs,
                sigs=arr, epoch=P, status=P, timeout=0, rank=0, world=2, B=2, H=8,
                HV=16, K=128, V=128, l2=0, stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    assert call(world=9) == _lib.GDN_ERR_ARG
    assert call(rank=2) == _lib.GDN_ERR_ARG
    assert call(epoch=None) == _lib.GDN_ERR_NULL
    assert call(epoch=P + 2) == _lib.GDN_ERR_ALIGN
    assert call(sigs=None) == _lib.GDN_ERR_NULL
    assert call(status=None) == _lib.GDN_ERR_NULL
    assert call(outs=(ctypes.c_void_p * 2)(O, None)) == _lib.GDN_ERR_NULL
    assert call(outs=(ctypes.c_void_p * 2)(O, O + 8)) == _lib.GDN_ERR_ALIGN
    assert call(K=64) == _lib.GDN_ERR_SHAPE
    # this rank's own output buffer is the one validated: bf16 alignment, and no
    # overlap with this rank's state (2 x 8 heads x 64 KiB from P)
    assert call(outs=(ctypes.c_void_p * 2)(O + 1, O)) == _lib.GDN_ERR_ALIGN
    assert call(outs=(ctypes.c_void_p * 2)(None, O)) == _lib.GDN_ERR_NULL
    assert call(outs=(ctypes.c_void_p * 2)(P + 4096, O)) == _lib.GDN_ERR_ALIAS
    assert call(outs=(ctypes.c_void_p * 2)(O, P + 4096), rank=1) == _lib.GDN_ERR_ALIAS


def test_prefill_rejects(gdn_lib):
    f = gdn_lib.gdn_prefill
    base = dict(q=P, k=P, v=P, state=P, A_log=P, a=P, dt_bias=P, b=P, cu=P, scale=0.0,
                out=P, new_state=P, N=2, total=8, H=16, HV=32, K=128, V=128, l2=0, stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    assert call(K=64) == _lib.GDN_ERR_SHAPE
    assert call(HV=24) == _lib.GDN_ERR_SHAPE
    assert call(N=-1) == _lib.GDN_ERR_SHAPE
    assert call(total=-1) == _lib.GDN_ERR_SHAPE
    assert call(N=0, q=None, cu=None, new_state=None) == _lib.GDN_OK   # nothing to do
    assert call(cu=None) == _lib.GDN_ERR_NULL
    assert call(new_state=None) == _lib.GDN_ERR_NULL
    assert call(q=None) == _lib.GDN_ERR_NULL
    assert call(cu=P + 2) == _lib.GDN_ERR_ALIGN
    assert call(new_state=P + 4) == _lib.GDN_ERR_ALIGN
    assert call(new_state=P + 4096) == _lib.GDN_ERR_ALIAS
    args = list(base.values())[:-1]                    # all but the stream
    assert gdn_lib.gdn_prefill_tuned(*args, 8, 3, 1, None) == _lib.GDN_ERR_SHAPE


def test_gated_norm_rejects(gdn_lib):
    f = gdn_lib.gdn_decode_gated_norm
    # valid except for the one field each call changes: every call fails validation
    # (or is the B = 0 no-op) before anything is launched
    args = [P] * 8 + [0.0, P, P, 1e-6, P, 1, 16, 32, 128, 128, 1, None]
    bad_eps = list(args)
    bad_eps[11] = -1.0
    assert f(*bad_eps) == _lib.GDN_ERR_ARG
    no_z = list(args)
    no_z[9] = None
    assert f(*no_z) == _lib.GDN_ERR_NULL
    odd_w = list(args)
    odd_w[10] = P + 1
    assert f(*odd_w) == _lib.GDN_ERR_ALIGN
    zero_b = list(args)
    zero_b[13] = 0
    assert f(*zero_b) == _lib.GDN_OK


def test_prefill_chunked_rejects(gdn_lib):
    f = gdn_lib.gdn_prefill_chunked
    base = dict(q=P, k=P, v=P, state=P, A_log=P, a=P, dt_bias=P, b=P, cu=P, scale=0.0,
                out=P, new_state=P, status=None, N=2, total=8, H=16, HV=32, K=128, V=128,
                stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    assert call(K=64) == _lib.GDN_ERR_SHAPE
    assert call(N=0, q=None, cu=None) == _lib.GDN_OK
    assert call(cu=None) == _lib.GDN_ERR_NULL
    assert call(q=P + 8) == _lib.GDN_ERR_ALIGN        # TMA sources need 16-byte alignment
    assert call(out=P + 2) == _lib.GDN_ERR_ALIGN
    assert call(new_state=P + 4096) == _lib.GDN_ERR_ALIAS


def test_prefill_wy_rejects(gdn_lib):
    f = gdn_lib.gdn_prefill_wy
    need = gdn_lib.gdn_prefill_workspace_bytes(2, 8, 32)
    assert need == (2 + 1) * 32 * 106496          # (N + ceil(total / 64)) x HV records
    assert gdn_lib.gdn_prefill_workspace_bytes(-1, 8, 32) == 0
    assert gdn_lib.gdn_prefill_workspace_bytes(2, 8, 0) == 0
    base = dict(q=P, k=P, v=P, state=P, A_log=P, a=P, dt_bias=P, b=P, cu=P, scale=0.0,
                out=P, new_state=P, status=None, ws=P, ws_bytes=need, N=2, total=8, H=16,
                HV=32, K=128, V=128, stream=None)

    def call(**over):
        d = dict(base)
        d.update(over)
        return f(*d.values())

    # valid except for the one field each call changes: every call fails validation (or
    # is the N = 0 no-op) before anything is launched
    assert call(K=64) == _lib.GDN_ERR_SHAPE
    assert call(N=0, q=None, cu=None, ws=None) == _lib.GDN_OK
    assert call(cu=None) == _lib.GDN_ERR_NULL
    assert call(ws=None) == _lib.GDN_ERR_NULL
    assert call(ws=P + 8) == _lib.GDN_ERR_ALIGN        # bulk copies need 16-byte alignment
    assert call(q=P + 8) == _lib.GDN_ERR_ALIGN
    assert call(ws_bytes=need - 16) == _lib.GDN_ERR_SHAPE
    assert call(new_state=P + 4096) == _lib.GDN_ERR_ALIAS
    g = gdn_lib.gdn_prefill_ws
    args = [P] * 9 + [0.0, P, P, P, need, 2, 8, 16, 32, 64, 128, 0, None]   # K = 64
    assert g(*args) == _lib.GDN_ERR_SHAPE
