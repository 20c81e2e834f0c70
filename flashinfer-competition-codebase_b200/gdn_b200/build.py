"""Build recipe for libgdn_b200.so (sm_100a only).

The library is a plain C-ABI shared object compiled by nvcc straight from
``csrc/*.cu``; it links the CUDA runtime statically, so loading it needs no
CUDA libraries on the loader path and works on a machine without a GPU.
The build output lives in-tree (``gdn_b200/_lib/``) so that a copy of the
repository carries it to the GPU host.

Usage:  python -m gdn_b200.build [--force]
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libgdn_b200.so")

SOURCES = ["gdn_decode.cu", "gdn_prefill_chunked.cu", "gdn_prefill_wy.cu"]
TVM_LIB_PATH = os.path.join(LIB_DIR, "libgdn_b200_tvm.so")
# measurement-only kernels of the benchmark (the state round-trip floor), kept out of
# the decode library
PROBE_LIB_PATH = os.path.join(LIB_DIR, "libgdn_b200_probe.so")
PROBE_SOURCES = ["roofline_probe.cu"]
TVM_SOURCES = ["tvm_ffi_entry.cu", "gdn_decode.cu", "gdn_prefill_chunked.cu", "gdn_prefill_wy.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xptxas", "-v",
    "-shared",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "static",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgdn_b200.so")


def _sources():
    return [os.path.join(SRC_DIR, s) for s in SOURCES]


def _deps():
    return _sources() + [os.path.join(SRC_DIR, "tc_common.cuh"),
                         os.path.join(INCLUDE_DIR, "gdn_b200.h"), os.path.abspath(__file__)]


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(d) > t for d in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libgdn_b200.so if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE_DIR, "-o", tmp, *_sources()]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "nvcc failed (%d):\n%s\n%s" % (proc.returncode, " ".join(cmd), proc.stderr[-8000:])
        )
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def _tvm_ffi_paths():
    """(include dirs, library dir) of the installed tvm_ffi package, or None."""
    try:
        from tvm_ffi import libinfo
    except ImportError:
        return None
    incs = [libinfo.find_include_path(), libinfo.find_dlpack_include_path()]
    return incs, os.path.dirname(libinfo.find_libtvm_ffi())


def build_tvm_ffi(force: bool = False) -> str | None:
    """Compile libgdn_b200_tvm.so: the decode step exported as the TVM-FFI function
    ``kernel_cuda_b200``, the reference's native boundary.  Skipped (None) when
    tvm_ffi is not installed."""
    paths = _tvm_ffi_paths()
    if paths is None:
        return None
    incs, libdir = paths
    deps = [os.path.join(SRC_DIR, s) for s in TVM_SOURCES] + _deps()
    if (not force and os.path.exists(TVM_LIB_PATH)
            and all(os.path.getmtime(d) <= os.path.getmtime(TVM_LIB_PATH) for d in deps)):
        return TVM_LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = TVM_LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE_DIR]
    for inc in incs:
        cmd += ["-I", inc]
    cmd += ["-o", tmp, *[os.path.join(SRC_DIR, s) for s in TVM_SOURCES],
            f"-L{libdir}", "-ltvm_ffi", "-Xlinker", f"-rpath={libdir}"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "nvcc failed (%d):\n%s\n%s" % (proc.returncode, " ".join(cmd), proc.stderr[-8000:])
        )
    os.replace(tmp, TVM_LIB_PATH)
    return TVM_LIB_PATH


def build_probe(force: bool = False) -> str:
    """Compile libgdn_b200_probe.so (benchmark-only kernels) if missing or stale."""
    srcs = [os.path.join(SRC_DIR, s) for s in PROBE_SOURCES]
    deps = srcs + [os.path.abspath(__file__)]
    if (not force and os.path.exists(PROBE_LIB_PATH)
            and all(os.path.getmtime(d) <= os.path.getmtime(PROBE_LIB_PATH) for d in deps)):
        return PROBE_LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = PROBE_LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, *srcs]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "nvcc failed (%d):\n%s\n%s" % (proc.returncode, " ".join(cmd), proc.stderr[-8000:])
        )
    os.replace(tmp, PROBE_LIB_PATH)
    return PROBE_LIB_PATH


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build(force=force, verbose="-v" in sys.argv))
    print(build_tvm_ffi(force=force))
    print(build_probe(force=force))
