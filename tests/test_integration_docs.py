"""The bindings a maintainer of the reference adds to route its decode path here,
run against the built library on the CPU.

* A plain C99 caller compiled with gcc against include/gdn_b200.h (warnings as
  errors), linked with libgdn_b200.so and run: the header is C, the library
  loads with no CUDA library on the loader path, and argument errors come back
  as codes before any CUDA call.
* The ctypes binding a maintainer copies next to the reference's
  solution/cuda/binding.py (integration/binding_b200.py, the replacement for
  its kernel_cuda), imported as is with the library path in GDN_B200_LIB: its
  argtypes agree with the header, and a bad shape raises with the library's
  own message.

Every call here fails validation or is a B = 0 no-op, so no GPU is needed.
"""

import importlib.util
import os
import shutil
import subprocess
import types

import pytest
import torch

from gdn_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
BINDING = os.path.join(ROOT, "flashinfer-competition-codebase_b200", "integration",
                       "binding_b200.py")

C_CALLER = r"""
#include <stdio.h>
#include <string.h>
#include "gdn_b200.h"

int main(void) {
  /* 256-byte aligned fake addresses: never dereferenced, every call fails
     validation (or is the B = 0 no-op) before touching the GPU */
  gdn_bf16* bf = (gdn_bf16*)(uintptr_t)(1u << 20);
  float* f32 = (float*)(uintptr_t)(1u << 21);
  int rc;
  if (gdn_abi_version() != GDN_ABI_VERSION) return 1;
  rc = gdn_decode(bf, bf, bf, f32, f32, bf, f32, bf, 0.0, bf, f32, 1, 16, 32, 64, 128, 0, NULL);
  if (rc != GDN_ERR_SHAPE) return 2;
  if (strstr(gdn_strerror(rc), "128") == NULL) return 3;
  rc = gdn_decode(NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 0.0, NULL, NULL,
                  0, 16, 32, 128, 128, 0, NULL);
  if (rc != GDN_OK) return 4;
  rc = gdn_decode(bf, bf, bf, f32, f32, bf, f32, bf, 0.0, bf, f32 + 1, 1, 16, 32, 128, 128, 0,
                  NULL);
  if (rc != GDN_ERR_ALIGN) return 5;
  rc = gdn_interleave_heads(NULL, bf, 2, 4, 8, 128, NULL);
  if (rc != GDN_ERR_NULL) return 6;
  printf("%s\n", gdn_strerror(GDN_OK));
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not installed")
def test_plain_c_caller_compiles_links_and_runs(gdn_lib, tmp_path):
    src = tmp_path / "caller.c"
    exe = tmp_path / "caller"
    src.write_text(C_CALLER)
    libdir = os.path.dirname(gdn_lib._name)
    libname = os.path.basename(gdn_lib._name)
    assert libname.startswith("lib") and libname.endswith(".so")
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{INCLUDE}",
           str(src), "-o", str(exe), f"-L{libdir}", f"-l{libname[3:-3]}",
           f"-Wl,-rpath,{libdir}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    env = {k: v for k, v in os.environ.items() if k != "LD_LIBRARY_PATH"}
    run = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=60)
    assert run.returncode == 0, (run.returncode, run.stderr)
    assert run.stdout.strip() == "ok"


def _load_binding(lib_path, monkeypatch):
    monkeypatch.setenv("GDN_B200_LIB", lib_path)
    spec = importlib.util.spec_from_file_location("binding_b200", BINDING)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_integration_ctypes_binding_matches_the_header(gdn_lib, monkeypatch):
    binding = _load_binding(gdn_lib._name, monkeypatch)
    stub_lib = binding._lib
    restype, argtypes = _lib.SIGNATURES["gdn_decode"]
    assert stub_lib.gdn_decode.restype is restype
    assert list(stub_lib.gdn_decode.argtypes) == argtypes

    # a bad head dimension is rejected by the library before any CUDA call, and the
    # stub raises with the library's message (the stream handle is never used)
    monkeypatch.setattr(torch.cuda, "current_stream",
                        lambda *a, **k: types.SimpleNamespace(cuda_stream=0))
    B, H, HV, K, V = 1, 16, 32, 64, 128
    bf = torch.bfloat16
    q = torch.zeros(B, 1, H, K, dtype=bf)
    k = torch.zeros(B, 1, H, K, dtype=bf)
    v = torch.zeros(B, 1, HV, V, dtype=bf)
    state = torch.zeros(B, HV, V, K)
    A_log, dt_bias = torch.zeros(HV), torch.zeros(HV)
    a = torch.zeros(B, 1, HV, dtype=bf)
    b = torch.zeros(B, 1, HV, dtype=bf)
    out = torch.empty(B, 1, HV, V, dtype=bf)
    with pytest.raises(RuntimeError, match="K and V must be 128"):
        binding.kernel_cuda_b200(q, k, v, state, A_log, a, dt_bias, b, None, out, state)
