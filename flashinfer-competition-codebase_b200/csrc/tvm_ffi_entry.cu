// tvm_ffi_entry.cu — the decode step behind the reference's own native boundary.
//
// The reference exposes its CUDA kernels through TVM-FFI typed functions taking
// TensorViews (solution/cuda/kernel.cu:216-254 `kernel_cuda`, :405-443
// `kernel_cuda_v4`), which flashinfer-bench's TVMFFIBuilder compiles and calls
// in destination-passing style.  This file exports `kernel_cuda_b200` with that
// exact signature, so a Solution whose entry point names it runs the B200
// kernel unchanged.  Unlike the reference export it validates what it is
// given (dtypes, ranks, contiguity) and raises instead of launching on error.
//
// Built as libgdn_b200_tvm.so together with gdn_decode.cu (one module, no
// dependency on libgdn_b200.so); needs the tvm_ffi headers and libtvm_ffi.

#include <dlpack/dlpack.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include "gdn_b200.h"

namespace {

using tvm::ffi::TensorView;

void* base_ptr(const TensorView& t) {
  return static_cast<char*>(t.data_ptr()) + t.byte_offset();
}

void expect(const TensorView& t, const char* name, uint8_t code, int bits, int ndim) {
  const DLDataType dt = t.dtype();
  if (dt.code != code || dt.bits != bits || dt.lanes != 1) {
    TVM_FFI_THROW(TypeError) << name << ": expected " << (code == kDLFloat ? "float" : "bfloat")
                             << bits;
  }
  if (t.ndim() != ndim) TVM_FFI_THROW(ValueError) << name << ": expected rank " << ndim;
  if (!t.IsContiguous()) TVM_FFI_THROW(ValueError) << name << ": must be contiguous";
  if (t.device().device_type != kDLCUDA) TVM_FFI_THROW(ValueError) << name << ": must be on CUDA";
}

void KernelCudaB200(TensorView q, TensorView k, TensorView v, TensorView state, TensorView A_log,
                    TensorView a, TensorView dt_bias, TensorView b_gate, double scale,
                    TensorView output, TensorView new_state) {
  expect(q, "q", kDLBfloat, 16, 4);
  expect(k, "k", kDLBfloat, 16, 4);
  expect(v, "v", kDLBfloat, 16, 4);
  expect(state, "state", kDLFloat, 32, 4);
  expect(A_log, "A_log", kDLFloat, 32, 1);
  expect(a, "a", kDLBfloat, 16, 3);
  expect(dt_bias, "dt_bias", kDLFloat, 32, 1);
  expect(b_gate, "b", kDLBfloat, 16, 3);
  expect(output, "output", kDLBfloat, 16, 4);
  expect(new_state, "new_state", kDLFloat, 32, 4);
  const int B = static_cast<int>(q.size(0));
  const int H = static_cast<int>(q.size(2));
  const int K = static_cast<int>(q.size(3));
  const int HV = static_cast<int>(v.size(2));
  const int V = static_cast<int>(v.size(3));
  if (q.size(1) != 1) TVM_FFI_THROW(ValueError) << "decode takes T == 1";
  if (state.size(0) != B || state.size(1) != HV || state.size(2) != V || state.size(3) != K ||
      output.size(0) != B || output.size(2) != HV || output.size(3) != V ||
      new_state.size(0) != B || a.size(2) != HV || b_gate.size(2) != HV ||
      A_log.size(0) != HV || dt_bias.size(0) != HV || k.size(2) != H || v.size(0) != B)
    TVM_FFI_THROW(ValueError) << "inconsistent tensor shapes";
  const DLDevice dev = q.device();
  void* stream = TVMFFIEnvGetStream(dev.device_type, dev.device_id);
  const int rc = gdn_decode(
      static_cast<const gdn_bf16*>(base_ptr(q)), static_cast<const gdn_bf16*>(base_ptr(k)),
      static_cast<const gdn_bf16*>(base_ptr(v)), static_cast<const float*>(base_ptr(state)),
      static_cast<const float*>(base_ptr(A_log)), static_cast<const gdn_bf16*>(base_ptr(a)),
      static_cast<const float*>(base_ptr(dt_bias)), static_cast<const gdn_bf16*>(base_ptr(b_gate)),
      scale, static_cast<gdn_bf16*>(base_ptr(output)), static_cast<float*>(base_ptr(new_state)),
      B, H, HV, K, V, 0, stream);
  if (rc != GDN_OK) TVM_FFI_THROW(RuntimeError) << "gdn_decode: " << gdn_strerror(rc);
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel_cuda_b200, KernelCudaB200);
