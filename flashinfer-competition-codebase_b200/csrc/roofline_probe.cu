// roofline_probe.cu — measurement-only kernels for the benchmark (libgdn_b200_probe.so).
//
// gdn_probe_state_roundtrip reads every 16-byte chunk of a state region and writes
// it back in place with exactly the decode kernel's default T=1 work split
// (8 lanes per 512-byte row, 1 row per lane, 4-warp CTAs: 16 rows of one head per
// CTA), the same cache hints (L1::no_allocate loads, evict-first .cs stores) and
// the same order (all loads of a thread issued before its stores), but no math.
// Its duration is the floor that any kernel which reads and writes the state in
// place reaches under the same launch shape, so the decode kernel's distance to
// it is what its arithmetic, gates and input loads cost.  Not part of the decode
// library: nothing on the product path links this file.

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace {

constexpr int kDim = 128;
constexpr int kLPR = 8;                  // lanes per row
constexpr int kWarps = 4;
constexpr int kRowsPerCta = (32 / kLPR) * kWarps;   // 16
constexpr int kChunks = kDim / 4 / kLPR;            // 16-byte chunks per lane: 4

__global__ void __launch_bounds__(kWarps * 32) roundtrip_kernel(float* state) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gl = lane & (kLPR - 1);
  const int grp = lane / kLPR;
  const size_t row = static_cast<size_t>(blockIdx.x) * kRowsPerCta + warp * (32 / kLPR) + grp;
  float* p = state + row * kDim + gl * 4;
  float4 x[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c)
    asm volatile("ld.global.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(x[c].x), "=f"(x[c].y), "=f"(x[c].z), "=f"(x[c].w)
                 : "l"(p + c * kLPR * 4)
                 : "memory");
#pragma unroll
  for (int c = 0; c < kChunks; ++c)
    asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p + c * kLPR * 4),
                 "f"(x[c].x), "f"(x[c].y), "f"(x[c].z), "f"(x[c].w)
                 : "memory");
}

}  // namespace

extern "C" {

// state: `heads` consecutive [128, 128] fp32 heads, 16-byte aligned.  Returns 0, or
// -2 for a bad size, -3 for misalignment, -4 for a failed launch.
__attribute__((visibility("default"))) int gdn_probe_state_roundtrip(float* state, long long heads,
                                                                     void* stream) {
  if (heads < 1 || heads * (kDim / kRowsPerCta) > 0x7fffffffLL) return -2;
  if (reinterpret_cast<uintptr_t>(state) % 16 != 0) return -3;
  const unsigned ctas = static_cast<unsigned>(heads * (kDim / kRowsPerCta));
  roundtrip_kernel<<<ctas, kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(state);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // extern "C"
