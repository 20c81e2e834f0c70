// tc_common.cuh — device helpers shared by the chunked prefill kernels: tcgen05 matrix
// products with TMEM accumulators, shared-memory descriptors, mbarriers, TMA tile loads,
// split-precision packing and the log2-domain gates; plus the host-side tensor-map
// encoder.  sm_100a only.
#pragma once

#include <cuda.h>            // CUtensorMap and its enums (the encoder is reached at run time)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

namespace gdn_tc {

constexpr int kC = 64;      // tokens per chunk
constexpr int kD = 128;     // K == V

// ---- named barriers ------------------------------------------------------------------
__device__ __forceinline__ void bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// barrier `id` over n threads that also returns the AND of x over them
__device__ __forceinline__ bool bar_and(int id, int n, bool x) {
  uint32_t r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, %2, %3, q;\n"
               "selp.u32 %0, 1, 0, p;\n}"
               : "=r"(r)
               : "r"(static_cast<uint32_t>(x)), "r"(id), "r"(n)
               : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- tcgen05 -------------------------------------------------------------------------
// shared-memory matrix descriptor, no swizzle (start, leading / stride byte offsets of
// the core-matrix grid, descriptor version 1)
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// instruction descriptor: fp32 accumulator, A/B format (1 = bf16, 2 = tf32), majors, N, M
__host__ __device__ constexpr uint32_t idesc(int fmt, int a_mn, int b_mn, int N, int M) {
  return (1u << 4) | (static_cast<uint32_t>(fmt) << 7) | (static_cast<uint32_t>(fmt) << 10) |
         (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D (TMEM) (+)= A B, A and B bf16 in shared memory
__device__ __forceinline__ void mma_bf16_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                            uint32_t acc) {
  asm volatile("{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
               "l"(a), "l"(b), "r"(id), "r"(acc));
}
// D (+)= A B, A tf32 in TMEM, B tf32 in shared memory
__device__ __forceinline__ void mma_tf32_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id,
                                            uint32_t acc) {
  asm volatile("{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
               "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}" ::"r"(d),
               "r"(a), "l"(b), "r"(id), "r"(acc));
}
// D (+)= A B, A bf16 in TMEM, B bf16 in shared memory
__device__ __forceinline__ void mma_bf16_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id,
                                            uint32_t acc) {
  asm volatile("{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d),
               "r"(a), "l"(b), "r"(id), "r"(acc));
}
// arrive on an mbarrier once every product this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tensor cores, bulk copies)
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarriers -----------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes)
               : "memory");
}
// Wait for phase `parity` of an mbarrier, bounded by 100 ms of %globaltimer: a failure
// shows as a status flag (and every later wait of the CTA is skipped), never a hang.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const unsigned long long t0 = global_ns();
  while (true) {
    uint32_t done;
    asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 "selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(done)
                 : "r"(addr), "r"(parity)
                 : "memory");
    if (done) return true;
    if (global_ns() - t0 > 100000000ull) return false;
  }
}

// ---- TMEM loads and stores (this thread's lane) --------------------------------------
// 32 consecutive TMEM columns
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float* x) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void tmem_st32(uint32_t addr, const float* x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(addr),
      "r"(__float_as_uint(x[0])), "r"(__float_as_uint(x[1])), "r"(__float_as_uint(x[2])),
      "r"(__float_as_uint(x[3])), "r"(__float_as_uint(x[4])), "r"(__float_as_uint(x[5])),
      "r"(__float_as_uint(x[6])), "r"(__float_as_uint(x[7])), "r"(__float_as_uint(x[8])),
      "r"(__float_as_uint(x[9])), "r"(__float_as_uint(x[10])), "r"(__float_as_uint(x[11])),
      "r"(__float_as_uint(x[12])), "r"(__float_as_uint(x[13])), "r"(__float_as_uint(x[14])),
      "r"(__float_as_uint(x[15])), "r"(__float_as_uint(x[16])), "r"(__float_as_uint(x[17])),
      "r"(__float_as_uint(x[18])), "r"(__float_as_uint(x[19])), "r"(__float_as_uint(x[20])),
      "r"(__float_as_uint(x[21])), "r"(__float_as_uint(x[22])), "r"(__float_as_uint(x[23])),
      "r"(__float_as_uint(x[24])), "r"(__float_as_uint(x[25])), "r"(__float_as_uint(x[26])),
      "r"(__float_as_uint(x[27])), "r"(__float_as_uint(x[28])), "r"(__float_as_uint(x[29])),
      "r"(__float_as_uint(x[30])), "r"(__float_as_uint(x[31]))
      : "memory");
}
// 16 consecutive TMEM columns
__device__ __forceinline__ void tmem_st16(uint32_t addr, const float* x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(addr),
      "r"(__float_as_uint(x[0])), "r"(__float_as_uint(x[1])), "r"(__float_as_uint(x[2])),
      "r"(__float_as_uint(x[3])), "r"(__float_as_uint(x[4])), "r"(__float_as_uint(x[5])),
      "r"(__float_as_uint(x[6])), "r"(__float_as_uint(x[7])), "r"(__float_as_uint(x[8])),
      "r"(__float_as_uint(x[9])), "r"(__float_as_uint(x[10])), "r"(__float_as_uint(x[11])),
      "r"(__float_as_uint(x[12])), "r"(__float_as_uint(x[13])), "r"(__float_as_uint(x[14])),
      "r"(__float_as_uint(x[15]))
      : "memory");
}

// ---- numbers -------------------------------------------------------------------------
__device__ __forceinline__ float bf16f(uint16_t x) {
  return __uint_as_float(static_cast<uint32_t>(x) << 16);
}
__device__ __forceinline__ uint16_t f2bf(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// Gates in the log2 domain (as the decode kernel): log2 g = -exp(A_log) softplus(x) log2 e
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// two fp32 -> packed bf16 pair (first value in the low half), each rounded to nearest even
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
// x = hi + lo with hi = bf16(x) and lo = bf16(x - hi): two bf16 products of such a split
// operand against an exact bf16 operand carry about 16 significant bits of x
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack2(x0, x1);
  const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&hi);
  lo = pack2(x0 - __low2float(h), x1 - __high2float(h));
}

// ---- bulk copies ---------------------------------------------------------------------
// One TMA tile load (no multicast: the source is this GPU's memory, the destination this
// CTA's shared memory): a box of 64 tokens x 8 bf16 features at (x = feature, y = token),
// completing on an mbarrier.  Tokens past the tensor are zero-filled.
__device__ __forceinline__ void tma_box(uint32_t dst, const CUtensorMap* map, int x, int y,
                                        uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}
// One untiled bulk copy global -> this CTA's shared memory (both addresses 16-byte
// aligned, bytes a multiple of 16), completing on an mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(mbar)
      : "memory");
}

// ---- gates ---------------------------------------------------------------------------
// Gates of one chunk by one warp: cumulative log2 decay L (inclusive warp scan), beta
// and the cumulative decay G = exp2(L) into g[0..63], g[64..127], g[128..191]; tokens
// t >= nv (padding) have no decay and beta = 0.  a, b: [total, HV] bf16.
__device__ __forceinline__ void chunk_gates(const uint16_t* a, const uint16_t* b, int HV,
                                            float* g, int tc0, int nv, int hv, float neg_exp_A,
                                            float dt_b, int lane) {
  float l2[2], be[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int t = lane * 2 + h;
    if (t < nv) {
      const size_t tok = static_cast<size_t>(tc0 + t);
      const float x = bf16f(__ldg(a + tok * HV + hv)) + dt_b;
      const float tx = x * kLog2e;
      const float sp2 = x > 20.0f ? tx : lg2(1.0f + ex2(tx));   // softplus * log2 e
      l2[h] = neg_exp_A * sp2;
      be[h] = __frcp_rn(1.0f + ex2(-bf16f(__ldg(b + tok * HV + hv)) * kLog2e));
    } else {
      l2[h] = 0.0f;
      be[h] = 0.0f;
    }
  }
  float s = l2[0] + l2[1];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += y;
  }
  const float e0 = s - l2[1];                       // inclusive through token 2 * lane
  g[lane * 2] = e0;
  g[lane * 2 + 1] = s;
  g[64 + lane * 2] = be[0];
  g[64 + lane * 2 + 1] = be[1];
  g[128 + lane * 2] = ex2(e0);
  g[128 + lane * 2 + 1] = ex2(s);
}

// ---- host: tensor maps ---------------------------------------------------------------
// cuTensorMapEncodeTiled, looked up once through the runtime's driver entry point (no
// link-time dependency on the driver library)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline EncodeTiledFn encode_tiled() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 map over [rows, cols] (row stride cols), boxes of 64 rows x 8 columns
inline bool token_map(CUtensorMap* map, const void* base, int rows, int cols) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {8, static_cast<cuuint32_t>(kC)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gdn_tc
