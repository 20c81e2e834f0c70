// gdn_prefill_wy.cu — chunked (WY) variable-length prefill in two launches on the
// 5th-generation tensor cores (tcgen05 + TMEM) of B200 (sm_100a).
//
// Same recurrence and chunk algebra as gdn_prefill_chunked.cu (the reference's
// kernel_prefill_reference loop, solution/triton/prefill_kernel.py:162-181, in the WY /
// UT form of the chunked algorithm of its fla_prefill_code.py).  For a chunk of C = 64
// tokens with state S0 at its start, cumulative decays G_t, beta_t and
// T = (I + A)^-1, A[t][j] = beta_t (G_t / G_j) k_t.k_j (j < t):
//   U = T diag(beta) Vc,  W = T diag(beta G) Kc,  QKm[t][j] = (G_t / G_j) q_t.k_j (j <= t)
//   Delta^T = U^T - S0 W^T
//   O^T = scale (diag-free P + R) with P = S0 Qc^T scaled by G_t per token column and
//         R = Delta^T QKm^T
//   S = G_C S0 + Delta^T diag(G_C / G) Kc
// U, W and QKm do not depend on the state, so every chunk of every sequence computes
// them at once in the first launch (gdn_wy_prep_kernel: one CTA per (chunk, v-head),
// two CTAs per SM), into workspace records.  The second launch (gdn_wy_state_kernel:
// one CTA per (sequence, v-head)) keeps only the state-dependent products on each
// sequence's sequential chain: two tf32 products against the state in TMEM, one
// elementwise pass, two split-bf16 products and the output conversion.
//
// Workspace: records of (chunk slot, v-head), 72 KB each, laid out as the shared-memory
// images the second launch copies in with bulk copies,
//   [0, 8K)    QKm bf16, K-major 64 x 64 (element (t, j) at (j / 8) * 1024 + t * 16 + (j % 8) * 2)
//   [8K, 40K)  W fp32 (read as tf32), K-major 64 x 128 (element (t, k) at (k / 4) * 1024 + t * 16 + (k % 4) * 4)
//   [40K, 72K) U fp32, [t][v] row-major
// followed by the chunks' q as fp32 K-major images of (chunk slot, q/k head), 32 KB each
// (the tf32 B operand of S Q^T; written by the first v-head of each q/k head).
// Chunk c of sequence s (tokens [t0, t1) after clamping its offsets to [0, total]) has
// slot s + floor(t0 / 64) + c: distinct for the chunks of sequences that do not overlap
// (non-decreasing offsets) and always below N + ceil(total / 64), so the workspace bound
// is known on the host without reading the offsets.

#include "gdn_b200.h"
#include "tc_common.cuh"

namespace {

using namespace gdn_tc;

constexpr uint32_t kRecQKm = 0;
constexpr uint32_t kRecW = 8192;
constexpr uint32_t kRecU = 8192 + 32768;
constexpr uint32_t kRecBytes = 8192 + 2 * 32768;

constexpr int kSA = 68;     // row stride (floats) of the fp32 A and T scratch

struct WyArgs {
  const uint16_t* q;        // [total, H, K] bf16
  const uint16_t* k;
  const uint16_t* v;        // [total, HV, V] bf16
  const float* state_in;    // [N, HV, V, K] or null (zeros)
  float* state_out;         // [N, HV, V, K]
  const float* A_log;       // [HV]
  const uint16_t* a;        // [total, HV] bf16
  const float* dt_bias;     // [HV]
  const uint16_t* b;        // [total, HV] bf16
  const int32_t* cu;        // [N + 1]
  uint16_t* out;            // [total, HV, V] bf16
  unsigned char* ws;        // [slots, HV] records of kRecBytes, then [slots, H] q images
  size_t qimg_off;          // byte offset of the q images in ws
  int32_t* status;          // set to 1 if a wait timed out (may be null)
  float scale;
  int N, total, H, HV;
};
constexpr uint32_t kQImgBytes = 32768;

// sequence bounds clamped to [0, total] (a sequence whose end precedes its start is empty)
__device__ __forceinline__ void seq_bounds(const WyArgs& p, int s, int& t0, int& t1) {
  const int c0 = __ldg(p.cu + s), c1 = __ldg(p.cu + s + 1);
  t0 = min(max(c0, 0), p.total);
  t1 = min(max(c1, t0), p.total);
}

__device__ __forceinline__ unsigned char* record(const WyArgs& p, int slot, int hv) {
  return p.ws + (static_cast<size_t>(slot) * p.HV + hv) * kRecBytes;
}
__device__ __forceinline__ unsigned char* qimage(const WyArgs& p, int slot, int hq) {
  return p.ws + p.qimg_off + (static_cast<size_t>(slot) * p.H + hq) * kQImgBytes;
}

// =====================================================================================
// Launch 1: chunk-local products.  256 threads; TMEM lane quarter = warp % 4, the two
// warps of a quarter split the columns (half = warp / 4).
// =====================================================================================
constexpr int kPT = 256;
constexpr uint32_t kPOffQK = 0;                         // [Q; K] bf16 K-major 128 x 128; after
                                                        // P1: T diag(beta) hi, lo, T diag(beta G) hi, lo
constexpr uint32_t kPOffTb = kPOffQK;
constexpr uint32_t kPOffTbg = kPOffQK + 2 * 8192;
constexpr uint32_t kPOffVmn = kPOffQK + 32768;          // V^T bf16 MN-major (v x c)
constexpr uint32_t kPOffKmn = kPOffVmn + 16384;         // K^T bf16 MN-major (k x c)
constexpr uint32_t kPOffA = kPOffKmn + 16384;           // A fp32 [64][kSA]
constexpr uint32_t kPOffT = kPOffA + 64 * kSA * 4;      // T fp32 [64][kSA]
constexpr uint32_t kPOffGate = kPOffT + 64 * kSA * 4;   // L2, beta, G [64] each
constexpr uint32_t kPOffBar = kPOffGate + 192 * 4;      // 4 mbarriers: TMA, P1, U/W, drain
constexpr uint32_t kPOffMisc = kPOffBar + 4 * 8;        // TMEM base, sequence index
constexpr uint32_t kPrepSmem = kPOffMisc + 16;
static_assert(2 * (kPrepSmem + 1024) <= 233472, "two prep CTAs fit one SM");

// TMEM (256 columns per CTA, two CTAs per SM)
constexpr uint32_t kPColP = 0;     // P1 (M = 128): rows 0-63 QK^T, 64-127 KK^T   64
constexpr uint32_t kPColW = 0;     // W (M = 64, N = 128), after P1 is consumed   128
constexpr uint32_t kPColU = 128;   // U^T (M = 128, N = 64)                       64

constexpr uint32_t kIdP1 = idesc(1, 0, 0, 64, 128);   // [Q;K] K^T
constexpr uint32_t kIdU = idesc(1, 1, 0, 64, 128);    // V^T (T diag b)^T, A MN-major
constexpr uint32_t kIdW = idesc(1, 0, 1, 128, 64);    // (T diag bG) K,   B MN-major, M = 64

__global__ void __launch_bounds__(kPT, 2)
    gdn_wy_prep_kernel(const WyArgs p, const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* gates = reinterpret_cast<float*>(sm + kPOffGate);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kPOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kPOffMisc);
  int* s_seq = reinterpret_cast<int*>(sm + kPOffMisc + 4);
  float* sA = reinterpret_cast<float*>(sm + kPOffA);
  float* sT = reinterpret_cast<float*>(sm + kPOffT);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int slot = blockIdx.x / p.HV;
  const int hv = blockIdx.x - slot * p.HV;

  // which sequence's chunk is this slot (none: a gap of the slot numbering)
  if (tid == 0) *s_seq = -1;
  __syncthreads();
  for (int s = tid; s < p.N; s += kPT) {
    int t0, t1;
    seq_bounds(p, s, t0, t1);
    const int nch = (t1 - t0 + kC - 1) / kC;
    const int first = s + (t0 >> 6);
    if (nch > 0 && slot >= first && slot < first + nch) atomicMax(s_seq, s);
  }
  __syncthreads();
  const int seq = *s_seq;
  if (seq < 0) return;
  int t0, t1;
  seq_bounds(p, seq, t0, t1);
  const int tc0 = t0 + (slot - seq - (t0 >> 6)) * kC;
  const int nv = min(kC, t1 - tc0);
  const int hq = hv / (p.HV / p.H);
  unsigned char* rec = record(p, slot, hv);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
        smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(bar + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  // inputs: 64 TMA boxes of 1 KB (Q and K rows K-major into [Q; K], K^T and V^T MN-major)
  if (tid == 0) {
    const uint32_t base = smem_u32(sm), mb = smem_u32(bar + 0);
    mbar_expect_tx(mb, 64 * 1024);
    for (int kc = 0; kc < 16; ++kc) {
      tma_box(base + kPOffQK + kc * 2048, &map_q, hq * kD + kc * 8, tc0, mb);
      tma_box(base + kPOffQK + kc * 2048 + 1024, &map_k, hq * kD + kc * 8, tc0, mb);
      tma_box(base + kPOffKmn + kc * 1024, &map_k, hq * kD + kc * 8, tc0, mb);
      tma_box(base + kPOffVmn + kc * 1024, &map_v, hv * kD + kc * 8, tc0, mb);
    }
  }
  if (warp == 1) {
    const float neg_exp_A = -ex2(__ldg(p.A_log + hv) * kLog2e);
    chunk_gates(p.a, p.b, p.HV, gates, tc0, nv, hv, neg_exp_A, __ldg(p.dt_bias + hv), lane);
  }
  const float* sL2 = gates;
  const float* sBeta = gates + 64;
  const float* sG = gates + 128;
  // the copies are always waited for (bounded), so none is in flight at exit
  bool ok = mbar_wait(bar + 0, 0);
  __syncthreads();                           // gates
  if (nv < kC) {
    // a partial chunk: the boxes hold the next tokens of the token array (or zeros); clear
    // those rows so that nothing but this sequence's tokens meets the products
    for (int e = tid; e < (kC - nv) * 16; e += kPT) {
      const int t = nv + e / 16, c = e % 16;
      const uint4 z = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sm + kPOffQK + c * 2048 + t * 16) = z;
      *reinterpret_cast<uint4*>(sm + kPOffQK + c * 2048 + 1024 + t * 16) = z;
      *reinterpret_cast<uint4*>(sm + kPOffKmn + c * 1024 + t * 16) = z;
      *reinterpret_cast<uint4*>(sm + kPOffVmn + c * 1024 + t * 16) = z;
    }
    fence_async_smem();
    __syncthreads();
  }

  const int row = (warp & 3) * 32 + lane;
  const int half = warp >> 2;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;

  // ---- P1: [Q; K] K^T -> rows 0-63 QK^T, rows 64-127 KK^T ----
  // (while it runs, the first v-head of each q/k head writes the chunk's q as the fp32
  // K-major image of the second launch: element (t, k) at (k / 4) * 1024 + t * 16)
  if (tid == 0 && ok) {
    fence_after();
    const uint32_t qk = smem_u32(sm + kPOffQK);
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks)
      mma_bf16_ss(tmem + kPColP, sdesc(qk + ks * 2 * 2048, 2048, 128),
                  sdesc(qk + 64 * 16 + ks * 2 * 2048, 2048, 128), kIdP1, ks > 0);
    mma_commit(bar + 1);
  }
  if (hv % (p.HV / p.H) == 0) {
    unsigned char* qi = qimage(p, slot, hq);
    for (int e = tid; e < kC * 16; e += kPT) {
      const int t = e & 63, kc = e >> 6;
      const uint4 w = *reinterpret_cast<const uint4*>(sm + kPOffQK + kc * 2048 + t * 16);
      *reinterpret_cast<float4*>(qi + (2 * kc) * 1024 + t * 16) =
          make_float4(bf16f(w.x & 0xffff), bf16f(w.x >> 16), bf16f(w.y & 0xffff), bf16f(w.y >> 16));
      *reinterpret_cast<float4*>(qi + (2 * kc + 1) * 1024 + t * 16) =
          make_float4(bf16f(w.z & 0xffff), bf16f(w.z >> 16), bf16f(w.w & 0xffff), bf16f(w.w >> 16));
    }
  }
  if (ok && !mbar_wait(bar + 1, 0)) ok = false;
  fence_after();
  {
    // row t = row (QK^T, quarters 0-1) or row - 64 (KK^T, quarters 2-3); this thread's
    // half of the 64 columns, 8 at a time
    const int t = row & 63;
    const float Lt = sL2[t];
    const float bt = sBeta[t];
    float x[32];
    const int j0 = half * 32;
    tmem_ld32(tmem + kPColP + lane_base + j0, x);
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) {
      float v8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = j0 + q8 * 8 + e;
        v8[e] = (row < 64 ? j <= t : j < t) ? ex2(Lt - sL2[j]) * x[q8 * 8 + e] : 0.0f;
      }
      const int j = j0 + q8 * 8;
      if (row < 64) {
        // QKm[t][j] = exp(L_t - L_j) q_t.k_j, j <= t: bf16 K-major (N = t, K = j)
        *reinterpret_cast<uint4*>(rec + kRecQKm + (j >> 3) * 1024 + t * 16) =
            make_uint4(pack2(v8[0], v8[1]), pack2(v8[2], v8[3]), pack2(v8[4], v8[5]),
                       pack2(v8[6], v8[7]));
      } else {
        // A[t][j] = beta_t exp(L_t - L_j) k_t.k_j, j < t
        float4* dst = reinterpret_cast<float4*>(sA + t * kSA + j);
        dst[0] = make_float4(bt * v8[0], bt * v8[1], bt * v8[2], bt * v8[3]);
        dst[1] = make_float4(bt * v8[4], bt * v8[5], bt * v8[6], bt * v8[7]);
      }
    }
  }
  fence_before();
  __syncthreads();

  // ---- T = (I + A)^-1 on the CUDA cores, 16 x 16 blocks ----
  // diagonal blocks D_w by substitution (warp w, lane c < 16: column c), upper blocks zero
  if (warp < 4 && lane < 16) {
    const int bse = warp * 16, c = lane;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      // the terms of x_0..x_{i-2} first, x_{i-1} (just computed) last: the chain from one
      // row to the next is one multiply-add
      float acc = (i == c) ? 1.0f : 0.0f;
      float acc2 = 0.0f;
#pragma unroll
      for (int j = 0; j + 1 < i; ++j) {
        if (j & 1) acc2 -= sA[(bse + i) * kSA + bse + j] * x[j];
        else acc -= sA[(bse + i) * kSA + bse + j] * x[j];
      }
      acc += acc2;
      if (i > 0) acc -= sA[(bse + i) * kSA + bse + i - 1] * x[i - 1];
      x[i] = (i < c) ? 0.0f : acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sT[(bse + i) * kSA + bse + c] = x[i];
  }
  for (int e = tid; e < 64 * 16; e += kPT) {     // float4 slots of the upper blocks
    const int r = e >> 4, c4 = (e & 15) * 4;
    if ((c4 >> 4) > (r >> 4))
      *reinterpret_cast<float4*>(sT + r * kSA + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  // Y_ik = D_i A_ik (k < i), parked in A's unused upper block (k, i); 2 x 2 outputs per
  // thread (rows r, r + 8; columns c, c + 8)
  for (int e = tid; e < 6 * 64; e += kPT) {
    const int blk = e >> 6, r = (e >> 3) & 7, c = e & 7;
    const int bi = blk == 0 ? 1 : (blk < 3 ? 2 : 3);
    const int bk = blk == 0 ? 0 : (blk < 3 ? blk - 1 : blk - 3);
    float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const float d0 = sT[(bi * 16 + r) * kSA + bi * 16 + m];
      const float d1 = sT[(bi * 16 + r + 8) * kSA + bi * 16 + m];
      const float b0 = sA[(bi * 16 + m) * kSA + bk * 16 + c];
      const float b1 = sA[(bi * 16 + m) * kSA + bk * 16 + c + 8];
      a00 = fmaf(d0, b0, a00); a01 = fmaf(d0, b1, a01);
      a10 = fmaf(d1, b0, a10); a11 = fmaf(d1, b1, a11);
    }
    sA[(bk * 16 + r) * kSA + bi * 16 + c] = a00;
    sA[(bk * 16 + r) * kSA + bi * 16 + c + 8] = a01;
    sA[(bk * 16 + r + 8) * kSA + bi * 16 + c] = a10;
    sA[(bk * 16 + r + 8) * kSA + bi * 16 + c + 8] = a11;
  }
  __syncthreads();
  // block rows: T_ij = -sum_{k=j}^{i-1} Y_ik T_kj  (T_jj = D_j)
  for (int bi = 1; bi < 4; ++bi) {
    for (int e = tid; e < bi * 64; e += kPT) {     // 2 x 2 outputs per thread
      const int bj = e >> 6, r = (e >> 3) & 7, c = e & 7;
      float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
      for (int bk = bj; bk < bi; ++bk) {
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          const float y0 = sA[(bk * 16 + r) * kSA + bi * 16 + m];
          const float y1 = sA[(bk * 16 + r + 8) * kSA + bi * 16 + m];
          const float t0v = sT[(bk * 16 + m) * kSA + bj * 16 + c];
          const float t1v = sT[(bk * 16 + m) * kSA + bj * 16 + c + 8];
          a00 = fmaf(y0, t0v, a00); a01 = fmaf(y0, t1v, a01);
          a10 = fmaf(y1, t0v, a10); a11 = fmaf(y1, t1v, a11);
        }
      }
      sT[(bi * 16 + r) * kSA + bj * 16 + c] = -a00;
      sT[(bi * 16 + r) * kSA + bj * 16 + c + 8] = -a01;
      sT[(bi * 16 + r + 8) * kSA + bj * 16 + c] = -a10;
      sT[(bi * 16 + r + 8) * kSA + bj * 16 + c + 8] = -a11;
    }
    __syncthreads();
  }
  // T diag(beta) and T diag(beta G), split hi + lo, as bf16 K-major operands (rows i,
  // 16-byte chunks of 8 columns j), over the [Q; K] tile (dead since P1 completed)
  for (int e = tid; e < 64 * 8; e += kPT) {
    const int i = e & 63, jc = e >> 6;
    const float4 ta = *reinterpret_cast<const float4*>(sT + i * kSA + jc * 8);
    const float4 tb = *reinterpret_cast<const float4*>(sT + i * kSA + jc * 8 + 4);
    const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
    uint32_t bh[4], bl[4], gh[4], gl[4];
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      const int j = jc * 8 + 2 * e2;
      const float x0 = tv[2 * e2] * sBeta[j], x1 = tv[2 * e2 + 1] * sBeta[j + 1];
      split2(x0, x1, bh[e2], bl[e2]);
      split2(x0 * sG[j], x1 * sG[j + 1], gh[e2], gl[e2]);
    }
    const uint32_t o = jc * 1024 + i * 16;
    *reinterpret_cast<uint4*>(sm + kPOffTb + o) = make_uint4(bh[0], bh[1], bh[2], bh[3]);
    *reinterpret_cast<uint4*>(sm + kPOffTb + 8192 + o) = make_uint4(bl[0], bl[1], bl[2], bl[3]);
    *reinterpret_cast<uint4*>(sm + kPOffTbg + o) = make_uint4(gh[0], gh[1], gh[2], gh[3]);
    *reinterpret_cast<uint4*>(sm + kPOffTbg + 8192 + o) = make_uint4(gl[0], gl[1], gl[2], gl[3]);
  }
  fence_async_smem();
  fence_before();
  __syncthreads();

  // ---- U^T = V^T (T diag b)^T (M = 128) and W = (T diag bG) K (M = 64), hi + lo ----
  if (tid == 0 && ok) {
    fence_after();
    const uint32_t vm = smem_u32(sm + kPOffVmn), km = smem_u32(sm + kPOffKmn);
    const uint32_t tb = smem_u32(sm + kPOffTb), tbg = smem_u32(sm + kPOffTbg);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int ks = 0; ks < kC / 16; ++ks) {
        mma_bf16_ss(tmem + kPColU, sdesc(vm + ks * 256, 128, 1024),
                    sdesc(tb + h * 8192 + ks * 2 * 1024, 1024, 128), kIdU, h + ks > 0);
        mma_bf16_ss(tmem + kPColW, sdesc(tbg + h * 8192 + ks * 2 * 1024, 1024, 128),
                    sdesc(km + ks * 256, 128, 1024), kIdW, h + ks > 0);
      }
    }
    mma_commit(bar + 2);
  }
  if (ok && !mbar_wait(bar + 2, 0)) ok = false;
  fence_after();
  {
    float x[32];
    // U[t][v] fp32 (lane = v): one coalesced 128-byte row piece per column t
    const int j0 = half * 32;
    tmem_ld32(tmem + kPColU + lane_base + j0, x);
    float* up = reinterpret_cast<float*>(rec + kRecU);
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) up[(j0 + jj) * kD + row] = x[jj];
    // W (M = 64 layout: row i = 16 * quarter + lane, lanes 0-15) as the tf32 K-major image
    const int i = (warp & 3) * 16 + lane;
    for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
      tmem_ld32(tmem + kPColW + lane_base + c0, x);
      if (lane < 16) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(rec + kRecW + ((c0 >> 2) + q) * 1024 + i * 16) =
              make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
      }
    }
  }
  if (!ok) {
    // a wait timed out: let every product issued finish (bounded) before TMEM is released
    if (tid == 0) mma_commit(bar + 3);
    mbar_wait(bar + 3, 0);
    if (tid == 0 && p.status != nullptr) atomicOr(p.status, 1);
  }
  fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

// =====================================================================================
// Launch 2: the state chain of one (sequence, v-head).  8 compute warps (TMEM lane
// quarter = warp % 4, half = warp / 4 of each region's columns) + one producer warp.
// Per chunk the chain is: state products X = S W^T, P = S Q^T (issued at the end of the
// chunk before) -> Delta pass -> Delta products (R, S update) -> issue the next chunk's
// state products, and convert this chunk's outputs while they run.  The producer streams
// the operands in three groups, each as soon as its buffer is free: Q and W are
// double-buffered (a chunk ahead), U, QKm and K^T single-buffered.
// =====================================================================================
constexpr int kST = 256;
constexpr int kSBlock = kST + 32;
constexpr uint32_t kSOffW = 0;                       // 2 x W tf32 image 64 x 128   (bulk)
constexpr uint32_t kSOffQf = kSOffW + 2 * 32768;     // 2 x Q fp32 image 64 x 128   (bulk)
constexpr uint32_t kSOffU = kSOffQf + 2 * 32768;     // U fp32 [t][v]               (bulk)
constexpr uint32_t kSOffQKm = kSOffU + 32768;        // QKm bf16 image 64 x 64      (bulk)
constexpr uint32_t kSOffKmn = kSOffQKm + 8192;       // K^T bf16 MN-major           (TMA)
constexpr uint32_t kSOffO = kSOffKmn + 16384;        // output staging bf16 [64][128]
constexpr uint32_t kSOffGate = kSOffO + 16384;       // 4 x {L2, beta, G} [64] (ring)
constexpr uint32_t kSOffBar = kSOffGate + 4 * 192 * 4;
constexpr uint32_t kSOffTmem = kSOffBar + 10 * 8;
constexpr uint32_t kStateSmem = kSOffTmem + 16;
static_assert(kStateSmem <= 227 * 1024, "fits one CTA's shared memory");

// mbarriers
constexpr int kBarG1 = 0;      // + (chunk & 1): gates, Q and W of the chunk landed
constexpr int kBarG2 = 2;      // U landed
constexpr int kBarG3 = 3;      // QKm and K^T landed
constexpr int kBarS12 = 4;     // state products (X, P) done
constexpr int kBarS34 = 5;     // Delta products (R, S update) done
constexpr int kBarUFree = 6;   // U consumed
constexpr int kBarWFree = 7;   // + (chunk & 1): the state products reading Q / W buffer done
constexpr int kBarDrain = 9;
constexpr uint32_t kTxG1 = 2 * 32768;
constexpr uint32_t kTxG2 = 32768;
constexpr uint32_t kTxG3 = 8192 + 16384;

// TMEM columns (512 allocated)
constexpr uint32_t kColS = 0;      // state S, fp32 [v][k]                       128
constexpr uint32_t kColX = 128;    // X = S W^T                                  64
constexpr uint32_t kColP0 = 192;   // P = S Q^T of even chunks                   64
constexpr uint32_t kColR = 256;    // R = Delta^T QKm^T                          64
constexpr uint32_t kColDT = 320;   // Delta^T hi / lo bf16 pairs                 64
constexpr uint32_t kColDF = 384;   // (Delta diag(G_C / G))^T hi / lo            64
constexpr uint32_t kColP1 = 448;   // P of odd chunks                            64

constexpr uint32_t kIdX = idesc(2, 0, 0, 64, 128);    // S W^T, S Q^T (tf32, A = S in TMEM)
constexpr uint32_t kIdR = idesc(1, 0, 0, 64, 128);    // Delta^T QKm^T (bf16, A in TMEM)
constexpr uint32_t kIdK = idesc(1, 0, 1, 128, 128);   // (Delta f)^T K (bf16, A in TMEM, B MN)

__device__ __forceinline__ void csync() { bar_sync(1, kST); }
__device__ __forceinline__ bool csync_and(bool x) { return bar_and(1, kST, x); }

__global__ void __launch_bounds__(kSBlock, 1)
    gdn_wy_state_kernel(const WyArgs p, const __grid_constant__ CUtensorMap map_k) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* gates = reinterpret_cast<float*>(sm + kSOffGate);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kSOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kSOffTmem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = blockIdx.x / p.HV;
  const int hv = blockIdx.x - seq * p.HV;
  const int hq = hv / (p.HV / p.H);
  int t0, t1;
  seq_bounds(p, seq, t0, t1);
  const int len = t1 - t0;
  const int nchunks = (len + kC - 1) / kC;
  const int slot0 = seq + (t0 >> 6);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
        smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(bar + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  // every warp, the producer included, starts after the mbarriers are initialised and
  // the TMEM address is published
  fence_before();
  __syncthreads();
  fence_after();

  if (warp == 8) {
    // producer (waits bounded; after a failed wait nothing more is issued)
    const float neg_exp_A = -ex2(__ldg(p.A_log + hv) * kLog2e);
    const float dt_b = __ldg(p.dt_bias + hv);
    const uint32_t base = smem_u32(sm);
    bool pok = true;
    for (int ch = 0; ch < nchunks; ++ch) {
      const int tc0 = t0 + ch * kC;
      const int nv = min(kC, t1 - tc0);
      const int b = ch & 1;
      const unsigned char* rec = record(p, slot0 + ch, hv);
      // group 1: the gates (ring of 4: slot ch & 3 was last read by chunk ch - 4, whose
      // outputs were stored before the state products of chunk ch - 2 were issued), Q and W
      // into buffer b, once the state products of chunk ch - 2 have read it
      if (ch >= 2 && pok) pok = mbar_wait(bar + kBarWFree + b, static_cast<uint32_t>(((ch >> 1) - 1) & 1));
      chunk_gates(p.a, p.b, p.HV, gates + (ch & 3) * 192, tc0, nv, hv, neg_exp_A, dt_b, lane);
      __syncwarp();
      if (lane == 0 && pok) {
        const uint32_t mb = smem_u32(bar + kBarG1 + b);
        mbar_expect_tx(mb, kTxG1);   // this arrival also publishes the gates
        bulk_load(base + kSOffQf + b * 32768, qimage(p, slot0 + ch, hq), 32768, mb);
        bulk_load(base + kSOffW + b * 32768, rec + kRecW, 32768, mb);
      }
      // group 2: U, once chunk ch - 1 has consumed its U
      if (ch >= 1 && pok) pok = mbar_wait(bar + kBarUFree, static_cast<uint32_t>((ch - 1) & 1));
      if (lane == 0 && pok) {
        const uint32_t mb = smem_u32(bar + kBarG2);
        mbar_expect_tx(mb, kTxG2);
        bulk_load(base + kSOffU, rec + kRecU, 32768, mb);
      }
      // group 3: QKm and K^T, once the Delta products of chunk ch - 1 are done
      if (ch >= 1 && pok) pok = mbar_wait(bar + kBarS34, static_cast<uint32_t>((ch - 1) & 1));
      if (lane == 0 && pok) {
        const uint32_t mb = smem_u32(bar + kBarG3);
        mbar_expect_tx(mb, kTxG3);
        bulk_load(base + kSOffQKm, rec + kRecQKm, 8192, mb);
        for (int kc = 0; kc < 16; ++kc)
          tma_box(base + kSOffKmn + kc * 1024, &map_k, hq * kD + kc * 8, tc0, mb);
      }
    }
    // the issuing thread stays until its last copies have landed (bounded waits)
    if (lane == 0 && nchunks > 0 && pok) {
      const int last = nchunks - 1;
      mbar_wait(bar + kBarG1 + (last & 1), static_cast<uint32_t>((last >> 1) & 1));
      if (last >= 1)
        mbar_wait(bar + kBarG1 + ((last - 1) & 1), static_cast<uint32_t>(((last - 1) >> 1) & 1));
      mbar_wait(bar + kBarG2, static_cast<uint32_t>(last & 1));
      mbar_wait(bar + kBarG3, static_cast<uint32_t>(last & 1));
    }
    return;
  }

  const uint32_t tmem = *tmem_slot;
  const int row = (warp & 3) * 32 + lane;
  const int half = warp >> 2;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t tS = tmem + kColS, tX = tmem + kColX, tR = tmem + kColR;
  const uint32_t tDT = tmem + kColDT, tDF = tmem + kColDF;

  // initial state: row v into TMEM lane v (fp32), or zeros; an empty sequence ends with
  // a zero state (the reference's zero-initialised new_state)
  const size_t state_off = (static_cast<size_t>(seq) * p.HV + hv) * kD * kD +
                           static_cast<size_t>(row) * kD;
  {
    float rowv[32];
    for (int j0 = half * 64; j0 < half * 64 + 64; j0 += 32) {
      if (p.state_in != nullptr && len > 0) {
        const float4* src = reinterpret_cast<const float4*>(p.state_in + state_off + j0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 x = __ldg(src + j);
          rowv[4 * j] = x.x; rowv[4 * j + 1] = x.y; rowv[4 * j + 2] = x.z; rowv[4 * j + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) rowv[j] = 0.0f;
      }
      tmem_st32(tS + lane_base + j0, rowv);
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  fence_before();
  csync();

  // the state products of chunk c (one thread issues; every compute thread has waited
  // for the chunk's group 1 before, so that barrier cannot run a phase ahead of a waiter)
  auto issue_state_products = [&](int c) {
    if (tid != 0) return;
    fence_after();
    const uint32_t wm = smem_u32(sm + kSOffW + (c & 1) * 32768);
    const uint32_t qm = smem_u32(sm + kSOffQf + (c & 1) * 32768);
    const uint32_t tP = tmem + ((c & 1) ? kColP1 : kColP0);
#pragma unroll
    for (int ks = 0; ks < kD / 8; ++ks) {
      mma_tf32_ts(tX, tS + ks * 8, sdesc(wm + ks * 2048, 1024, 128), kIdX, ks > 0);
      mma_tf32_ts(tP, tS + ks * 8, sdesc(qm + ks * 2048, 1024, 128), kIdX, ks > 0);
    }
    mma_commit(bar + kBarS12);
    mma_commit(bar + kBarWFree + (c & 1));
  };

  bool ok = true;
  if (nchunks > 0) {
    if (!mbar_wait(bar + kBarG1, 0)) ok = false;
    ok = csync_and(ok);
    if (ok) issue_state_products(0);
  }
  // every chunk runs even after a failed wait (the barrier phases must stay in step); the
  // waits and tensor-core products are skipped once one has failed
  for (int ch = 0; ch < nchunks; ++ch) {
    const int tc0 = t0 + ch * kC;
    const int nv = min(kC, t1 - tc0);
    const uint32_t par = static_cast<uint32_t>(ch & 1);
    const float* sL2 = gates + (ch & 3) * 192;
    const float* sG = sL2 + 128;

    if (ok && !mbar_wait(bar + kBarS12, par)) ok = false;
    if (ok && !mbar_wait(bar + kBarG2, par)) ok = false;     // U
    fence_after();
    // Delta^T = U^T - X (row v), this thread's 32 of the 64 columns, as bf16 hi/lo pairs,
    // and the same scaled by f_t = G_C / G_t for the state update; then S <- G_C S
    {
      float x[32];
      const int j0 = half * 32;
      tmem_ld32(tX + lane_base + j0, x);
      const float* su = reinterpret_cast<const float*>(sm + kSOffU);
      const float LC = sL2[kC - 1];
      float dh[16], dl[16], fh[16], fl[16];
#pragma unroll
      for (int jj = 0; jj < 32; jj += 2) {
        const float d0 = su[(j0 + jj) * kD + row] - x[jj];
        const float d1 = su[(j0 + jj + 1) * kD + row] - x[jj + 1];
        uint32_t h0, l0, h1, l1;
        split2(d0, d1, h0, l0);
        const float f0 = ex2(LC - sL2[j0 + jj]), f1 = ex2(LC - sL2[j0 + jj + 1]);
        split2(d0 * f0, d1 * f1, h1, l1);
        dh[jj / 2] = __uint_as_float(h0);
        dl[jj / 2] = __uint_as_float(l0);
        fh[jj / 2] = __uint_as_float(h1);
        fl[jj / 2] = __uint_as_float(l1);
      }
      // the pair words of columns [j0, j0+32): hi at j0/2, lo at 32 + j0/2
      tmem_st16(tDT + lane_base + (j0 >> 1), dh);
      tmem_st16(tDT + lane_base + 32 + (j0 >> 1), dl);
      tmem_st16(tDF + lane_base + (j0 >> 1), fh);
      tmem_st16(tDF + lane_base + 32 + (j0 >> 1), fl);
      const float GC = sG[kC - 1];
      for (int js = half * 64; js < half * 64 + 64; js += 32) {
        tmem_ld32(tS + lane_base + js, x);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) x[jj] *= GC;
        tmem_st32(tS + lane_base + js, x);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    csync();
    if (tid == 0) mbar_arrive(bar + kBarUFree);
    if (ok && !mbar_wait(bar + kBarG3, par)) ok = false;     // QKm, K^T
    if (nv < kC) {
      // padded tokens: zero their K^T columns (the next sequence's tokens or the fill)
      for (int e = tid; e < (kC - nv) * 16; e += kST) {
        const int t = nv + e / 16, c = e % 16;
        *reinterpret_cast<uint4*>(sm + kSOffKmn + c * 1024 + t * 16) = make_uint4(0, 0, 0, 0);
      }
      fence_async_smem();
      csync();
    }

    // ---- R = Delta^T QKm^T;  S += (Delta diag f)^T K   (bf16 hi + lo, A in TMEM) ----
    if (tid == 0 && ok) {
      fence_after();
      const uint32_t qkm = smem_u32(sm + kSOffQKm), km = smem_u32(sm + kSOffKmn);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int ks = 0; ks < kC / 16; ++ks) {
          mma_bf16_ts(tR, tDT + h * 32 + ks * 8, sdesc(qkm + ks * 2 * 1024, 1024, 128), kIdR,
                      h + ks > 0);
          mma_bf16_ts(tS, tDF + h * 32 + ks * 8, sdesc(km + ks * 256, 128, 1024), kIdK, 1);
        }
      }
      mma_commit(bar + kBarS34);
    }
    if (ok && !mbar_wait(bar + kBarS34, par)) ok = false;
    // the next chunk's state products run while this chunk's outputs are converted
    if (ch + 1 < nchunks) {
      const int c1 = ch + 1;
      if (ok && !mbar_wait(bar + kBarG1 + (c1 & 1), static_cast<uint32_t>((c1 >> 1) & 1))) ok = false;
      ok = csync_and(ok);
      if (ok) issue_state_products(c1);
    }
    fence_after();
    // outputs: O[t][v] = scale (G_t P[v][t] + R[v][t]), staged as bf16 rows in shared
    // memory, then stored as 16-byte pieces of the valid tokens' rows
    {
      float pv[32], rv[32];
      uint16_t* so = reinterpret_cast<uint16_t*>(sm + kSOffO);
      const int j0 = half * 32;
      const uint32_t tP = tmem + ((ch & 1) ? kColP1 : kColP0);
      tmem_ld32(tP + lane_base + j0, pv);
      tmem_ld32(tR + lane_base + j0, rv);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        so[(j0 + jj) * kD + row] = f2bf(p.scale * fmaf(sG[j0 + jj], pv[jj], rv[jj]));
    }
    csync();
    for (int e = tid; e < nv * 16; e += kST) {
      const int t = e >> 4, pc = e & 15;
      *reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(tc0 + t) * p.HV + hv) * kD + pc * 8) =
          *reinterpret_cast<const uint4*>(sm + kSOffO + t * 256 + pc * 16);
    }
    fence_before();
    ok = csync_and(ok);                  // uniform across the compute warps
  }

  if (!ok) {
    // a wait timed out: let every product this thread issued finish (bounded) before the
    // tensor memory is released
    if (tid == 0) mma_commit(bar + kBarDrain);
    mbar_wait(bar + kBarDrain, 0);
  }
  // final state (row v) to new_state
  {
    float rowv[32];
    fence_after();
    for (int j0 = half * 64; j0 < half * 64 + 64; j0 += 32) {
      tmem_ld32(tS + lane_base + j0, rowv);
      float4* dst = reinterpret_cast<float4*>(p.state_out + state_off + j0);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        dst[j] = make_float4(rowv[4 * j], rowv[4 * j + 1], rowv[4 * j + 2], rowv[4 * j + 3]);
    }
  }
  if (!ok && lane == 0 && p.status != nullptr) atomicOr(p.status, 1);
  fence_before();
  csync();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace

extern "C" {

size_t gdn_prefill_workspace_bytes(int num_seqs, int total_tokens, int H, int HV) {
  if (num_seqs < 0 || total_tokens < 0 || H < 1 || HV < 1) return 0;
  const size_t slots = static_cast<size_t>(num_seqs) + (static_cast<size_t>(total_tokens) + kC - 1) / kC;
  return slots * (static_cast<size_t>(HV) * kRecBytes + static_cast<size_t>(H) * kQImgBytes);
}

int gdn_prefill_wy(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* state,
                   const float* A_log, const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
                   const int32_t* cu_seqlens, double scale, gdn_bf16* output, float* new_state,
                   int32_t* status, void* workspace, size_t workspace_bytes, int num_seqs,
                   int total_tokens, int H, int HV, int K, int V, void* stream) {
  if (K != kD || V != kD) return GDN_ERR_SHAPE;
  if (num_seqs < 0 || total_tokens < 0 || H < 1 || HV < 1 || HV % H != 0) return GDN_ERR_SHAPE;
  if (static_cast<long long>(num_seqs) * HV > 0x7fffffffLL) return GDN_ERR_SHAPE;
  const long long slots = static_cast<long long>(num_seqs) + (total_tokens + kC - 1LL) / kC;
  if (slots * HV > 0x7fffffffLL) return GDN_ERR_SHAPE;
  if (num_seqs == 0) return GDN_OK;
  if (!cu_seqlens || !new_state || !A_log || !dt_bias) return GDN_ERR_NULL;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !output || !workspace)) return GDN_ERR_NULL;
  auto al = [](const void* ptr, size_t n) { return reinterpret_cast<uintptr_t>(ptr) % n == 0; };
  if (!al(q, 16) || !al(k, 16) || !al(v, 16) || !al(state, 16) || !al(new_state, 16) ||
      !al(a, 2) || !al(b, 2) || !al(output, 16) || !al(A_log, 4) || !al(dt_bias, 4) ||
      !al(cu_seqlens, 4) || !al(status, 4) || !al(workspace, 16))
    return GDN_ERR_ALIGN;
  if (total_tokens > 0 && workspace_bytes < gdn_prefill_workspace_bytes(num_seqs, total_tokens, H, HV))
    return GDN_ERR_SHAPE;
  const size_t bytes = static_cast<size_t>(num_seqs) * HV * kD * kD * sizeof(float);
  if (state && state != new_state) {
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(state), s1 = reinterpret_cast<uintptr_t>(new_state);
    if (s0 < s1 + bytes && s1 < s0 + bytes) return GDN_ERR_ALIAS;
  }
  WyArgs p{};
  p.q = q; p.k = k; p.v = v; p.state_in = state; p.state_out = new_state;
  p.A_log = A_log; p.a = a; p.dt_bias = dt_bias; p.b = b; p.cu = cu_seqlens; p.out = output;
  p.ws = static_cast<unsigned char*>(workspace);
  p.qimg_off = static_cast<size_t>(slots) * HV * kRecBytes;
  p.status = status;
  p.scale = (scale == 0.0) ? 0.08838834764831845f : static_cast<float>(scale);
  p.N = num_seqs; p.total = total_tokens; p.H = H; p.HV = HV;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap mq{}, mk{}, mv{};
  if (total_tokens > 0) {
    if (!token_map(&mq, q, total_tokens, H * kD) || !token_map(&mk, k, total_tokens, H * kD) ||
        !token_map(&mv, v, total_tokens, HV * kD))
      return GDN_ERR_LAUNCH;
    if (cudaFuncSetAttribute(gdn_wy_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPrepSmem)) != cudaSuccess)
      return GDN_ERR_LAUNCH;
    gdn_wy_prep_kernel<<<static_cast<unsigned>(slots * HV), kPT, kPrepSmem, st>>>(p, mq, mk, mv);
    if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  }
  if (cudaFuncSetAttribute(gdn_wy_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kStateSmem)) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  gdn_wy_state_kernel<<<static_cast<unsigned>(num_seqs * HV), kSBlock, kStateSmem, st>>>(p, mk);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // extern "C"
