// gdn_prefill_chunked.cu — chunked (WY) variable-length prefill on the 5th-generation
// tensor cores (tcgen05 + TMEM) of B200 (sm_100a).
//
// The token recurrence of every (sequence, v-head) pair,
//   S_t = g_t S_{t-1} + delta_t k_t^T,  delta_t = beta_t (v_t - g_t S_{t-1} k_t),
//   o_t = scale S_t q_t                  (S is [V, K], k-last),
// is the reference's kernel_prefill_reference loop (solution/triton/prefill_kernel.py:
// 162-181).  Over a chunk of C = 64 tokens with the state S0 at its start, cumulative
// decays G_t = g_1 ... g_t (t inclusive) and T = (I + A)^-1, where A is strictly lower
// triangular with A[t][j] = beta_t (G_t / G_j) k_t.k_j, the recurrence is equivalent to
// (the WY / UT form of the delta rule, as in the chunked algorithm the reference's
// fla_prefill_code.py implements):
//   U = T diag(beta) Vc,  W = T diag(beta G) Kc              (C x V, C x K)
//   Delta^T = U^T - S0 W^T                                  (V x C)
//   O^T = scale (S0 (diag(G) Qc)^T + Delta^T QKm^T)         QKm[t][j] = (G_t/G_j) q_t.k_j, j <= t
//   S  = G_C S0 + Delta^T diag(G_C / G) Kc
// Only the last three lines depend on S, so each chunk costs a handful of matrix
// products instead of 64 dependent rank-1 updates.
//
// One CTA of 256 threads per (sequence, v-head) walks its chunks in order.  TMEM lane i
// is state row v = i (and row i of every M = 128 product); the two warps of each lane
// quarter split the columns.
// Tensor-core products (one elected thread issues them, completion through an
// mbarrier):
//   P1  [Qc; Kc] Kc^T          bf16 x bf16 -> fp32   M=128 N=64  K=128   (QK^T and KK^T)
//   P2  U^T = Vc^T (T diag b)^T       bf16 hi + lo    M=128 N=64  K=64    (A MN-major)
//   P3  W = (T diag bG) Kc            bf16 hi + lo    M=64  N=128 K=64    (B MN-major)
//   S12 S [W; diag(G) Qc]^T    tf32, A = S from TMEM  M=128 N=128 K=128
//   S3  += Delta^T QKm^T       bf16 hi + lo, A in TMEM M=128 N=64 K=64
//   S4  S += (Delta diag f)^T Kc  bf16 hi + lo, A in TMEM M=128 N=128 K=64 (B MN-major)
// The state stays in TMEM in fp32 for the whole sequence and feeds the tf32 products
// directly.  Every bf16 operand that is not an exact bf16 input (T diag(beta),
// T diag(beta G), Delta) is split as hi + lo, two bf16 values whose sum carries about 16
// significant bits, and both halves are multiplied.  T is solved on the CUDA cores
// (16 x 16 diagonal blocks by substitution, then block substitution).
// Operands live in shared memory in the canonical no-swizzle layouts of the tcgen05
// descriptors (8-row x 16-byte core matrices).

#include "gdn_b200.h"
#include "tc_common.cuh"

namespace {

using namespace gdn_tc;

constexpr int kThreads = 256;   // 8 compute warps: warps w and w + 4 share TMEM lane quarter w % 4
constexpr int kBlock = kThreads + 32;   // + one producer warp (loads and gates)

// named barriers: 1 = the producer may overwrite the input tiles, 2 = the next chunk's
// inputs and gates are in shared memory, 3 = the 256 compute threads
__device__ __forceinline__ void csync() { bar_sync(3, kThreads); }
__device__ __forceinline__ bool csync_and(bool x) { return bar_and(3, kThreads, x); }
constexpr int kSA = 68;     // row stride (floats) of the fp32 A and T scratch: 16-byte rows
                            // that fall on different banks

// shared-memory map (bytes)
constexpr uint32_t kOffQK = 0;                          // [Q; K] bf16 K-major, 128 x 128
// MN-major tiles (m = feature, k = token): feature group m/8 at (m/8) * 1024, token t's
// 16 bytes of that group at t * 16, so one TMA box of 64 tokens x 8 features lands as one
// contiguous 1 KB block (leading byte offset 128 between groups of 8 tokens, stride byte
// offset 1024 between groups of 8 features)
constexpr uint32_t kOffVmn = kOffQK + 128 * 128 * 2;    // V^T bf16 MN-major (v x c)
constexpr uint32_t kOffKmn = kOffVmn + 128 * 64 * 2;    // 2 x K^T bf16 MN-major (k x c)
constexpr uint32_t kOffTb = kOffKmn + 2 * 128 * 64 * 2; // T diag(beta): hi, lo   bf16 K-major
constexpr uint32_t kOffTbg = kOffTb + 2 * 64 * 64 * 2;  // T diag(beta G): hi, lo bf16 K-major
constexpr uint32_t kOffA = kOffTbg + 2 * 64 * 64 * 2;   // A fp32 [64][kSA]
constexpr uint32_t kOffT = kOffA + 64 * kSA * 4;        // T fp32 [64][kSA]
// [W; diag(G) Q]: one tf32 K-major tile of 128 rows (W rows 0-63, Q' rows 64-127) over
// A and T (dead once T diag(beta) / T diag(beta G) are built) and the space after them
constexpr uint32_t kOffWQ = kOffA;
constexpr uint32_t kOffO = kOffA;                       // output staging bf16 [64][128] (after WQ)
constexpr uint32_t kOffQKm = kOffA + 128 * 128 * 4;     // QKm bf16 K-major 64 x 64
constexpr uint32_t kOffGate = kOffQKm + 64 * 64 * 2;    // 2 x {L2, beta, G} [64]
constexpr uint32_t kOffBar = kOffGate + 2 * 3 * 64 * 4; // 6 mbarriers (5: TMA inputs)
constexpr uint32_t kOffTmem = kOffBar + 6 * 8;          // TMEM base address
constexpr uint32_t kSmemBytes = kOffTmem + 16;
static_assert(kOffT + 64 * kSA * 4 <= kOffQKm, "A and T fit under the WQ tile");
static_assert(kSmemBytes <= 227 * 1024, "fits one CTA's shared memory");

// TMEM columns (512 allocated)
constexpr uint32_t kColS = 0;      // state S, fp32 [v][k]                    128
constexpr uint32_t kColP = 128;    // P1 (M = 128): rows 0-63 QK^T, 64-127 KK^T  64
constexpr uint32_t kColW = 128;    // W (M = 64, after P1 is consumed)        128
constexpr uint32_t kColU = 256;    // U^T                                    64
constexpr uint32_t kColX = 320;    // S W^T                                  64
constexpr uint32_t kColO = 384;    // O^T (unscaled): with X one N = 128 product  64
constexpr uint32_t kColDT = 128;   // Delta^T hi / lo bf16 pairs (in W's columns)  64
constexpr uint32_t kColDF = 448;   // (Delta diag(G_C / G))^T hi / lo          64

struct ChunkArgs {
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
  int32_t* status;          // set to 1 if a wait timed out (may be null)
  float scale;
  int N, total, H, HV;
};

constexpr uint32_t kIdP1 = idesc(1, 0, 0, 64, 128);   // [Q;K] K^T
constexpr uint32_t kIdU = idesc(1, 1, 0, 64, 128);    // V^T (T diag b)^T, A MN-major
constexpr uint32_t kIdW = idesc(1, 0, 1, 128, 64);    // (T diag bG) K,   B MN-major, M = 64
constexpr uint32_t kIdS = idesc(2, 0, 0, 128, 128);   // S [W; diag(G) Q]^T (tf32)
constexpr uint32_t kIdO = idesc(1, 0, 0, 64, 128);    // Delta^T QKm^T (bf16, A in TMEM)
constexpr uint32_t kIdK = idesc(1, 0, 1, 128, 128);   // (Delta f)^T K (bf16, A in TMEM, B MN)

__global__ void __launch_bounds__(kBlock, 1)
    gdn_prefill_chunk_kernel(const ChunkArgs p, const __grid_constant__ CUtensorMap map_q,
                             const __grid_constant__ CUtensorMap map_k,
                             const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* gates = reinterpret_cast<float*>(sm + kOffGate);       // 2 x [L2 | beta | G]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffTmem);
  float* sA = reinterpret_cast<float*>(sm + kOffA);
  float* sT = reinterpret_cast<float*>(sm + kOffT);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = blockIdx.x / p.HV;
  const int hv = blockIdx.x - seq * p.HV;
  const int hq = hv / (p.HV / p.H);
  const int c0 = __ldg(p.cu + seq), c1 = __ldg(p.cu + seq + 1);
  const int t0 = min(max(c0, 0), p.total);
  const int t1 = min(max(c1, t0), p.total);
  const int len = t1 - t0;
  const int nchunks = (len + kC - 1) / kC;
  const float neg_exp_A = -ex2(__ldg(p.A_log + hv) * kLog2e);
  const float dt_b = __ldg(p.dt_bias + hv);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
        smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(bar + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  // every warp, the producer included, starts after the mbarriers are initialised (the
  // producer's first TMA completes on one) and the TMEM address is published
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 8) {
    // producer: each chunk's inputs by TMA (64 boxes of 1 KB: Q and K rows K-major into the
    // [Q; K] tile, K^T and V^T MN-major) and its gates, as soon as the compute warps release
    // the input tiles of the chunk before (the K^T tile is double-buffered)
    const uint32_t mb = smem_u32(bar + 5);
    for (int ch = 0; ch < nchunks; ++ch) {
      const int tc0 = t0 + ch * kC;
      const int nv = min(kC, t1 - tc0);
      if (ch > 0) bar_sync(1, kBlock);
      if (lane == 0) {
        const uint32_t base = smem_u32(sm);
        const uint32_t kmn = base + kOffKmn + (ch & 1) * (128 * 64 * 2);
        mbar_expect_tx(mb, 64 * 1024);
        for (int kc = 0; kc < 16; ++kc) {
          tma_box(base + kOffQK + kc * 2048, &map_q, hq * kD + kc * 8, tc0, mb);
          tma_box(base + kOffQK + kc * 2048 + 1024, &map_k, hq * kD + kc * 8, tc0, mb);
          tma_box(kmn + kc * 1024, &map_k, hq * kD + kc * 8, tc0, mb);
          tma_box(base + kOffVmn + kc * 1024, &map_v, hv * kD + kc * 8, tc0, mb);
        }
      }
      chunk_gates(p.a, p.b, p.HV, gates + (ch & 1) * 192, tc0, nv, hv, neg_exp_A, dt_b, lane);
      bar_arrive(2, kBlock);
    }
    // the issuing thread stays until its last bulk copies have landed (bounded wait)
    if (lane == 0 && nchunks > 0) mbar_wait(bar + 5, static_cast<uint32_t>((nchunks - 1) & 1));
    return;
  }
  const uint32_t tmem = *tmem_slot;
  // thread -> TMEM lane row = 32 (warp % 4) + lane, and half = warp / 4 of each region's
  // columns (a warp may only access its own quarter of the lanes)
  const int row = (warp & 3) * 32 + lane;
  const int half = warp >> 2;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t tS = tmem + kColS, tP = tmem + kColP, tU = tmem + kColU, tW = tmem + kColW;
  const uint32_t tX = tmem + kColX, tO = tmem + kColO, tDF = tmem + kColDF;
  const uint32_t tDT = tmem + kColDT;

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

  bool ok = true;
  // every chunk runs even after a failed wait (the producer's barriers must match); the
  // waits and tensor-core products are skipped once one has failed
  for (int ch = 0; ch < nchunks; ++ch) {
    const int tc0 = t0 + ch * kC;
    const int nv = min(kC, t1 - tc0);              // valid tokens in this chunk
    const uint32_t par = static_cast<uint32_t>(ch & 1);
    const uint32_t kmn_off = kOffKmn + (ch & 1) * (128 * 64 * 2);
    const float* sL2 = gates + (ch & 1) * 192;
    const float* sBeta = sL2 + 64;
    const float* sG = sL2 + 128;

    bar_sync(2, kBlock);                 // this chunk's gates are in place
    // its inputs: TMA completion (never skipped, so no copy is in flight afterwards)
    if (!mbar_wait(bar + 5, par)) ok = false;
    if (nv < kC) {
      // a partial chunk: the boxes hold the next tokens of the token array (or zeros);
      // clear those rows so that nothing but this sequence's tokens meets the products
      for (int e = tid; e < (kC - nv) * 16; e += kThreads) {
        const int t = nv + e / 16, c = e % 16;
        const uint4 z = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sm + kOffQK + c * 2048 + t * 16) = z;
        *reinterpret_cast<uint4*>(sm + kOffQK + c * 2048 + 1024 + t * 16) = z;
        *reinterpret_cast<uint4*>(sm + kmn_off + c * 1024 + t * 16) = z;
        *reinterpret_cast<uint4*>(sm + kOffVmn + c * 1024 + t * 16) = z;
      }
      fence_async_smem();
      csync();
    }

    // ---- P1: [Q; K] K^T -> rows 0-63 QK^T, rows 64-127 KK^T ----
    if (tid == 0 && ok) {
      fence_after();
      const uint32_t qk = smem_u32(sm + kOffQK);
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks)
        mma_bf16_ss(tP, sdesc(qk + ks * 2 * 2048, 2048, 128),
                    sdesc(qk + 64 * 16 + ks * 2 * 2048, 2048, 128), kIdP1, ks > 0);
      mma_commit(bar + 0);
    }
    if (ok && !mbar_wait(bar + 0, par)) ok = false;
    fence_after();
    {
      // row t = row (QK^T, lane quarters 0-1) or row - 64 (KK^T, quarters 2-3); this
      // thread's half of the 64 columns, 8 at a time
      const int t = row & 63;
      const float Lt = sL2[t];
      const float bt = sBeta[t];
      float x[32];
      {
        const int j0 = half * 32;
        tmem_ld32(tP + lane_base + j0, x);
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
            *reinterpret_cast<uint4*>(sm + kOffQKm + (j >> 3) * 1024 + t * 16) =
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
    }
    csync();

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
    for (int e = tid; e < 64 * 16; e += kThreads) {     // float4 slots of the upper blocks
      const int r = e >> 4, c4 = (e & 15) * 4;
      if ((c4 >> 4) > (r >> 4))
        *reinterpret_cast<float4*>(sT + r * kSA + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    csync();
    // Y_ik = D_i A_ik (k < i), parked in A's unused upper block (k, i); 2 x 2 outputs per
    // thread (rows r, r + 8; columns c, c + 8)
    for (int e = tid; e < 6 * 64; e += kThreads) {
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
    csync();
    // block rows: T_ij = -sum_{k=j}^{i-1} Y_ik T_kj  (T_jj = D_j)
    for (int bi = 1; bi < 4; ++bi) {
      for (int e = tid; e < bi * 64; e += kThreads) {     // 2 x 2 outputs per thread
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
      csync();
    }
    // T diag(beta) and T diag(beta G), split hi + lo, as bf16 K-major B / A operands
    // (rows i, 16-byte chunks of 8 columns j)
    for (int e = tid; e < 64 * 8; e += kThreads) {
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
      *reinterpret_cast<uint4*>(sm + kOffTb + o) = make_uint4(bh[0], bh[1], bh[2], bh[3]);
      *reinterpret_cast<uint4*>(sm + kOffTb + 8192 + o) = make_uint4(bl[0], bl[1], bl[2], bl[3]);
      *reinterpret_cast<uint4*>(sm + kOffTbg + o) = make_uint4(gh[0], gh[1], gh[2], gh[3]);
      *reinterpret_cast<uint4*>(sm + kOffTbg + 8192 + o) = make_uint4(gl[0], gl[1], gl[2], gl[3]);
    }
    fence_async_smem();
    fence_before();
    csync();

    // ---- U^T = V^T (T diag b)^T (M = 128) and W = (T diag bG) K (M = 64), hi + lo ----
    if (tid == 0 && ok) {
      fence_after();
      const uint32_t vm = smem_u32(sm + kOffVmn), km = smem_u32(sm + kmn_off);
      const uint32_t tb = smem_u32(sm + kOffTb), tbg = smem_u32(sm + kOffTbg);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int ks = 0; ks < kC / 16; ++ks) {
          mma_bf16_ss(tU, sdesc(vm + ks * 256, 128, 1024),
                      sdesc(tb + h * 8192 + ks * 2 * 1024, 1024, 128), kIdU, h + ks > 0);
          mma_bf16_ss(tW, sdesc(tbg + h * 8192 + ks * 2 * 1024, 1024, 128),
                      sdesc(km + ks * 256, 128, 1024), kIdW, h + ks > 0);
        }
      }
      mma_commit(bar + 1);
    }
    // while they run: diag(G) Q as rows 64-127 of the tf32 K-major B operand [W; diag(G) Q]
    for (int e = tid; e < 64 * 16; e += kThreads) {
      const int t = e & 63, kc = e >> 6;
      const uint4 w = *reinterpret_cast<const uint4*>(sm + kOffQK + kc * 2048 + t * 16);
      const float gt = sG[t];
      *reinterpret_cast<float4*>(sm + kOffWQ + (2 * kc) * 2048 + (64 + t) * 16) =
          make_float4(gt * bf16f(w.x & 0xffff), gt * bf16f(w.x >> 16), gt * bf16f(w.y & 0xffff),
                      gt * bf16f(w.y >> 16));
      *reinterpret_cast<float4*>(sm + kOffWQ + (2 * kc + 1) * 2048 + (64 + t) * 16) =
          make_float4(gt * bf16f(w.z & 0xffff), gt * bf16f(w.z >> 16), gt * bf16f(w.w & 0xffff),
                      gt * bf16f(w.w >> 16));
    }
    if (ok && !mbar_wait(bar + 1, par)) ok = false;
    fence_after();
    // W rows (M = 64 layout: row i = 16 * warp + lane in lanes 0-15 of each quarter) as rows
    // 0-63 of the tf32 K-major B operand [W; diag(G) Q] (N = 128, K = k)
    {
      float x[32];
      const int i = (warp & 3) * 16 + lane;
      for (int j0 = half * 64; j0 < half * 64 + 64; j0 += 32) {
        tmem_ld32(tW + lane_base + j0, x);
        if (lane < 16) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(sm + kOffWQ + ((j0 >> 2) + q) * 2048 + i * 16) =
                make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
        }
      }
    }
    fence_async_smem();
    fence_before();
    csync();

    // ---- S1 + S2: [X | O] = S [W; diag(G) Q]^T  (tf32, A = S from TMEM, N = 128) ----
    if (tid == 0 && ok) {
      fence_after();
      const uint32_t wq = smem_u32(sm + kOffWQ);
#pragma unroll
      for (int ks = 0; ks < kD / 8; ++ks)
        mma_tf32_ts(tX, tS + ks * 8, sdesc(wq + ks * 2 * 2048, 2048, 128), kIdS, ks > 0);
      mma_commit(bar + 2);
    }
    // the [Q; K] and V^T tiles and the other K^T buffer are free: the producer may load
    // the next chunk while the tensor cores work on this one
    if (ch + 1 < nchunks) bar_arrive(1, kBlock);
    if (ok && !mbar_wait(bar + 2, par)) ok = false;
    fence_after();
    // Delta^T = U^T - X (row v), this thread's 32 of the 64 columns, as bf16 hi/lo pairs
    // (W's columns are free now), and the same scaled by f_c = G_C / G_c for the state
    // update; then S <- G_C S
    {
      float u[32], x[32];
      const int j0 = half * 32;
      tmem_ld32(tU + lane_base + j0, u);
      tmem_ld32(tX + lane_base + j0, x);
      const float LC = sL2[kC - 1];
      {
        float dh[16], dl[16], fh[16], fl[16];
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          const float d0 = u[jj] - x[jj], d1 = u[jj + 1] - x[jj + 1];
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
      }
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

    // ---- S3: O += Delta^T QKm^T;  S4: S += (Delta diag f)^T K   (bf16 hi + lo, A in TMEM) ----
    if (tid == 0 && ok) {
      fence_after();
      const uint32_t qkm = smem_u32(sm + kOffQKm), km = smem_u32(sm + kmn_off);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int ks = 0; ks < kC / 16; ++ks) {
          mma_bf16_ts(tO, tDT + h * 32 + ks * 8, sdesc(qkm + ks * 2 * 1024, 1024, 128), kIdO, 1);
          mma_bf16_ts(tS, tDF + h * 32 + ks * 8, sdesc(km + ks * 256, 128, 1024), kIdK, 1);
        }
      }
      mma_commit(bar + 3);
    }
    if (ok && !mbar_wait(bar + 3, par)) ok = false;
    fence_after();
    // outputs: O[t][v] = scale * O^T[v][t], staged as bf16 rows in shared memory, then
    // stored as 16-byte pieces of the valid tokens' rows
    {
      float x[32];
      uint16_t* so = reinterpret_cast<uint16_t*>(sm + kOffO);
      const int j0 = half * 32;
      tmem_ld32(tO + lane_base + j0, x);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) so[(j0 + jj) * kD + row] = f2bf(p.scale * x[jj]);
    }
    csync();
    for (int e = tid; e < nv * 16; e += kThreads) {
      const int t = e >> 4, pc = e & 15;
      *reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(tc0 + t) * p.HV + hv) * kD + pc * 8) =
          *reinterpret_cast<const uint4*>(sm + kOffO + t * 256 + pc * 16);
    }
    fence_before();
    ok = csync_and(ok);                  // uniform across the compute warps
  }

  if (!ok) {
    // a wait timed out: let every product this thread issued finish (bounded) before the
    // tensor memory is released
    if (tid == 0) mma_commit(bar + 4);
    mbar_wait(bar + 4, 0);
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

int gdn_prefill_chunked(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                        const float* state, const float* A_log, const gdn_bf16* a,
                        const float* dt_bias, const gdn_bf16* b, const int32_t* cu_seqlens,
                        double scale, gdn_bf16* output, float* new_state, int32_t* status,
                        int num_seqs, int total_tokens, int H, int HV, int K, int V,
                        void* stream) {
  if (K != kD || V != kD) return GDN_ERR_SHAPE;
  if (num_seqs < 0 || total_tokens < 0 || H < 1 || HV < 1 || HV % H != 0) return GDN_ERR_SHAPE;
  if (static_cast<long long>(num_seqs) * HV > 0x7fffffffLL) return GDN_ERR_SHAPE;
  if (static_cast<long long>(total_tokens) * HV * kD > 0x7fffffffffffLL) return GDN_ERR_SHAPE;
  if (num_seqs == 0) return GDN_OK;
  if (!cu_seqlens || !new_state || !A_log || !dt_bias) return GDN_ERR_NULL;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !output)) return GDN_ERR_NULL;
  auto al = [](const void* ptr, size_t n) { return reinterpret_cast<uintptr_t>(ptr) % n == 0; };
  if (!al(q, 16) || !al(k, 16) || !al(v, 16) || !al(state, 16) || !al(new_state, 16) ||
      !al(a, 2) || !al(b, 2) || !al(output, 16) || !al(A_log, 4) || !al(dt_bias, 4) ||
      !al(cu_seqlens, 4) || !al(status, 4))
    return GDN_ERR_ALIGN;
  const size_t bytes = static_cast<size_t>(num_seqs) * HV * kD * kD * sizeof(float);
  if (state && state != new_state) {
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(state), s1 = reinterpret_cast<uintptr_t>(new_state);
    if (s0 < s1 + bytes && s1 < s0 + bytes) return GDN_ERR_ALIAS;
  }
  ChunkArgs p{};
  p.q = q; p.k = k; p.v = v; p.state_in = state; p.state_out = new_state;
  p.A_log = A_log; p.a = a; p.dt_bias = dt_bias; p.b = b; p.cu = cu_seqlens; p.out = output;
  p.status = status;
  p.scale = (scale == 0.0) ? 0.08838834764831845f : static_cast<float>(scale);
  p.N = num_seqs; p.total = total_tokens; p.H = H; p.HV = HV;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap mq{}, mk{}, mv{};
  if (total_tokens > 0 &&
      (!token_map(&mq, q, total_tokens, H * kD) || !token_map(&mk, k, total_tokens, H * kD) ||
       !token_map(&mv, v, total_tokens, HV * kD)))
    return GDN_ERR_LAUNCH;
  if (cudaFuncSetAttribute(gdn_prefill_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kSmemBytes)) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  gdn_prefill_chunk_kernel<<<static_cast<unsigned>(num_seqs * HV), kBlock, kSmemBytes, st>>>(
      p, mq, mk, mv);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // extern "C"
