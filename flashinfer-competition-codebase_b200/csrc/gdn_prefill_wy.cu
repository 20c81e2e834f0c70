// gdn_prefill_wy.cu — chunked (WY) variable-length prefill in two launches on the
// 5th-generation tensor cores (tcgen05 + TMEM) of B200 (sm_100a).
//
// Same recurrence and chunk algebra as gdn_prefill_chunked.cu (the reference's
// kernel_prefill_reference loop, solution/triton/prefill_kernel.py:162-181, in the WY /
// UT form of the chunked algorithm of its fla_prefill_code.py).  For a chunk of C = 64
// tokens with state S0 at its start, cumulative decays G_t, beta_t and
// T = (I + A)^-1, A[t][j] = beta_t (G_t / G_j) k_t.k_j (j < t):
//   U = T diag(beta) Vc,  W = T diag(beta G) Kc,  Q' = diag(G) Qc,
//   QKm[t][j] = (G_t / G_j) q_t.k_j (j <= t)
//   X = S0 W^T,  Delta^T = U^T - X
//   O^T = scale (S0 Q'^T + Delta^T QKm^T)
//   S = G_C S0 + Delta^T diag(G_C / G) Kc
// (X and S0 Q'^T come out of one tf32 product [X | O] = S0 [W; Q']^T.)
// U, W, Q' and QKm do not depend on the state, so every chunk of every sequence computes
// them at once in the first launch (gdn_wy_prep_kernel: one CTA per (chunk, v-head), two CTAs
// per SM) into workspace records.  The second launch (gdn_wy_state_kernel: one CTA per
// (sequence, v-head)) runs each sequence's chain of state-dependent products with the
// state in TMEM, its warps specialised so that the tensor cores, the elementwise Delta
// pass and the output conversion overlap.
//
// Workspace record of (chunk slot, v-head), 104 KB, laid out as the shared-memory
// operand images the second launch copies in with bulk copies:
//   [0, 8K)      QKm bf16, K-major 64 x 64 (element (t, j) at (j / 8) * 1024 + t * 16 + (j % 8) * 2)
//   [8K, 72K)    [W; Q'] fp32 (read as tf32), one K-major 128 x 128 operand: W row t (of
//                64) and Q' row t at rows t and 64 + t (element (r, k) at
//                (k / 4) * 2048 + r * 16 + (k % 4) * 4)
//   [72K, 104K)  U  fp32, [t][v] row-major
// Chunk c of sequence s (tokens [t0, t1) after clamping its offsets to [0, total]) has
// slot s + floor(t0 / 64) + c: distinct for the chunks of sequences that do not overlap
// (non-decreasing offsets) and always below N + ceil(total / 64), so the workspace bound
// is known on the host without reading the offsets.

#include "gdn_b200.h"
#include "tc_common.cuh"

namespace {

using namespace gdn_tc;

constexpr uint32_t kRecQKm = 0;
constexpr uint32_t kRecWQ = 8192;                 // [W; Q'] (W rows, then Q' rows at +1024)
constexpr uint32_t kRecU = 8192 + 65536;
constexpr uint32_t kRecBytes = 8192 + 3 * 32768;

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
  unsigned char* ws;        // [slots, HV] records of kRecBytes
  int32_t* status;          // set to 1 if a wait timed out (may be null)
  float scale;
  int N, total, H, HV;
  int hpc;                  // v-heads per prep CTA (2 when HV / H is even, else 1)
};

// sequence bounds clamped to [0, total] (a sequence whose end precedes its start is empty)
__device__ __forceinline__ void seq_bounds(const WyArgs& p, int s, int& t0, int& t1) {
  const int c0 = __ldg(p.cu + s), c1 = __ldg(p.cu + s + 1);
  t0 = min(max(c0, 0), p.total);
  t1 = min(max(c1, t0), p.total);
}

__device__ __forceinline__ unsigned char* record(const WyArgs& p, int slot, int hv) {
  return p.ws + (static_cast<size_t>(slot) * p.HV + hv) * kRecBytes;
}

// =====================================================================================
// Launch 1: chunk-local products of one chunk slot for `hpc` v-heads that share a q/k
// head (hpc = 2 when HV / H is even, else 1): the chunk's q/k are loaded and multiplied
// once, then each v-head's mask, triangular solve and U / W products run in turn.  256
// threads; TMEM lane quarter = warp % 4, the two warps of a quarter split the columns
// (half = warp / 4).
// =====================================================================================
constexpr int kPT = 256;
constexpr int kMaxHpc = 2;
// [Q; K] bf16 K-major 128 x 128: row r (Q rows 0-63, K rows 64-127) at r * 16 of each
// 2 KB block of 8 features.  Its K rows double as the MN-major K^T operand of W.  After
// every head's Q' is written, the Q halves (the first 1 KB of each block) hold the
// current head's T diag(beta) (hi in blocks 0-7, lo in blocks 8-15).
constexpr uint32_t kPOffQK = 0;
constexpr uint32_t kPOffVmn = kPOffQK + 32768;              // hpc x V^T bf16 MN-major
// A, then T diag(beta G) (hi, lo; 8 KB each)
constexpr uint32_t kPOffA = kPOffVmn + kMaxHpc * 16384;     // A fp32 [64][kSA]
constexpr uint32_t kPOffT = kPOffA + 64 * kSA * 4;          // T fp32 [64][kSA]
// per head: L2, beta, G, then c_j = exp2(L_31 - L_j) and r_t = exp2(L_t - L_31) [64] each
constexpr uint32_t kPOffGate = kPOffT + 64 * kSA * 4;
// 5 mbarriers: q/k loads, P1, U/W, drain, v loads
constexpr uint32_t kPOffBar = kPOffGate + kMaxHpc * 320 * 4;
constexpr uint32_t kPOffMisc = kPOffBar + 5 * 8;            // TMEM base, sequence index
constexpr uint32_t kPrepSmem = kPOffMisc + 16;
static_assert(2 * (kPrepSmem + 1024) <= 233472, "two prep CTAs fit one SM");

// TMEM (256 columns per CTA, two CTAs per SM)
constexpr uint32_t kPColW = 0;     // W (M = 64, N = 128)                         128
constexpr uint32_t kPColU = 128;   // U^T (M = 128, N = 64)                       64
constexpr uint32_t kPColP = 192;   // P1 (M = 128): rows 0-63 QK^T, 64-127 KK^T   64

constexpr uint32_t kIdP1 = idesc(1, 0, 0, 64, 128);   // [Q;K] K^T
constexpr uint32_t kIdU = idesc(1, 1, 0, 64, 128);    // V^T (T diag b)^T, A MN-major
constexpr uint32_t kIdW = idesc(1, 0, 1, 128, 64);    // (T diag bG) K,   B MN-major, M = 64

__global__ void __launch_bounds__(kPT, 2)
    gdn_wy_prep_kernel(const WyArgs p, const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kPOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kPOffMisc);
  int* s_seq = reinterpret_cast<int*>(sm + kPOffMisc + 4);
  float* sA = reinterpret_cast<float*>(sm + kPOffA);
  float* sT = reinterpret_cast<float*>(sm + kPOffT);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the state kernel is this grid's programmatic dependent: it may launch once every CTA
  // here has started, and reads no record before this grid has completed
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int hpc = p.hpc;
  const int groups = p.HV / hpc;
  const int slot = blockIdx.x / groups;
  const int hv0 = (blockIdx.x - slot * groups) * hpc;

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
  const int hq = hv0 / (p.HV / p.H);          // the same for every head of this CTA

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(bar + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  __syncthreads();

  // inputs first: TMA boxes of 1 KB, Q and K rows K-major into [Q; K] (barrier 0, needed
  // first), each head's V^T MN-major (barrier 4, needed only by the U product); the tensor
  // memory is allocated while they are in flight
  if (tid == 0) {
    const uint32_t base = smem_u32(sm), mb = smem_u32(bar + 0), mv = smem_u32(bar + 4);
    mbar_expect_tx(mb, 32 * 1024);
    for (int kc = 0; kc < 16; ++kc) {
      tma_box(base + kPOffQK + kc * 2048, &map_q, hq * kD + kc * 8, tc0, mb);
      tma_box(base + kPOffQK + kc * 2048 + 1024, &map_k, hq * kD + kc * 8, tc0, mb);
    }
    mbar_expect_tx(mv, 16 * 1024 * hpc);
    for (int kc = 0; kc < 16; ++kc)
      for (int h = 0; h < hpc; ++h)
        tma_box(base + kPOffVmn + h * 16384 + kc * 1024, &map_v, (hv0 + h) * kD + kc * 8, tc0, mv);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
        smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp >= 1 && warp <= hpc) {
    // gates of head hv0 + warp - 1
    const int hv = hv0 + warp - 1;
    float* g = reinterpret_cast<float*>(sm + kPOffGate) + (warp - 1) * 320;
    const float neg_exp_A = -ex2(__ldg(p.A_log + hv) * kLog2e);
    chunk_gates(p.a, p.b, p.HV, g, tc0, nv, hv, neg_exp_A, __ldg(p.dt_bias + hv), lane);
    __syncwarp();
    // exp2(L_t - L_j) = r_t c_j around the chunk's middle token (used when the chunk's
    // whole decay range keeps both factors inside the normal fp32 range)
    const float Lr = g[31];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = lane * 2 + h;
      g[192 + t] = ex2(Lr - g[t]);
      g[256 + t] = ex2(g[t] - Lr);
    }
  }
  // the copies are always waited for (bounded), so none is in flight at exit
  bool ok = mbar_wait(bar + 0, 0);
  fence_before();
  __syncthreads();                           // gates, TMEM address
  fence_after();
  const uint32_t tmem = *tmem_slot;
  if (nv < kC) {
    // a partial chunk: the boxes hold the next tokens of the token array (or zeros); clear
    // those rows so that nothing but this sequence's tokens meets the products
    for (int e = tid; e < (kC - nv) * 16; e += kPT) {
      const int t = nv + e / 16, c = e % 16;
      const uint4 z = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sm + kPOffQK + c * 2048 + t * 16) = z;
      *reinterpret_cast<uint4*>(sm + kPOffQK + c * 2048 + 1024 + t * 16) = z;
    }
    fence_async_smem();
    __syncthreads();
  }

  const int row = (warp & 3) * 32 + lane;
  const int half = warp >> 2;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;

  // ---- P1: [Q; K] K^T -> rows 0-63 QK^T, rows 64-127 KK^T (shared by the heads) ----
  if (tid == 0 && ok) {
    fence_after();
    const uint32_t qk = smem_u32(sm + kPOffQK);
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks)
      mma_bf16_ss(tmem + kPColP, sdesc(qk + ks * 2 * 2048, 2048, 128),
                  sdesc(qk + 64 * 16 + ks * 2 * 2048, 2048, 128), kIdP1, ks > 0);
    mma_commit(bar + 1);
  }
  // while it runs: every head's Q' = diag(G) Q as the fp32 K-major image of its record
  // (element (t, k) at (k / 4) * 1024 + t * 16)
  for (int h = 0; h < hpc; ++h) {
    const float* sG = reinterpret_cast<const float*>(sm + kPOffGate) + h * 320 + 128;
    unsigned char* rec = record(p, slot, hv0 + h);
    for (int e = tid; e < kC * 16; e += kPT) {
      const int t = e & 63, kc = e >> 6;
      const uint4 w = *reinterpret_cast<const uint4*>(sm + kPOffQK + kc * 2048 + t * 16);
      const float g = sG[t];
      *reinterpret_cast<float4*>(rec + kRecWQ + (2 * kc) * 2048 + 1024 + t * 16) =
          make_float4(g * bf16f(w.x & 0xffff), g * bf16f(w.x >> 16), g * bf16f(w.y & 0xffff),
                      g * bf16f(w.y >> 16));
      *reinterpret_cast<float4*>(rec + kRecWQ + (2 * kc + 1) * 2048 + 1024 + t * 16) =
          make_float4(g * bf16f(w.z & 0xffff), g * bf16f(w.z >> 16), g * bf16f(w.w & 0xffff),
                      g * bf16f(w.w >> 16));
    }
  }
  if (ok && !mbar_wait(bar + 1, 0)) ok = false;
  fence_after();
  __syncthreads();          // every head's Q' read the Q rows before T diag(beta) lands there

  for (int h = 0; h < hpc; ++h) {
    const float* gates = reinterpret_cast<const float*>(sm + kPOffGate) + h * 320;
    const float* sL2 = gates;
    const float* sBeta = gates + 64;
    const float* sG = gates + 128;
    unsigned char* rec = record(p, slot, hv0 + h);
    {
      // row t = row (QK^T, quarters 0-1) or row - 64 (KK^T, quarters 2-3); this thread's
      // half of the 64 columns, 8 at a time
      const int t = row & 63;
      const float Lt = sL2[t];
      const float bt = sBeta[t];
      float x[32];
      const int j0 = half * 32;
      tmem_ld32(tmem + kPColP + lane_base + j0, x);
      auto post = [&](auto decay) {
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float v8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = j0 + q8 * 8 + e;
            v8[e] = (row < 64 ? j <= t : j < t) ? decay(j) * x[q8 * 8 + e] : 0.0f;
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
      };
      if (sL2[0] - sL2[63] < 100.0f) {
        // |L_t - L_31| < 100 for every token: exp2(L_t - L_j) = r_t c_j (two multiplies)
        const float rt = gates[256 + t];
        post([&](int j) { return rt * gates[192 + j]; });
      } else {
        post([&](int j) { return ex2(Lt - sL2[j]); });
      }
    }
    fence_before();
    __syncthreads();

    // ---- T = (I + A)^-1 on the CUDA cores, by 2 x 2 block inversion ----
    // [[M11, 0], [M21, M22]]^-1 = [[M11^-1, 0], [-M22^-1 M21 M11^-1, M22^-1]], first for the
    // four 16 x 16 diagonal blocks (by substitution), then the two 32 x 32 halves, then the
    // whole; the temporaries live in A's unused upper triangle.
    // level 1: diagonal blocks D_w (warp w, lane c < 16: column c); upper blocks of T zero
    if (warp < 4 && lane < 16) {
      const int bse = warp * 16, c = lane;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // the terms of x_0..x_{i-2} first, x_{i-1} (just computed) last: the chain from
        // one row to the next is one multiply-add
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
    {
      // level 2: the 32 x 32 halves.  Thread: block b2 (0: rows 16-31 / cols 0-15, 1: rows
      // 48-63 / cols 32-47), row r, columns c, c + 1.
      const int b2 = tid >> 7, r = (tid >> 3) & 15, c = (tid & 7) * 2;
      const int ro = b2 ? 48 : 16, co = b2 ? 32 : 0;
      // P = A_ro,co D_co -> A[co + r][ro + c] (upper triangle)
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float av = sA[(ro + r) * kSA + co + m];
        a0 = fmaf(av, sT[(co + m) * kSA + co + c], a0);
        a1 = fmaf(av, sT[(co + m) * kSA + co + c + 1], a1);
      }
      sA[(co + r) * kSA + ro + c] = a0;
      sA[(co + r) * kSA + ro + c + 1] = a1;
      __syncthreads();
      // T_ro,co = -D_ro P
      a0 = 0.f; a1 = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float d = sT[(ro + r) * kSA + ro + m];
        a0 = fmaf(d, sA[(co + m) * kSA + ro + c], a0);
        a1 = fmaf(d, sA[(co + m) * kSA + ro + c + 1], a1);
      }
      sT[(ro + r) * kSA + co + c] = -a0;
      sT[(ro + r) * kSA + co + c + 1] = -a1;
    }
    __syncthreads();
    {
      // level 3: T21 = -T22 A21 T11 (32 x 32 blocks).  Thread: rows i, i + 1; columns j, j + 1.
      const int i = (tid >> 4) * 2, j = (tid & 15) * 2;
      // P = A21 T11 -> A[i][32 + j] (upper triangle); T11 holds zeros above its diagonal
      float p00 = 0.f, p01 = 0.f, p10 = 0.f, p11 = 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float a0 = sA[(32 + i) * kSA + k], a1 = sA[(33 + i) * kSA + k];
        const float2 t = *reinterpret_cast<const float2*>(sT + k * kSA + j);
        p00 = fmaf(a0, t.x, p00); p01 = fmaf(a0, t.y, p01);
        p10 = fmaf(a1, t.x, p10); p11 = fmaf(a1, t.y, p11);
      }
      *reinterpret_cast<float2*>(sA + i * kSA + 32 + j) = make_float2(p00, p01);
      *reinterpret_cast<float2*>(sA + (i + 1) * kSA + 32 + j) = make_float2(p10, p11);
      __syncthreads();
      // T21 = -T22 P; T22 holds zeros above its diagonal
      p00 = 0.f; p01 = 0.f; p10 = 0.f; p11 = 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float t0 = sT[(32 + i) * kSA + 32 + k], t1 = sT[(33 + i) * kSA + 32 + k];
        const float2 pv = *reinterpret_cast<const float2*>(sA + k * kSA + 32 + j);
        p00 = fmaf(t0, pv.x, p00); p01 = fmaf(t0, pv.y, p01);
        p10 = fmaf(t1, pv.x, p10); p11 = fmaf(t1, pv.y, p11);
      }
      *reinterpret_cast<float2*>(sT + (32 + i) * kSA + j) = make_float2(-p00, -p01);
      *reinterpret_cast<float2*>(sT + (33 + i) * kSA + j) = make_float2(-p10, -p11);
    }
    __syncthreads();
    // T diag(beta) and T diag(beta G), split hi + lo, as bf16 K-major operands (rows i,
    // 16-byte chunks of 8 columns j): T diag(beta) into the Q halves of the [Q; K] tile
    // (block jc at jc * 2048, lo from block 8), T diag(beta G) over A (dead once T is done)
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
      *reinterpret_cast<uint4*>(sm + kPOffQK + jc * 2048 + i * 16) =
          make_uint4(bh[0], bh[1], bh[2], bh[3]);
      *reinterpret_cast<uint4*>(sm + kPOffQK + (8 + jc) * 2048 + i * 16) =
          make_uint4(bl[0], bl[1], bl[2], bl[3]);
      *reinterpret_cast<uint4*>(sm + kPOffA + jc * 1024 + i * 16) =
          make_uint4(gh[0], gh[1], gh[2], gh[3]);
      *reinterpret_cast<uint4*>(sm + kPOffA + 8192 + jc * 1024 + i * 16) =
          make_uint4(gl[0], gl[1], gl[2], gl[3]);
    }
    if (h == 0) {
      // the V^T tiles (always waited for, bounded, so no copy is in flight at exit)
      if (!mbar_wait(bar + 4, 0)) ok = false;
      if (nv < kC) {
        for (int e = tid; e < (kC - nv) * 16 * hpc; e += kPT) {
          const int hh = e / ((kC - nv) * 16), r = e % ((kC - nv) * 16);
          const int t = nv + r / 16, c = r % 16;
          *reinterpret_cast<uint4*>(sm + kPOffVmn + hh * 16384 + c * 1024 + t * 16) =
              make_uint4(0, 0, 0, 0);
        }
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();

    // ---- U^T = V^T (T diag b)^T (M = 128) and W = (T diag bG) K (M = 64), hi + lo ----
    if (tid == 0 && ok) {
      fence_after();
      const uint32_t vm = smem_u32(sm + kPOffVmn + h * 16384), qk = smem_u32(sm + kPOffQK);
      const uint32_t tbg = smem_u32(sm + kPOffA);
#pragma unroll
      for (int hl = 0; hl < 2; ++hl) {
#pragma unroll
        for (int ks = 0; ks < kC / 16; ++ks) {
          mma_bf16_ss(tmem + kPColU, sdesc(vm + ks * 256, 128, 1024),
                      sdesc(qk + hl * 8 * 2048 + ks * 2 * 2048, 2048, 128), kIdU, hl + ks > 0);
          mma_bf16_ss(tmem + kPColW, sdesc(tbg + hl * 8192 + ks * 2 * 1024, 1024, 128),
                      sdesc(qk + 1024 + ks * 256, 128, 2048), kIdW, hl + ks > 0);
        }
      }
      mma_commit(bar + 2);
    }
    if (ok && !mbar_wait(bar + 2, static_cast<uint32_t>(h & 1))) ok = false;
    fence_after();
    {
      float x[32];
      // U[t][v] fp32 (lane = v): one coalesced 128-byte row piece per column t
      const int j0 = half * 32;
      tmem_ld32(tmem + kPColU + lane_base + j0, x);
      float* up = reinterpret_cast<float*>(rec + kRecU);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) up[(j0 + jj) * kD + row] = x[jj];
      // W (M = 64 layout: row i = 16 * quarter + lane, lanes 0-15) as the tf32 K-major
      // image: 16 consecutive rows' 16-byte pieces per store instruction
      const int i = (warp & 3) * 16 + lane;
      for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
        tmem_ld32(tmem + kPColW + lane_base + c0, x);
        if (lane < 16) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(rec + kRecWQ + ((c0 >> 2) + q) * 2048 + i * 16) =
                make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
        }
      }
    }
    // the next head reuses A, T, the Q halves of [Q; K] and the U / W columns
    fence_before();
    __syncthreads();
  }
  if (!ok) {
    // a wait timed out: let every product issued finish (bounded) before TMEM is released
    if (tid == 0) mma_commit(bar + 3);
    mbar_wait(bar + 3, 0);
    if (tid == 0 && p.status != nullptr) atomicOr(p.status, 1);
  }
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

// =====================================================================================
// Launch 2: the state chain of one (sequence, v-head), warp-specialised:
//   warps 0-7    Delta pass and the state rescale (TMEM lane quarter = warp % 4, the two
//                warps of a quarter split the columns)
//   warps 8-11   outputs (lane quarter = warp % 4, all 64 columns)
//   warp 12      producer: gates and the bulk / TMA copies of each chunk's operands
//   warp 13      tensor-core issue (one lane)
// Per chunk c:  [X | O] = S [W; Q']^T (one N = 128 product)  ->  Delta pass and state
// rescale  ->  O += Delta^T QKm^T, S += (Delta f)^T K  ->  [X | O] of chunk c + 1, while
// the output warps convert O of chunk c.  [W; Q'] is double-buffered (loaded a chunk
// ahead), [X | O] double-buffered in TMEM.
// =====================================================================================
constexpr int kDeltaThreads = 256;
constexpr int kOutThreads = 128;
constexpr int kSBlock = kDeltaThreads + kOutThreads + 64;
constexpr int kWarpOut0 = 8, kWarpProd = 12, kWarpMma = 13;

constexpr uint32_t kSOffWQ = 0;                      // 2 x [W; Q'] tf32 128 x 128    (bulk)
constexpr uint32_t kSOffU = kSOffWQ + 2 * 65536;     // U fp32 [t][v]                (bulk)
constexpr uint32_t kSOffQKm = kSOffU + 32768;        // QKm bf16 image 64 x 64       (bulk)
constexpr uint32_t kSOffKmn = kSOffQKm + 8192;       // K^T bf16 MN-major            (TMA)
constexpr uint32_t kSOffO = kSOffKmn + 16384;        // output staging bf16 [64][128]
constexpr uint32_t kSOffGate = kSOffO + 16384;       // 2 x {f_t [64], G_C} (80 floats each)
constexpr uint32_t kSOffBar = kSOffGate + 2 * 80 * 4;
constexpr uint32_t kSOffTmem = kSOffBar + 16 * 8;
constexpr uint32_t kStateSmem = kSOffTmem + 16;
static_assert(kStateSmem <= 227 * 1024, "fits one CTA's shared memory");

// mbarriers (arrival count 1 each)
constexpr int kBarG1 = 0;        // + (c & 1): [W; Q'] of chunk c landed
constexpr int kBarG2 = 2;        // U and the gates of the chunk landed
constexpr int kBarG3 = 3;        // QKm and K^T landed
constexpr int kBarX = 4;         // [X | O] = S [W; Q']^T done (the state may be rescaled)
constexpr int kBarS34 = 5;       // Delta products done (S and O final for the chunk)
constexpr int kBarWFree = 6;     // + (c & 1): the product reading [W; Q'] buffer c & 1 done
constexpr int kBarUFree = 8;     // U consumed
constexpr int kBarDelta = 9;     // Delta pass and rescale done
constexpr int kBarOFree = 10;    // + (c & 1): [X | O] buffer c & 1 read out
constexpr int kBarInit = 12;     // the initial state is in TMEM
constexpr int kBarDrain = 13;
constexpr int kNumBars = 14;
constexpr uint32_t kTxG1 = 65536;
constexpr uint32_t kTxG2 = 32768;
constexpr uint32_t kTxG3 = 8192 + 16384;

// named barriers: 1 = Delta warps, 2 = output warps, 3 = every warp but the producer
constexpr int kNbDelta = 1, kNbOut = 2, kNbEnd = 3;
constexpr int kEndThreads = kDeltaThreads + kOutThreads + 32;

// TMEM columns (512 allocated)
constexpr uint32_t kColS = 0;      // state S, fp32 [v][k]                       128
constexpr uint32_t kColXO = 128;   // + 128 (c & 1): [X | O^T (unscaled)] of chunk c  2 x 128
constexpr uint32_t kColDT = 384;   // Delta^T hi / lo bf16 pairs                 64
constexpr uint32_t kColDF = 448;   // (Delta diag(G_C / G))^T hi / lo            64

constexpr uint32_t kIdXO = idesc(2, 0, 0, 128, 128);  // S [W; Q']^T (tf32, A = S in TMEM)
constexpr uint32_t kIdR = idesc(1, 0, 0, 64, 128);    // Delta^T QKm^T (bf16, A in TMEM)
constexpr uint32_t kIdK = idesc(1, 0, 1, 128, 128);   // (Delta f)^T K (bf16, A in TMEM, B MN)

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
    for (int i = 0; i < kNumBars; ++i) mbar_init(bar + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  // every warp, the producer included, starts after the mbarriers are initialised and
  // the TMEM address is published
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---------------------------------------------------------------- producer ----------
  if (warp == kWarpProd) {
    // Launched as a programmatic dependent of the prep kernel: the other warps allocate
    // TMEM and load the initial state while the prep grid finishes; the records are read
    // (by this warp only) once it has completed and its stores are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
    // waits bounded; after a failed wait nothing more is issued
    const float neg_exp_A = -ex2(__ldg(p.A_log + hv) * kLog2e);
    const float dt_b = __ldg(p.dt_bias + hv);
    const uint32_t base = smem_u32(sm);
    bool pok = true;
    // group 1 of chunk c: [W; Q'] into buffer c & 1, once the product of chunk c - 2 has
    // read it; issued a chunk ahead (chunk c + 1 during chunk c), the earliest of the
    // three groups to be free, so that the 64 KB copy lands before it is needed
    auto load_g1 = [&](int c) {
      if (c >= 2 && pok)
        pok = mbar_wait(bar + kBarWFree + (c & 1), static_cast<uint32_t>(((c >> 1) - 1) & 1));
      if (lane == 0 && pok) {
        const uint32_t mb = smem_u32(bar + kBarG1 + (c & 1));
        mbar_expect_tx(mb, kTxG1);
        bulk_load(base + kSOffWQ + (c & 1) * 65536, record(p, slot0 + c, hv) + kRecWQ, 65536, mb);
      }
    };
    if (nchunks > 0) load_g1(0);
    for (int ch = 0; ch < nchunks; ++ch) {
      const int tc0 = t0 + ch * kC;
      const int nv = min(kC, t1 - tc0);
      const int b = ch & 1;
      const unsigned char* rec = record(p, slot0 + ch, hv);
      if (ch + 1 < nchunks) load_g1(ch + 1);
      // this chunk's cumulative log2 decay L (inclusive scan, padding without decay) and
      // f_t = exp2(L_C - L_t)
      float l2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = lane * 2 + h;
        l2[h] = 0.0f;
        if (t < nv) {
          const float x = bf16f(__ldg(p.a + static_cast<size_t>(tc0 + t) * p.HV + hv)) + dt_b;
          const float tx = x * kLog2e;
          l2[h] = neg_exp_A * (x > 20.0f ? tx : lg2(1.0f + ex2(tx)));
        }
      }
      float s = l2[0] + l2[1];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      const float LC = __shfl_sync(0xffffffffu, s, 31);
      const float f0 = ex2(LC - (s - l2[1])), f1 = ex2(LC - s);
      // group 2: the gates (slot b, last read by chunk ch - 2) and U, once chunk ch - 1
      // has consumed its U; the arrival also publishes the gates
      if (ch >= 1 && pok) pok = mbar_wait(bar + kBarUFree, static_cast<uint32_t>((ch - 1) & 1));
      float* g = gates + b * 80;
      g[lane * 2] = f0;
      g[lane * 2 + 1] = f1;
      if (lane == 31) g[64] = ex2(LC);
      __syncwarp();
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

  bool ok = true;
  // ---------------------------------------------------------------- MMA issue ---------
  if (warp == kWarpMma) {
    const uint32_t tS = tmem + kColS;
    const uint32_t tDT = tmem + kColDT, tDF = tmem + kColDF;
    if (nchunks > 0 && !mbar_wait(bar + kBarInit, 0)) ok = false;
    for (int ch = 0; ch < nchunks; ++ch) {
      const int tc0 = t0 + ch * kC;
      const int nv = min(kC, t1 - tc0);
      const int b = ch & 1;
      const uint32_t tXO = tmem + kColXO + b * 128;
      const uint32_t tO = tXO + 64;
      // [X | O] = S [W; Q']^T into buffer b, once the state is final for chunk ch - 1,
      // [W; Q'] has landed and the output warps have read buffer b out (chunk ch - 2)
      if (ch >= 1 && ok && !mbar_wait(bar + kBarS34, static_cast<uint32_t>((ch - 1) & 1))) ok = false;
      if (ok && !mbar_wait(bar + kBarG1 + b, static_cast<uint32_t>((ch >> 1) & 1))) ok = false;
      if (ch >= 2 && ok &&
          !mbar_wait(bar + kBarOFree + b, static_cast<uint32_t>(((ch >> 1) - 1) & 1)))
        ok = false;
      if (lane == 0 && ok) {
        fence_after();
        const uint32_t wq = smem_u32(sm + kSOffWQ + b * 65536);
#pragma unroll
        for (int ks = 0; ks < kD / 8; ++ks)
          mma_tf32_ts(tXO, tS + ks * 8, sdesc(wq + ks * 2 * 2048, 2048, 128), kIdXO, ks > 0);
        mma_commit(bar + kBarX);
        mma_commit(bar + kBarWFree + b);
      }
      // Delta products, once QKm / K^T have landed and the Delta pass is done
      if (ok && !mbar_wait(bar + kBarG3, static_cast<uint32_t>(ch & 1))) ok = false;
      if (nv < kC) {
        // padded tokens: zero their K^T columns (the next sequence's tokens or the fill)
        for (int e = lane; e < (kC - nv) * 16; e += 32) {
          const int t = nv + e / 16, c = e % 16;
          *reinterpret_cast<uint4*>(sm + kSOffKmn + c * 1024 + t * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_async_smem();
        __syncwarp();
      }
      if (ok && !mbar_wait(bar + kBarDelta, static_cast<uint32_t>(ch & 1))) ok = false;
      if (lane == 0 && ok) {
        fence_after();
        const uint32_t qkm = smem_u32(sm + kSOffQKm), km = smem_u32(sm + kSOffKmn);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int ks = 0; ks < kC / 16; ++ks) {
            mma_bf16_ts(tO, tDT + h * 32 + ks * 8, sdesc(qkm + ks * 2 * 1024, 1024, 128), kIdR, 1);
            mma_bf16_ts(tS, tDF + h * 32 + ks * 8, sdesc(km + ks * 256, 128, 1024), kIdK, 1);
          }
        }
        mma_commit(bar + kBarS34);
      }
      __syncwarp();
    }
    // a failed wait: let every product issued finish (bounded) before TMEM is released
    if (!ok) {
      if (lane == 0) mma_commit(bar + kBarDrain);
      mbar_wait(bar + kBarDrain, 0);
      if (lane == 0 && p.status != nullptr) atomicOr(p.status, 1);
    }
    fence_before();
    bar_sync(kNbEnd, kEndThreads);
    return;
  }

  // ---------------------------------------------------------------- outputs -----------
  if (warp >= kWarpOut0) {
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint16_t* so = reinterpret_cast<uint16_t*>(sm + kSOffO);
    const int otid = tid - kWarpOut0 * 32;
    for (int ch = 0; ch < nchunks; ++ch) {
      const int tc0 = t0 + ch * kC;
      const int nv = min(kC, t1 - tc0);
      if (ok && !mbar_wait(bar + kBarS34, static_cast<uint32_t>(ch & 1))) ok = false;
      // O of chunk ch - 1 was read out in the previous iteration: release its buffer now,
      // after this wait, so that the products of chunk ch + 1 cannot complete before this
      // warp group has seen those of chunk ch
      if (ch >= 1 && otid == 0) mbar_arrive(bar + kBarOFree + ((ch - 1) & 1));
      fence_after();
      // O[t][v] = scale * O^T[v][t] (row v = this thread's lane), staged as bf16 rows
      const uint32_t tO = tmem + kColXO + (ch & 1) * 128 + 64;
#pragma unroll
      for (int j0 = 0; j0 < 64; j0 += 32) {
        float x[32];
        tmem_ld32(tO + lane_base + j0, x);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) so[(j0 + jj) * kD + row] = f2bf(p.scale * x[jj]);
      }
      fence_before();
      bar_sync(kNbOut, kOutThreads);
      for (int e = otid; e < nv * 16; e += kOutThreads) {
        const int t = e >> 4, pc = e & 15;
        *reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(tc0 + t) * p.HV + hv) * kD + pc * 8) =
            *reinterpret_cast<const uint4*>(sm + kSOffO + t * 256 + pc * 16);
      }
      bar_sync(kNbOut, kOutThreads);
    }
    if (!ok && lane == 0 && p.status != nullptr) atomicOr(p.status, 1);
    fence_before();
    bar_sync(kNbEnd, kEndThreads);
    return;
  }

  // ---------------------------------------------------------------- Delta warps -------
  const int row = (warp & 3) * 32 + lane;
  const int half = warp >> 2;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t tS = tmem + kColS;
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
  bar_sync(kNbDelta, kDeltaThreads);
  if (tid == 0) mbar_arrive(bar + kBarInit);

  for (int ch = 0; ch < nchunks; ++ch) {
    const uint32_t par = static_cast<uint32_t>(ch & 1);
    const float* g = gates + (ch & 1) * 80;
    if (ok && !mbar_wait(bar + kBarX, par)) ok = false;
    if (ok && !mbar_wait(bar + kBarG2, par)) ok = false;     // U, gates
    fence_after();
    // Delta^T = U^T - X (row v), this thread's 32 of the 64 columns, as bf16 hi/lo pairs,
    // and the same scaled by f_t = G_C / G_t for the state update
    {
      float x[32];
      const int j0 = half * 32;
      tmem_ld32(tmem + kColXO + (ch & 1) * 128 + lane_base + j0, x);
      const float* su = reinterpret_cast<const float*>(sm + kSOffU);
      float dh[16], dl[16], fh[16], fl[16];
#pragma unroll
      for (int jj = 0; jj < 32; jj += 2) {
        const float d0 = su[(j0 + jj) * kD + row] - x[jj];
        const float d1 = su[(j0 + jj + 1) * kD + row] - x[jj + 1];
        uint32_t h0, l0, h1, l1;
        split2(d0, d1, h0, l0);
        split2(d0 * g[j0 + jj], d1 * g[j0 + jj + 1], h1, l1);
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
    // S <- G_C S ([X | O], the last reader of this state, is done)
    {
      float x[32];
      const float GC = g[64];
      for (int js = half * 64; js < half * 64 + 64; js += 32) {
        tmem_ld32(tS + lane_base + js, x);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) x[jj] *= GC;
        tmem_st32(tS + lane_base + js, x);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    fence_before();
    ok = bar_and(kNbDelta, kDeltaThreads, ok);
    if (tid == 0) {
      mbar_arrive(bar + kBarUFree);
      mbar_arrive(bar + kBarDelta);
    }
  }

  // final state (row v) to new_state, once the last Delta products are done
  if (nchunks > 0 && ok &&
      !mbar_wait(bar + kBarS34, static_cast<uint32_t>((nchunks - 1) & 1)))
    ok = false;
  fence_after();
  {
    float rowv[32];
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
  bar_sync(kNbEnd, kEndThreads);
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace

extern "C" {

size_t gdn_prefill_workspace_bytes(int num_seqs, int total_tokens, int HV) {
  if (num_seqs < 0 || total_tokens < 0 || HV < 1) return 0;
  const size_t slots = static_cast<size_t>(num_seqs) + (static_cast<size_t>(total_tokens) + kC - 1) / kC;
  return slots * static_cast<size_t>(HV) * kRecBytes;
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
  if (total_tokens > 0 && workspace_bytes < gdn_prefill_workspace_bytes(num_seqs, total_tokens, HV))
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
  p.status = status;
  p.scale = (scale == 0.0) ? 0.08838834764831845f : static_cast<float>(scale);
  p.N = num_seqs; p.total = total_tokens; p.H = H; p.HV = HV;
  p.hpc = (HV / H) % 2 == 0 ? 2 : 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap mq{}, mk{}, mv{};
  if (total_tokens > 0) {
    if (!token_map(&mq, q, total_tokens, H * kD) || !token_map(&mk, k, total_tokens, H * kD) ||
        !token_map(&mv, v, total_tokens, HV * kD))
      return GDN_ERR_LAUNCH;
    if (cudaFuncSetAttribute(gdn_wy_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPrepSmem)) != cudaSuccess)
      return GDN_ERR_LAUNCH;
    gdn_wy_prep_kernel<<<static_cast<unsigned>(slots * (HV / p.hpc)), kPT, kPrepSmem, st>>>(
        p, mq, mk, mv);
    if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  }
  if (cudaFuncSetAttribute(gdn_wy_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kStateSmem)) != cudaSuccess)
    return GDN_ERR_LAUNCH;
  // a programmatic dependent of the prep kernel (when there is one): its CTAs start on
  // the SMs the prep grid's tail leaves free
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(num_seqs * HV));
  cfg.blockDim = dim3(kSBlock);
  cfg.dynamicSmemBytes = kStateSmem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = total_tokens > 0 ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gdn_wy_state_kernel, p, mk) == cudaSuccess ? GDN_OK
                                                                             : GDN_ERR_LAUNCH;
}

}  // extern "C"
