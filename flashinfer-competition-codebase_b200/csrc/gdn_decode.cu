// gdn_decode.cu — Gated DeltaNet decode kernels for B200 (sm_100a) and their C ABI.
//
// The decode step is a batched rank-1 update of an fp32 [V=128, K=128] state per
// (batch entry, v-head): every state byte is read once and written once, so the
// path is HBM-bound (about 0.9 flop per byte); it stays on the FP32 pipes and
// never touches the tensor cores.
//
// Work decomposition.  A "row" is one V-row of one head's state: 128 fp32 = 512 B,
// contiguous in the k-last layout.  A row is owned by a group of LPR lanes
// (LPR = 8, 16 or 32); lane j of the group holds the 16-byte chunks
// j, j+LPR, j+2*LPR, ... of the row, so each warp-wide 16-byte load touches
// 32/LPR whole 128-byte lines.  A lane holds RG rows, a warp RPW = (32/LPR)*RG
// consecutive rows, a CTA W warps.  One CTA covers RPC = RPW*W rows of one head;
// the 1-D grid walks (batch, head, row-tile) in memory order.  Every state load
// of a thread is issued before any arithmetic, so at small batch the kernel
// costs one DRAM round trip and at large batch the many resident warps keep
// enough bytes in flight to stream at HBM rate.
//
// Arithmetic per row (h = old row, k/q of the row's q/k head, v_r = v[row]):
//   kh = k.h, qh = q.h              (both on the OLD row: one reduction round)
//   dv = beta * (v_r - g*kh)        (= new_v - old_v of the reference)
//   o  = scale * (g*qh + dv*(q.k))  (= scale * q.h_new)
//   h  = g*h + dv*k
// which is the reference's sequence old=g*S; old_v=k@old; new_v=beta*v+(1-beta)*old_v;
// S=old-k*old_v+k*new_v; o=scale*q@S (solution/triton/kernel.py:101-110) with the
// algebra folded so that both dot products share one warp-shuffle reduction and
// q.k is computed once per warp instead of once per row.

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

#include "gdn_b200.h"

namespace {

constexpr int kDim = 128;                // K == V == 128 on this path
constexpr int kHeadElems = kDim * kDim;  // fp32 elements of one head's state
constexpr int kMaxRanks = 8;             // GPUs of one NVLink node

struct StepArgs {
  const uint16_t* q;        // [B, T, H, K]  bf16
  const uint16_t* k;        // [B, T, H, K]  bf16
  const uint16_t* v;        // [B, T, HV, V] bf16
  const void* state_in;     // [slots, HV, V, K] fp32 or bf16 (the kernel's StateT)
  void* state_out;          // [slots, HV, V, K] (may equal state_in)
  const float* A_log;       // [HV]
  const uint16_t* a;        // [B, T, HV] bf16
  const float* dt_bias;     // [HV]
  const uint16_t* b;        // [B, T, HV] bf16
  uint16_t* out;            // [B, T, HV, V] bf16
  void* inter;              // [B, cache_steps, HV, V, K] StateT, or null
  const int32_t* idx_in;    // [B] read slots, or null (slot = batch entry)
  const int32_t* idx_out;   // [B] write slots, or null (= read slot)
  int32_t* bad_count;       // device counter of out-of-range indices, or null
  const int32_t* cu;        // VARLEN: [B + 1] token offsets of the B sequences
  int total;                // VARLEN: tokens in q/k/v/a/b/out (sequence bounds clamp to it)
  float scale;
  int B, T, H, HV;
  int pool;                 // number of slots in state_in/state_out
  int cache_steps;
  int l2norm;
  int write_final;
  uint32_t hv_mul, hv_shift;  // n / HV        as (umulhi(n, mul) + n) >> shift
  uint32_t hq_mul, hq_shift;  // n / (HV / H)
  // Tensor-parallel output scatter (SCATTER kernels only).  This rank owns v-heads
  // [hv0, hv0 + HV) of hv_total; its outputs go to every rank's output buffer.
  uint16_t* peer_out[kMaxRanks];  // [B, hv_total, V] bf16 of each rank, mapped here
  int world, hv0, hv_total;
  // Chained tensor-parallel step (launched as a programmatic dependent of the previous
  // step's barrier kernel): the state loads run before griddepcontrol.wait, everything
  // else after it.
  int chained;
  // Gated RMSNorm epilogue (GNORM kernels only): out = bf16(bf16(w * bf16(o * r)) *
  // silu(z)) with r = rsqrt(mean over V of o^2 + eps), o the bf16-rounded head output.
  const uint16_t* z;        // [B, 1, HV, V] bf16 gate
  const uint16_t* norm_w;   // [V] bf16 norm weight
  float eps;
};

// Arguments of the cross-rank barrier that completes a tensor-parallel step.
struct BarrierArgs {
  uint32_t* peer_sig[kMaxRanks];  // [world] signal words of each rank, mapped here
  uint32_t* epoch;                // this rank's count of completed barriers (device)
  int32_t* status;                // set to 1 if a wait timed out
  unsigned long long timeout_ns;
  int rank, world;
};

// Division by a runtime divisor d >= 1 for 0 <= n < 2^31 with one multiply-high,
// one add and one shift (round-up multiplier method, Granlund & Montgomery 1994):
// shift = ceil(log2 d), mul = floor(2^32 * (2^shift - d) / d) + 1.
__device__ __forceinline__ int div_fast(int n, uint32_t mul, uint32_t shift) {
  return static_cast<int>((__umulhi(static_cast<uint32_t>(n), mul) + static_cast<uint32_t>(n)) >> shift);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t x) {
  return __uint_as_float(static_cast<uint32_t>(x) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// 16-byte state load that does not allocate in L1 (each line is used once).
__device__ __forceinline__ float4 ld_state(const float* ptr) {
  float4 r;
  asm volatile("ld.global.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(ptr)
               : "memory");
  return r;
}

// 16-byte streaming state store (evict-first: the line is not re-read).
__device__ __forceinline__ void st_state(float* ptr, const float4& x) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "f"(x.x), "f"(x.y),
               "f"(x.z), "f"(x.w)
               : "memory");
}

// 16-byte bf16 load/store of state chunks (the bf16-state variant).
__device__ __forceinline__ uint4 ld_state_u4(const void* ptr) {
  uint4 r;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr)
               : "memory");
  return r;
}
__device__ __forceinline__ void st_state_u4(void* ptr, const uint4& x) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(x.x), "r"(x.y),
               "r"(x.z), "r"(x.w)
               : "memory");
}
// two fp32 -> packed bf16x2 in one paired conversion, each rounded to nearest even
// (low half = first value)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// One 16-byte chunk of a state row in the state's storage type, widened to fp32
// registers: 4 elements for fp32 state, 8 for bf16 state.  The math is fp32 either
// way; a bf16 state is rounded (nearest even) only when it is stored.
template <typename StateT>
struct StateChunk;

template <>
struct StateChunk<float> {
  static constexpr int kVec = 4;
  __device__ static void load(const void* ptr, float* x) {
    const float4 v = ld_state(static_cast<const float*>(ptr));
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  }
  __device__ static void store(void* ptr, const float* x) {
    st_state(static_cast<float*>(ptr), make_float4(x[0], x[1], x[2], x[3]));
  }
};

template <>
struct StateChunk<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static void load(const void* ptr, float* x) {
    const uint4 v = ld_state_u4(ptr);
    x[0] = bf16_lo(v.x); x[1] = bf16_hi(v.x); x[2] = bf16_lo(v.y); x[3] = bf16_hi(v.y);
    x[4] = bf16_lo(v.z); x[5] = bf16_hi(v.z); x[6] = bf16_lo(v.w); x[7] = bf16_hi(v.w);
  }
  __device__ static void store(void* ptr, const float* x) {
    st_state_u4(ptr, make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]),
                                pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7])));
  }
};

// kVec consecutive bf16 inputs (q or k) of one chunk, loaded as one 8- or 16-byte word.
template <int kVec>
struct BfChunk;
template <>
struct BfChunk<4> {
  uint2 w;
  __device__ void load(const uint16_t* ptr) { w = __ldg(reinterpret_cast<const uint2*>(ptr)); }
  __device__ void widen(float* x) const {
    x[0] = bf16_lo(w.x); x[1] = bf16_hi(w.x); x[2] = bf16_lo(w.y); x[3] = bf16_hi(w.y);
  }
};
template <>
struct BfChunk<8> {
  uint4 w;
  __device__ void load(const uint16_t* ptr) { w = __ldg(reinterpret_cast<const uint4*>(ptr)); }
  __device__ void widen(float* x) const {
    x[0] = bf16_lo(w.x); x[1] = bf16_hi(w.x); x[2] = bf16_lo(w.y); x[3] = bf16_hi(w.y);
    x[4] = bf16_lo(w.z); x[5] = bf16_hi(w.z); x[6] = bf16_lo(w.w); x[7] = bf16_hi(w.w);
  }
};

// Cross-GPU signalling over NVLink peer memory (system scope).
__device__ __forceinline__ void st_relaxed_sys(uint32_t* ptr, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <int LPR>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// All-reduce of two values over the LPR lanes of a row group with log2(LPR)+1
// shuffles instead of 2*log2(LPR): the first exchange swaps halves so each half
// reduces one of the two values, the last exchange hands each half the other sum.
// All lanes of a group end with bit-identical sums.
template <int LPR>
__device__ __forceinline__ void group_sum2(float& x, float& y, int lane) {
  constexpr int kHalf = LPR / 2;
  const bool hi = (lane & kHalf) != 0;
  const float send = hi ? x : y;
  float keep = hi ? y : x;
  keep += __shfl_xor_sync(0xffffffffu, send, kHalf);
#pragma unroll
  for (int o = kHalf / 2; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
  const float other = __shfl_xor_sync(0xffffffffu, keep, kHalf);
  x = hi ? other : keep;
  y = hi ? keep : other;
}

// Gate math on the critical path of every warp, written in the log2 domain so
// that it costs three hardware exp2/log2 approximations (ex2/lg2.approx, relative
// error ~2^-22) instead of the longer accurate expf/log1pf sequences:
//   softplus(x) * log2(e) = log2(1 + 2^(x log2 e))     (x if x > 20: PyTorch's
//                                                      threshold, kernel.py:74, :290)
//   g    = exp(-exp(A_log) * softplus(x)) = 2^(neg_exp_A * softplus(x) * log2 e)
//   beta = 1 / (1 + 2^(-b log2 e))
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float log2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// -exp(A_log)
__device__ __forceinline__ float neg_exp(float a_log) { return -exp2_approx(a_log * kLog2e); }
// decay g from neg_exp_A = -exp(A_log) and x = a + dt_bias
__device__ __forceinline__ float decay_gate(float neg_exp_A, float x) {
  const float t = x * kLog2e;
  const float sp2 = x > 20.0f ? t : log2_approx(1.0f + exp2_approx(t));
  return exp2_approx(neg_exp_A * sp2);
}
__device__ __forceinline__ float update_gate(float b) {
  return __frcp_rn(1.0f + exp2_approx(-b * kLog2e));
}

// Per-token inputs of one warp, kept packed until they are used so that the
// next token's loads can be in flight while this token computes.
template <int NC, int RG, int VEC>
struct TokenRaw {
  BfChunk<VEC> q[NC];
  BfChunk<VEC> k[NC];
  uint16_t v[RG];
  uint16_t a, b;
};

// One kernel body for every variant of the step:
//   TT == 1: single token (decode), TT == 0: T tokens from p.T (multi-token);
//   POOL: slots come from p.idx_in / p.idx_out; L2N: q and k are L2-normalised.
// The flags are compile-time so that the plain decode path carries no code for
// the variants it does not use (at small batch instruction fetch after a cold
// start is part of the critical path).
//   SCATTER (T = 1, no pool): tensor-parallel step; the CTA's output rows are
//   staged in shared memory and stored into every rank's output buffer over
//   NVLink, then the ranks meet at a bounded barrier (see the epilogue).
//   VARLEN (TT == 0, no pool): variable-length prefill; batch entry bi is sequence bi
//   with tokens cu[bi] .. cu[bi+1]-1 of flat [total, ...] inputs and state slot bi.
//   GNORM (T = 1, no pool): the head's outputs go through the decode layer's gated
//   RMSNorm before they are stored (see the epilogue).  GNORM == 1: the CTA holds a
//   whole head.  GNORM == 2: the kDim / kRPC CTAs of a head form a thread-block
//   cluster and add their partial sums of squares through distributed shared memory.
template <int LPR, int RG, int W, int TT, bool POOL, bool L2N, bool SCATTER,
          typename StateT = float, bool VARLEN = false, int GNORM = 0>
__global__ void __launch_bounds__(W * 32) gdn_step_kernel(const StepArgs p) {
  using Chunk = StateChunk<StateT>;
  constexpr int kVec = Chunk::kVec;     // state elements per 16-byte chunk
  constexpr int kGroups = 32 / LPR;     // row groups per warp
  constexpr int kRPW = kGroups * RG;    // rows per warp
  constexpr int kRPC = kRPW * W;        // rows per CTA
  constexpr int kEPL = kDim / LPR;      // elements per lane per row
  constexpr int kNC = kEPL / kVec;      // 16-byte chunks per lane per row
  constexpr int kTPH = kDim / kRPC;     // CTAs per head
  static_assert(kNC >= 1, "a lane holds at least one 16-byte chunk of a row");
  static_assert(kDim % kRPC == 0, "rows per CTA must divide V");
  static_assert(!SCATTER || (TT == 1 && !POOL && kRPC % 8 == 0),
                "the scatter epilogue moves whole 16-byte chunks of T=1 outputs");
  static_assert(!VARLEN || (TT == 0 && !POOL && !SCATTER), "varlen prefill is multi-token");
  static_assert(!GNORM || (TT == 1 && !POOL && !SCATTER && !VARLEN && kRPC <= 32 * W),
                "the gated norm is a T = 1 epilogue with one thread per output row");
  static_assert(GNORM != 1 || kRPC == kDim, "GNORM == 1 needs a whole head per CTA");
  static_assert(GNORM != 2 || (kTPH >= 2 && kTPH <= 8 && kRPC <= 32),
                "GNORM == 2: a portable cluster of 2..8 CTAs, one warp reduces a CTA's rows");
  __shared__ __align__(16) uint16_t s_out[SCATTER ? kRPC : 1];
  // GNORM: [0, kRPC) the CTA's bf16-rounded outputs, [kRPC] unused, [kRPC + 1] the
  // head's rsqrt, [kRPC + 2 + c] (GNORM == 2) the sum of squares of cluster CTA c's rows,
  // stored there by CTA c
  __shared__ float s_norm[GNORM ? kRPC + 2 + 8 : 1];
  // GNORM == 2: an mbarrier that completes once all kTPH partial sums have landed here
  // (each CTA's st.async carries 4 bytes of transaction count).  It is initialised and
  // armed before the cluster barrier's one phase, which is arrived at here and waited on
  // just before the first store into another CTA, so every CTA is running and has armed
  // its mbarrier by then.
  __shared__ __align__(8) uint64_t s_nbar[GNORM == 2 ? 1 : 1];
  if constexpr (GNORM == 2) {
    if (threadIdx.x == 0) {
      const uint32_t nb = static_cast<uint32_t>(__cvta_generic_to_shared(s_nbar));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(nb) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(nb),
                   "r"(static_cast<uint32_t>(kTPH * 4)) : "memory");
    }
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  }

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gl = lane & (LPR - 1);
  const int grp = lane / LPR;

  // The step's barrier kernel is this grid's programmatic dependent: it may launch once
  // every CTA has started, and waits (griddepcontrol.wait) for the whole grid to finish.
  if constexpr (SCATTER) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int bh = blockIdx.x / kTPH;
  const int tile_in_head = blockIdx.x - bh * kTPH;
  const int row0 = tile_in_head * kRPC + warp * kRPW + grp;  // row of r is row0 + r*kGroups
  const int bi = div_fast(bh, p.hv_mul, p.hv_shift);
  const int hv = bh - bi * p.HV;
  const int hq = div_fast(hv, p.hq_mul, p.hq_shift);
  int T = TT ? TT : p.T;
  int tok0 = 0;  // VARLEN: first token of the sequence
  if constexpr (VARLEN) {
    // sequence bounds clamped to [0, total] so that no offsets can leave the inputs
    const int c0 = __ldg(p.cu + bi), c1 = __ldg(p.cu + bi + 1);
    tok0 = min(max(c0, 0), p.total);
    T = min(max(c1, tok0), p.total) - tok0;
  }

  // ---- slots -------------------------------------------------------------
  int slot_in = bi;
  int slot_out = bi;
  bool active = true;
  bool do_write = p.write_final != 0;
  if constexpr (POOL) {
    slot_in = __ldg(p.idx_in + bi);
    const bool counted = (hv == 0 && tile_in_head == 0 && threadIdx.x == 0);
    if (slot_in < 0 || slot_in >= p.pool) {
      if (slot_in >= p.pool && counted && p.bad_count) atomicAdd(p.bad_count, 1);
      active = false;
    }
    slot_out = slot_in;
    if (active && p.idx_out != nullptr) {
      slot_out = __ldg(p.idx_out + bi);
      if (slot_out < 0) {
        slot_out = 0;  // null-buffer convention of the pool API
      } else if (slot_out >= p.pool) {
        if (counted && p.bad_count) atomicAdd(p.bad_count, 1);
        do_write = false;
      }
    }
  }

  // Offsets into q/k/v/a/b/output fit in 31 bits (checked on the host).
  auto load_token = [&](int t, TokenRaw<kNC, RG, kVec>& raw) {
    const int bt = VARLEN ? tok0 + t : bi * T + t;
    const uint16_t* qp = p.q + (bt * p.H + hq) * kDim + gl * kVec;
    const uint16_t* kp = p.k + (bt * p.H + hq) * kDim + gl * kVec;
#pragma unroll
    for (int c = 0; c < kNC; ++c) {
      raw.q[c].load(qp + c * LPR * kVec);
      raw.k[c].load(kp + c * LPR * kVec);
    }
    const uint16_t* vp = p.v + (bt * p.HV + hv) * kDim + row0;
#pragma unroll
    for (int r = 0; r < RG; ++r) raw.v[r] = __ldg(vp + r * kGroups);
    raw.a = __ldg(p.a + bt * p.HV + hv);
    raw.b = __ldg(p.b + bt * p.HV + hv);
  };

  // Single-token steps outside the tensor-parallel chain fetch the token's q/k/v and
  // gates before the state: they arrive first, so the gate chain and q.k run while the
  // state is still in flight (at small batch that latency is the step's critical path).
  // A chained tensor-parallel step may read only the state before its dependency wait.
  constexpr bool kTokFirst = TT == 1 && !SCATTER;
  TokenRaw<kNC, RG, kVec> tok_first;
  float neg_exp_A = 0.0f, dt_b = 0.0f;
  if constexpr (kTokFirst) {
    load_token(0, tok_first);
    neg_exp_A = neg_exp(__ldg(p.A_log + hv));
    dt_b = __ldg(p.dt_bias + hv);
  }

  // ---- state loads: the only large transfer --------------------------------
  // Lane gl holds chunks gl, gl+LPR, ... of each of its rows: element
  // (c*LPR + gl)*kVec + e of the row is h[r][c*kVec + e].
  float h[RG][kEPL];
  if (VARLEN && (p.state_in == nullptr || T == 0)) {
    // no initial state: start from zeros; an empty sequence ends with a zero state
    // (the reference's zero-initialised new_state, prefill_kernel.py:145-157)
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int e = 0; e < kEPL; ++e) h[r][e] = 0.0f;
  } else if (active) {
    const StateT* src = static_cast<const StateT*>(p.state_in) +
                        (static_cast<size_t>(slot_in) * p.HV + hv) * kHeadElems +
                        static_cast<size_t>(row0) * kDim + gl * kVec;
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int c = 0; c < kNC; ++c)
        Chunk::load(src + r * kGroups * kDim + c * LPR * kVec, &h[r][c * kVec]);
  }

  // GNORM: the gate z and the norm weight of this thread's output row, fetched here so
  // that their latency hides under the state loads.
  uint16_t z_raw = 0, w_raw = 0;
  if constexpr (GNORM != 0) {
    if (threadIdx.x < kRPC) {
      const int row = tile_in_head * kRPC + threadIdx.x;
      z_raw = __ldg(p.z + (static_cast<size_t>(bi) * p.HV + hv) * kDim + row);
      w_raw = __ldg(p.norm_w + row);
    }
  }

  if constexpr (SCATTER) {
    // A chained step may start while the previous step's barrier kernel still waits
    // for the other ranks: only the state (last written by a decode grid that had
    // completed before that barrier let this grid launch) is read before this point.  The wait returns once
    // the barrier grid has completed and its memory operations are visible, so the
    // inputs, the outputs of other ranks and this rank's peer stores below are ordered
    // after it (the two-buffer rule of the output buffers relies on that).  Without a
    // programmatic launch the wait returns at once.
    if (p.chained) asm volatile("griddepcontrol.wait;" ::: "memory");
  }

  TokenRaw<kNC, RG, kVec> cur;
  if constexpr (kTokFirst) {
    cur = tok_first;
  } else {
    if (!VARLEN || T > 0) load_token(0, cur);
    neg_exp_A = neg_exp(__ldg(p.A_log + hv));
    dt_b = __ldg(p.dt_bias + hv);
  }

  for (int t = 0; t < T; ++t) {
    TokenRaw<kNC, RG, kVec> nxt;
    if (TT != 1 && t + 1 < T) load_token(t + 1, nxt);

    // Gates (solution/triton/kernel.py:73-75): g = exp(-exp(A_log)*softplus(a+dt_bias)),
    // beta = sigmoid(b).
    const float g = decay_gate(neg_exp_A, bf16_to_f32(cur.a) + dt_b);
    const float beta = update_gate(bf16_to_f32(cur.b));

    float qf[kEPL], kf[kEPL];
#pragma unroll
    for (int c = 0; c < kNC; ++c) {
      cur.q[c].widen(&qf[c * kVec]);
      cur.k[c].widen(&kf[c * kVec]);
    }
    float qk = 0.0f;
#pragma unroll
    for (int e = 0; e < kEPL; ++e) qk = fmaf(qf[e], kf[e], qk);
    if constexpr (L2N) {
      // x * rsqrt(sum(x^2) + 1e-6), the convention of
      // flashinfer/gdn_kernels/gdn_decode_pretranspose.py:253-254.
      float qq = 0.0f, kk = 0.0f;
#pragma unroll
      for (int e = 0; e < kEPL; ++e) {
        qq = fmaf(qf[e], qf[e], qq);
        kk = fmaf(kf[e], kf[e], kk);
      }
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) {
        qq += __shfl_xor_sync(0xffffffffu, qq, o);
        kk += __shfl_xor_sync(0xffffffffu, kk, o);
        qk += __shfl_xor_sync(0xffffffffu, qk, o);
      }
      const float rq = rsqrtf(qq + 1e-6f);
      const float rk = rsqrtf(kk + 1e-6f);
#pragma unroll
      for (int e = 0; e < kEPL; ++e) {
        qf[e] *= rq;
        kf[e] *= rk;
      }
      qk *= rq * rk;
    } else {
      qk = group_sum<LPR>(qk);
    }

    const int bt = VARLEN ? tok0 + t : bi * T + t;
    uint16_t* op = p.out + (bt * p.HV + hv) * kDim + row0;
    if (active) {
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        float kh0 = 0.0f, kh1 = 0.0f, qh0 = 0.0f, qh1 = 0.0f;
#pragma unroll
        for (int e = 0; e < kEPL; e += 2) {
          kh0 = fmaf(kf[e], h[r][e], kh0);
          kh1 = fmaf(kf[e + 1], h[r][e + 1], kh1);
          qh0 = fmaf(qf[e], h[r][e], qh0);
          qh1 = fmaf(qf[e + 1], h[r][e + 1], qh1);
        }
        float kh = kh0 + kh1;
        float qh = qh0 + qh1;
        group_sum2<LPR>(kh, qh, lane);
        const float dv = beta * (bf16_to_f32(cur.v[r]) - g * kh);
        const float o = p.scale * fmaf(g, qh, dv * qk);
#pragma unroll
        for (int e = 0; e < kEPL; ++e) h[r][e] = fmaf(dv, kf[e], g * h[r][e]);
        if (gl == 0) {
          if constexpr (GNORM) {
            s_norm[warp * kRPW + r * kGroups + grp] = bf16_to_f32(f32_to_bf16(o));
          } else if constexpr (SCATTER) {
            s_out[warp * kRPW + r * kGroups + grp] = f32_to_bf16(o);
          } else {
            op[r * kGroups] = f32_to_bf16(o);
          }
        }
      }
      if (TT != 1 && p.inter != nullptr) {
        StateT* ip = static_cast<StateT*>(p.inter) +
                     ((static_cast<size_t>(bi) * p.cache_steps + t) * p.HV + hv) * kHeadElems +
                     static_cast<size_t>(row0) * kDim + gl * kVec;
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
          for (int c = 0; c < kNC; ++c)
            Chunk::store(ip + r * kGroups * kDim + c * LPR * kVec, &h[r][c * kVec]);
      }
    } else if (gl == 0) {
#pragma unroll
      for (int r = 0; r < RG; ++r) op[r * kGroups] = 0;
    }
    if (TT != 1) cur = nxt;
  }

  if (active && do_write) {
    StateT* dst = static_cast<StateT*>(p.state_out) +
                  (static_cast<size_t>(slot_out) * p.HV + hv) * kHeadElems +
                  static_cast<size_t>(row0) * kDim + gl * kVec;
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int c = 0; c < kNC; ++c)
        Chunk::store(dst + r * kGroups * kDim + c * LPR * kVec, &h[r][c * kVec]);
  }

  if constexpr (GNORM != 0) {
    // Gated RMSNorm of the head's bf16 output o[0..127] (Qwen3-Next's decode layer,
    // transformers models/qwen3_next/modeling_qwen3_next.py:73-82):
    //   x = o * rsqrt(mean(o^2) + eps)   (fp32), rounded to bf16
    //   y = w * x                        (bf16 * bf16, rounded to bf16)
    //   out = y * silu(z)                (fp32), rounded to bf16
    __syncthreads();
    if constexpr (GNORM == 1) {
      if (warp == 0) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < kDim / 32; ++j) {
          const float x = s_norm[lane * (kDim / 32) + j];
          ss = fmaf(x, x, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) s_norm[kRPC + 1] = rsqrtf(ss * (1.0f / kDim) + p.eps);
      }
      __syncthreads();
    } else {
      // The cluster is the kTPH CTAs of this head (cluster rank = tile_in_head).  Each
      // sends the sum of squares of its rows to slot kRPC + 2 + tile_in_head of every
      // CTA's shared memory (its own included) with st.async, which completes 4 bytes of
      // the receiving CTA's mbarrier transaction count; each CTA waits on its own
      // mbarrier and reads its own copy.  No cluster-scope fence is involved, and a CTA
      // exits only after every partial sum addressed to it has landed.  The wait is
      // bounded (it cannot run out while every CTA of the cluster runs, which the
      // cluster launch guarantees); if it ever did, the head's outputs would be NaN.
      asm volatile("barrier.cluster.wait.aligned;" ::: "memory");   // all CTAs armed
      if (warp == 0) {
        const float x = lane < kRPC ? s_norm[lane] : 0.0f;
        float ss = x * x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane < kTPH) {
          const uint32_t local =
              static_cast<uint32_t>(__cvta_generic_to_shared(&s_norm[kRPC + 2 + tile_in_head]));
          const uint32_t lbar = static_cast<uint32_t>(__cvta_generic_to_shared(s_nbar));
          uint32_t remote, rbar;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(lane));
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(lbar), "r"(lane));
          asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                       ::"r"(remote), "r"(__float_as_uint(ss)), "r"(rbar) : "memory");
        }
        const uint32_t nb = static_cast<uint32_t>(__cvta_generic_to_shared(s_nbar));
        uint32_t done = 0;
        for (int it = 0; it < (1 << 22) && !done; ++it) {
          asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n"
                       "selp.u32 %0, 1, 0, p;\n}" : "=r"(done) : "r"(nb) : "memory");
        }
        float tot = (done && lane < kTPH) ? s_norm[kRPC + 2 + lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        if (lane == 0) s_norm[kRPC + 1] = done ? rsqrtf(tot * (1.0f / kDim) + p.eps) : __int_as_float(0x7fc00000);
      }
      __syncthreads();
    }
    if (threadIdx.x < kRPC) {
      const int row = tile_in_head * kRPC + threadIdx.x;
      const size_t off = (static_cast<size_t>(bi) * p.HV + hv) * kDim + row;
      const float x = bf16_to_f32(f32_to_bf16(s_norm[threadIdx.x] * s_norm[kRPC + 1]));
      const float y = bf16_to_f32(f32_to_bf16(bf16_to_f32(w_raw) * x));
      const float zf = bf16_to_f32(z_raw);
      const float silu = zf / (1.0f + expf(-zf));
      p.out[off] = f32_to_bf16(y * silu);
    }
  }

  if constexpr (SCATTER) {
    // The CTA's kRPC outputs (one head, rows tile_in_head*kRPC ...) go to every
    // rank's output buffer as 16-byte NVLink stores, overlapping the other CTAs'
    // math.  Completion is established by tp_barrier_kernel, which signals the other
    // ranks only after its griddepcontrol.wait has seen this grid finish (all of its
    // stores performed).
    constexpr int kChunks = kRPC * 2 / 16;
    __syncthreads();
    if (threadIdx.x < p.world * kChunks) {
      const int peer = threadIdx.x / kChunks;
      const int c = threadIdx.x - peer * kChunks;
      uint4* dst = reinterpret_cast<uint4*>(
          p.peer_out[peer] + (static_cast<size_t>(bi) * p.hv_total + p.hv0 + hv) * kDim +
          tile_in_head * kRPC);
      dst[c] = reinterpret_cast<const uint4*>(s_out)[c];
    }
  }
}

// Cross-rank barrier of a tensor-parallel step, one thread per rank j: announce to
// rank j that this rank's outputs are in place (the step's epoch into word `rank` of
// j's signal array), then wait until rank j has announced the same in this rank's
// array (acquire).  The epoch is this rank's device counter of completed barriers
// plus one (every rank runs the same sequence of barriers, so the values agree),
// advanced here after the waits: the kernel takes no per-call value and can be
// replayed from a CUDA graph.  Each wait is bounded: past timeout_ns it records the
// failure in *status and gives up.
//
// The kernel is launched as a programmatic dependent of the step's decode grid, so its
// launch overlaps that grid's last wave.  griddepcontrol.wait returns once the decode
// grid has completed and its memory operations are performed, the stores into the
// other ranks' buffers included (they are performed where they land, in the owner's
// memory); the signal stores come after it in program order, so a rank that sees the
// signal finds this rank's rows in its buffer.  The signal is therefore a relaxed
// system-scope store: a release store, or a fence.sys before it, adds about 2 us per
// step on B200 (measured: a one-thread kernel takes 1.0 us empty, 1.4 us with a
// relaxed system-scope store, 3.3 us with a release store, 5.3 us with fence + release
// + acquire poll) and orders nothing more here.
__global__ void tp_barrier_kernel(const BarrierArgs p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Let a chained next step (this grid's programmatic dependent) launch now that the
  // decode grid is complete (every state it wrote is in memory): its CTAs load their
  // state while this kernel waits, and wait for this grid before touching anything else.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = *p.epoch + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int j = threadIdx.x;
  if (j < p.world) {
    st_relaxed_sys(p.peer_sig[j] + p.rank, e);
    const uint32_t* mine = p.peer_sig[p.rank] + j;
    const unsigned long long t0 = global_ns();
    while (static_cast<int>(ld_acquire_sys(mine) - e) < 0) {
      if (global_ns() - t0 > p.timeout_ns) {
        atomicOr(p.status, 1);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *p.epoch = e;
}

// Tensor-parallel head interleave: gathered [W, rows, HVl, V] -> out [rows, W*HVl, V],
// moved as 8-byte words (V % 4 == 0).
__global__ void interleave_heads_kernel(const uint2* __restrict__ src, uint2* __restrict__ dst,
                                        int world, int rows, int hvl, int v4) {
  const size_t per_rank = static_cast<size_t>(rows) * hvl * v4;
  const size_t total = per_rank * world;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t w = i / per_rank;
    const size_t rem = i - w * per_rank;
    const size_t r = rem / (static_cast<size_t>(hvl) * v4);
    const size_t jv = rem - r * hvl * v4;  // j * v4 + e
    dst[(r * world + w) * hvl * v4 + jv] = src[i];
  }
}

// ---- host side --------------------------------------------------------------

struct LaunchShape {
  int lpr, rg, warps;
};

using LaunchFn = cudaError_t (*)(const StepArgs&, cudaStream_t);

template <int LPR, int RG, int W, int TT, bool POOL, bool L2N, bool SCATTER = false>
cudaError_t launch_step(const StepArgs& p, cudaStream_t stream) {
  constexpr int kRPC = (32 / LPR) * RG * W;
  const long long ctas = static_cast<long long>(p.B) * p.HV * (kDim / kRPC);
  if (SCATTER && p.chained) {
    // programmatic dependent launch after the previous step's barrier kernel
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(W * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gdn_step_kernel<LPR, RG, W, TT, POOL, L2N, SCATTER>, p);
  }
  gdn_step_kernel<LPR, RG, W, TT, POOL, L2N, SCATTER>
      <<<static_cast<unsigned>(ctas), W * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

// Tensor-parallel (scatter) kernels exist for the two default T=1 shapes.
LaunchFn pick_scatter(LaunchShape s, bool l2n) {
  if (s.lpr == 8 && s.rg == 1 && s.warps == 4)
    return l2n ? &launch_step<8, 1, 4, 1, false, true, true> : &launch_step<8, 1, 4, 1, false, false, true>;
  if (s.lpr == 8 && s.rg == 4 && s.warps == 1)
    return l2n ? &launch_step<8, 4, 1, 1, false, true, true> : &launch_step<8, 4, 1, 1, false, false, true>;
  return nullptr;
}


// Every launch shape is instantiated for the plain path (tuning sweeps); the pooled
// and L2-normalised paths carry the shapes the default heuristic can choose.
template <int TT, bool POOL, bool L2N>
LaunchFn pick_launch(LaunchShape s) {
#define GDN_SHAPE(L, R, W) \
  if (s.lpr == L && s.rg == R && s.warps == W) return &launch_step<L, R, W, TT, POOL, L2N>;
#define GDN_SHAPES_W(L, R) GDN_SHAPE(L, R, 1) GDN_SHAPE(L, R, 2) GDN_SHAPE(L, R, 4) GDN_SHAPE(L, R, 8)
#define GDN_SHAPES_R(L) GDN_SHAPES_W(L, 1) GDN_SHAPES_W(L, 2) GDN_SHAPES_W(L, 4)
  if constexpr (!POOL && !L2N) {
    GDN_SHAPES_R(8)
    GDN_SHAPES_R(16)
    GDN_SHAPES_R(32)
  } else {
    GDN_SHAPE(8, 1, 4)
    GDN_SHAPE(8, 4, 1)
  }
#undef GDN_SHAPES_R
#undef GDN_SHAPES_W
#undef GDN_SHAPE
  return nullptr;
}

template <int TT>
LaunchFn pick_variant(LaunchShape s, bool pool, bool l2n) {
  if (pool) return l2n ? pick_launch<TT, true, true>(s) : pick_launch<TT, true, false>(s);
  return l2n ? pick_launch<TT, false, true>(s) : pick_launch<TT, false, false>(s);
}

// bf16-state kernels (the FlashInfer bf16-state backend's storage): the two default
// shapes, one or many tokens, with or without pool indices and q/k L2-norm.
template <int LPR, int RG, int W, int TT, bool POOL, bool L2N>
cudaError_t launch_bf16(const StepArgs& p, cudaStream_t stream) {
  constexpr int kRPC = (32 / LPR) * RG * W;
  const long long ctas = static_cast<long long>(p.B) * p.HV * (kDim / kRPC);
  gdn_step_kernel<LPR, RG, W, TT, POOL, L2N, false, __nv_bfloat16>
      <<<static_cast<unsigned>(ctas), W * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int TT, bool POOL, bool L2N>
LaunchFn pick_bf16_shape(LaunchShape s) {
  if (s.lpr == 16 && s.rg == 4 && s.warps == 2) return &launch_bf16<16, 4, 2, TT, POOL, L2N>;
  if (s.lpr == 8 && s.rg == 1 && s.warps == 4) return &launch_bf16<8, 1, 4, TT, POOL, L2N>;
  if (s.lpr == 8 && s.rg == 4 && s.warps == 1) return &launch_bf16<8, 4, 1, TT, POOL, L2N>;
  return nullptr;
}

template <int TT>
LaunchFn pick_bf16_variant(LaunchShape s, bool pool, bool l2n) {
  if (pool) return l2n ? pick_bf16_shape<TT, true, true>(s) : pick_bf16_shape<TT, true, false>(s);
  return l2n ? pick_bf16_shape<TT, false, true>(s) : pick_bf16_shape<TT, false, false>(s);
}

// Decode step with the gated RMSNorm epilogue, with and without the q/k L2-norm.
// At small batch (few heads) a head is spread over a cluster of 8 CTAs of 4 warps (the
// plain step's split: 16 rows per CTA, 8 lanes per row), which keeps as many SMs
// loading state as the plain step does; the CTAs add their partial sums of squares
// through distributed shared memory.  At large batch one CTA of 8 warps (4 rows per
// lane) holds a whole head and the norm needs no cluster.
template <bool L2N>
cudaError_t launch_gated_norm(const StepArgs& p, cudaStream_t stream) {
  const long long heads = static_cast<long long>(p.B) * p.HV;
  if (heads <= 512) {
    constexpr int kTPH = 8;  // CTAs per head = cluster size
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(heads * kTPH));
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kTPH;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gdn_step_kernel<8, 1, 4, 1, false, L2N, false, float, false, 2>,
                              p);
  }
  gdn_step_kernel<8, 4, 8, 1, false, L2N, false, float, false, 1>
      <<<static_cast<unsigned>(heads), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// Variable-length prefill kernels (fp32 state): a few work splits, with and without
// the q/k L2-norm.
template <int LPR, int RG, int W, bool L2N>
cudaError_t launch_prefill(const StepArgs& p, cudaStream_t stream) {
  constexpr int kRPC = (32 / LPR) * RG * W;
  const long long ctas = static_cast<long long>(p.B) * p.HV * (kDim / kRPC);
  gdn_step_kernel<LPR, RG, W, 0, false, L2N, false, float, true>
      <<<static_cast<unsigned>(ctas), W * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

LaunchFn pick_prefill(LaunchShape s, bool l2n) {
#define GDN_PF_SHAPE(L, R, W) \
  if (s.lpr == L && s.rg == R && s.warps == W) \
    return l2n ? &launch_prefill<L, R, W, true> : &launch_prefill<L, R, W, false>;
  GDN_PF_SHAPE(8, 1, 1)
  GDN_PF_SHAPE(8, 2, 1)
  GDN_PF_SHAPE(8, 4, 1)
  GDN_PF_SHAPE(8, 1, 4)
  GDN_PF_SHAPE(16, 1, 1)
#undef GDN_PF_SHAPE
  return nullptr;
}

// Prefill work split: the token loop of every sequence is one dependent chain per row,
// so a few (sequence, head) pairs are spread over as many SMs as possible (4 rows per
// CTA); many pairs keep several independent rows per lane instead.
LaunchShape prefill_shape(long long heads) {
  if (heads <= 64) return LaunchShape{8, 1, 1};
  return LaunchShape{8, 4, 1};
}

// Launch shape by regime, from CUPTI sweeps of all 36 shapes on B200 (16/32 heads):
//  - T = 1: 4-warp CTAs of 4-row warps (8 lanes per row) are fastest or within
//    1 % of the fastest at B = 1 (256 CTAs over 148 SMs, latency-bound), B = 64
//    and B = 256 (bandwidth-bound); between 65 and 512 heads (B <= 16) warps of 16
//    rows in 1-warp CTAs win (B = 8: 7.4 us vs 7.7 us);
//  - T > 1: 16 rows per warp keep four independent rows per lane in flight across
//    the token loop (B = 64, T = 2..4: best at 8/4/1, 8/1/4 is 1.9x slower).
LaunchShape default_shape(long long heads, int T) {
  if (T > 1) return LaunchShape{8, 4, 1};
  if (heads > 64 && heads <= 512) return LaunchShape{8, 4, 1};
  return LaunchShape{8, 1, 4};
}

// Constants of div_fast for divisor d >= 1.
void div_constants(uint32_t d, uint32_t& mul, uint32_t& shift) {
  shift = 0;
  while ((1ull << shift) < d) ++shift;
  mul = static_cast<uint32_t>(((1ull << 32) * ((1ull << shift) - d)) / d + 1);
}

bool aligned(const void* ptr, size_t n) { return (reinterpret_cast<uintptr_t>(ptr) % n) == 0; }

bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + nb && pb < pa + na;
}

float resolve_scale(double scale, int K) {
  return (scale == 0.0) ? static_cast<float>(1.0 / sqrt(static_cast<double>(K))) : static_cast<float>(scale);
}

// Returned by check_common when the sizes are valid and B == 0: the call is a
// no-op (empty tensors may carry NULL pointers).
constexpr int kNothingToDo = 1;

int check_common(const void* q, const void* k, const void* v, const void* state, const void* A_log,
                 const void* a, const void* dt_bias, const void* b, const void* output, int B, int T,
                 int H, int HV, int K, int V, long long slots) {
  if (K != kDim || V != kDim) return GDN_ERR_SHAPE;
  if (B < 0 || T < 1 || H < 1 || HV < 1 || HV % H != 0) return GDN_ERR_SHAPE;
  // grid size and 32-bit index products stay in range
  if (static_cast<long long>(B) * HV * kDim > 0x7fffffffLL) return GDN_ERR_SHAPE;
  if (static_cast<long long>(B) * T * H > 0x7fffffffLL / kDim) return GDN_ERR_SHAPE;
  if (static_cast<long long>(B) * T * HV > 0x7fffffffLL / kDim) return GDN_ERR_SHAPE;
  if (B == 0) return kNothingToDo;
  if (slots < 1) return GDN_ERR_SHAPE;
  if (!q || !k || !v || !state || !A_log || !a || !dt_bias || !b || !output) return GDN_ERR_NULL;
  if (!aligned(state, 16) || !aligned(q, 8) || !aligned(k, 8) || !aligned(v, 2) ||
      !aligned(a, 2) || !aligned(b, 2) || !aligned(output, 2) || !aligned(A_log, 4) ||
      !aligned(dt_bias, 4))
    return GDN_ERR_ALIGN;
  return GDN_OK;
}

int run(const StepArgs& p, LaunchShape shape, int TT, cudaStream_t stream) {
  if (p.B == 0) return GDN_OK;
  const bool pool = p.idx_in != nullptr, l2n = p.l2norm != 0;
  LaunchFn fn = (TT == 1) ? pick_variant<1>(shape, pool, l2n) : pick_variant<0>(shape, pool, l2n);
  if (!fn) return GDN_ERR_SHAPE;
  return fn(p, stream) == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

StepArgs make_args(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* state_in,
                   float* state_out, const float* A_log, const gdn_bf16* a, const float* dt_bias,
                   const gdn_bf16* b, double scale, gdn_bf16* output, int B, int T, int H, int HV,
                   int K, int pool, int use_qk_l2norm) {
  StepArgs p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.state_in = state_in;
  p.state_out = state_out;
  p.A_log = A_log;
  p.a = a;
  p.dt_bias = dt_bias;
  p.b = b;
  p.out = output;
  p.scale = resolve_scale(scale, K);
  p.B = B;
  p.T = T;
  p.H = H;
  p.HV = HV;
  p.pool = pool;
  p.cache_steps = T;
  p.l2norm = use_qk_l2norm ? 1 : 0;
  p.write_final = 1;
  div_constants(static_cast<uint32_t>(HV), p.hv_mul, p.hv_shift);
  div_constants(static_cast<uint32_t>(HV / H), p.hq_mul, p.hq_shift);
  return p;
}

}  // namespace

extern "C" {

int gdn_abi_version(void) { return GDN_ABI_VERSION; }

const char* gdn_strerror(int code) {
  switch (code) {
    case GDN_OK: return "ok";
    case GDN_ERR_NULL: return "a required pointer is NULL";
    case GDN_ERR_SHAPE: return "unsupported or inconsistent sizes (K and V must be 128, HV a multiple of H)";
    case GDN_ERR_ALIGN: return "misaligned pointer (state needs 16 B, q/k 8 B, fp32 vectors 4 B, bf16 2 B)";
    case GDN_ERR_LAUNCH: return "CUDA kernel launch failed";
    case GDN_ERR_ALIAS: return "state and new_state overlap without being the same buffer";
    case GDN_ERR_ARG: return "invalid argument value (rank or world out of range)";
    case GDN_ERR_LIMIT: return "beyond the fixed scratch of gdn_decode_tp_static (channel must be 0..63)";
    default: return "unknown gdn error code";
  }
}

int gdn_decode(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* state,
               const float* A_log, const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
               double scale, gdn_bf16* output, float* new_state, int B, int H, int HV, int K, int V,
               int use_qk_l2norm, void* stream) {
  const int rc = check_common(q, k, v, state, A_log, a, dt_bias, b, output, B, 1, H, HV, K, V,
                              B);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!new_state) return GDN_ERR_NULL;
  if (!aligned(new_state, 16)) return GDN_ERR_ALIGN;
  const size_t bytes = static_cast<size_t>(B) * HV * kHeadElems * sizeof(float);
  if (state != new_state && overlaps(state, bytes, new_state, bytes)) return GDN_ERR_ALIAS;
  StepArgs p = make_args(q, k, v, state, new_state, A_log, a, dt_bias, b, scale, output, B, 1, H,
                         HV, K, B, use_qk_l2norm);
  return run(p, default_shape(static_cast<long long>(B) * HV, 1), 1,
             static_cast<cudaStream_t>(stream));
}

int gdn_decode_pooled(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state_pool,
                      int pool_size, const int32_t* state_indices,
                      const int32_t* output_state_indices, const float* A_log, const gdn_bf16* a,
                      const float* dt_bias, const gdn_bf16* b, double scale, gdn_bf16* output,
                      int B, int H, int HV, int K, int V, int use_qk_l2norm,
                      int32_t* bad_index_count, void* stream) {
  const int rc = check_common(q, k, v, state_pool, A_log, a, dt_bias, b, output, B, 1, H, HV, K,
                              V, pool_size);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!state_indices) return GDN_ERR_NULL;
  if (!aligned(state_indices, 4) || !aligned(output_state_indices, 4) ||
      !aligned(bad_index_count, 4))
    return GDN_ERR_ALIGN;
  StepArgs p = make_args(q, k, v, state_pool, state_pool, A_log, a, dt_bias, b, scale, output, B,
                         1, H, HV, K, pool_size, use_qk_l2norm);
  p.idx_in = state_indices;
  p.idx_out = output_state_indices;
  p.bad_count = bad_index_count;
  return run(p, default_shape(static_cast<long long>(B) * HV, 1), 1,
             static_cast<cudaStream_t>(stream));
}

int gdn_decode_mtp(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state_pool,
                   int pool_size, const int32_t* state_indices, const float* A_log,
                   const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b, double scale,
                   gdn_bf16* output, float* intermediate_states, int cache_steps,
                   int disable_state_update, int B, int T, int H, int HV, int K, int V,
                   int use_qk_l2norm, int32_t* bad_index_count, void* stream) {
  const int rc = check_common(q, k, v, state_pool, A_log, a, dt_bias, b, output, B, T, H, HV, K,
                              V, pool_size);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!state_indices && pool_size < B) return GDN_ERR_SHAPE;
  if (intermediate_states && cache_steps < T) return GDN_ERR_SHAPE;
  if (!aligned(state_indices, 4) || !aligned(intermediate_states, 16) ||
      !aligned(bad_index_count, 4))
    return GDN_ERR_ALIGN;
  StepArgs p = make_args(q, k, v, state_pool, state_pool, A_log, a, dt_bias, b, scale, output, B,
                         T, H, HV, K, pool_size, use_qk_l2norm);
  p.idx_in = state_indices;
  p.bad_count = bad_index_count;
  p.inter = intermediate_states;
  p.cache_steps = intermediate_states ? cache_steps : T;
  p.write_final = disable_state_update ? 0 : 1;
  if (T == 1 && !intermediate_states)
    return run(p, default_shape(static_cast<long long>(B) * HV, 1), 1,
               static_cast<cudaStream_t>(stream));
  return run(p, default_shape(static_cast<long long>(B) * HV, T), 0,
             static_cast<cudaStream_t>(stream));
}

int gdn_decode_bf16_state(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                          gdn_bf16* state_pool, int pool_size, const int32_t* state_indices,
                          const int32_t* output_state_indices, const float* A_log,
                          const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
                          double scale, gdn_bf16* output, gdn_bf16* intermediate_states,
                          int cache_steps, int disable_state_update, int B, int T, int H,
                          int HV, int K, int V, int use_qk_l2norm, int32_t* bad_index_count,
                          void* stream) {
  const int rc = check_common(q, k, v, state_pool, A_log, a, dt_bias, b, output, B, T, H, HV, K,
                              V, pool_size);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!state_indices && pool_size < B) return GDN_ERR_SHAPE;
  if (output_state_indices && !state_indices) return GDN_ERR_ARG;
  if (intermediate_states && cache_steps < T) return GDN_ERR_SHAPE;
  // a bf16 chunk of q/k is 16 bytes (8 values)
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(intermediate_states, 16) ||
      !aligned(state_indices, 4) || !aligned(output_state_indices, 4) ||
      !aligned(bad_index_count, 4))
    return GDN_ERR_ALIGN;
  StepArgs p = make_args(q, k, v, nullptr, nullptr, A_log, a, dt_bias, b, scale, output, B, T, H,
                         HV, K, pool_size, use_qk_l2norm);
  p.state_in = state_pool;
  p.state_out = state_pool;
  p.idx_in = state_indices;
  p.idx_out = output_state_indices;
  p.bad_count = bad_index_count;
  p.inter = intermediate_states;
  p.cache_steps = intermediate_states ? cache_steps : T;
  p.write_final = disable_state_update ? 0 : 1;
  const int TT = (T == 1 && !intermediate_states) ? 1 : 0;
  // A bf16 row is half the bytes of an fp32 row, so at large batch each lane keeps
  // four rows in flight (16 lanes per row, 2-warp CTAs): B = 256, 16/32 heads,
  // 86 us vs 103 us for the fp32 default shape (CUPTI sweep of 7 shapes).
  LaunchShape shape = default_shape(static_cast<long long>(B) * HV, TT == 1 ? 1 : T);
  if (TT == 1 && static_cast<long long>(B) * HV > 512) shape = LaunchShape{16, 4, 2};
  const bool pool = state_indices != nullptr, l2n = p.l2norm != 0;
  LaunchFn fn = (TT == 1) ? pick_bf16_variant<1>(shape, pool, l2n)
                          : pick_bf16_variant<0>(shape, pool, l2n);
  if (!fn) return GDN_ERR_SHAPE;
  return fn(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_decode_tuned(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state_pool,
                     int pool_size, const int32_t* state_indices, const float* A_log,
                     const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b, double scale,
                     gdn_bf16* output, int B, int T, int H, int HV, int K, int V,
                     int use_qk_l2norm, int lanes_per_row, int rows_per_lane, int warps_per_cta,
                     void* stream) {
  const int rc = check_common(q, k, v, state_pool, A_log, a, dt_bias, b, output, B, T, H, HV, K,
                              V, pool_size);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!state_indices && pool_size < B) return GDN_ERR_SHAPE;
  if (!aligned(state_indices, 4)) return GDN_ERR_ALIGN;
  StepArgs p = make_args(q, k, v, state_pool, state_pool, A_log, a, dt_bias, b, scale, output, B,
                         T, H, HV, K, pool_size, use_qk_l2norm);
  p.idx_in = state_indices;
  LaunchShape s = default_shape(static_cast<long long>(B) * HV, T);
  if (lanes_per_row > 0) s.lpr = lanes_per_row;
  if (rows_per_lane > 0) s.rg = rows_per_lane;
  if (warps_per_cta > 0) s.warps = warps_per_cta;
  return run(p, s, T == 1 ? 1 : 0, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {

int tp_step(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state,
            const float* A_log, const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
            double scale, gdn_bf16* const* peer_outputs, uint32_t* const* peer_signals,
            uint32_t* epoch_counter, int32_t* status, uint32_t timeout_us, int rank, int world,
            int B, int H, int HV, int K, int V, int use_qk_l2norm, int chained, void* stream) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return GDN_ERR_ARG;
  if (static_cast<long long>(HV) * world > 0x7fffffffLL / kDim) return GDN_ERR_SHAPE;
  // this rank's own output buffer is the one its outputs (and the checks) refer to
  const gdn_bf16* own_out = peer_outputs ? peer_outputs[rank] : nullptr;
  const int rc = check_common(q, k, v, state, A_log, a, dt_bias, b, own_out, B, 1, H,
                              HV * world, K, V, B);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!peer_signals || !status || !epoch_counter) return GDN_ERR_NULL;
  if (!aligned(status, 4) || !aligned(epoch_counter, 4)) return GDN_ERR_ALIGN;
  const size_t state_bytes = static_cast<size_t>(B) * HV * kHeadElems * sizeof(float);
  const size_t out_bytes = static_cast<size_t>(B) * HV * world * kDim * sizeof(gdn_bf16);
  if (overlaps(state, state_bytes, own_out, out_bytes)) return GDN_ERR_ALIAS;
  StepArgs p = make_args(q, k, v, state, state, A_log, a, dt_bias, b, scale, nullptr, B, 1, H, HV,
                         K, B, use_qk_l2norm);
  BarrierArgs bar{};
  for (int r = 0; r < world; ++r) {
    if (!peer_outputs[r] || !peer_signals[r]) return GDN_ERR_NULL;
    if (!aligned(peer_outputs[r], 16) || !aligned(peer_signals[r], 4)) return GDN_ERR_ALIGN;
    p.peer_out[r] = peer_outputs[r];
    bar.peer_sig[r] = peer_signals[r];
  }
  p.out = peer_outputs[rank];
  p.world = world;
  p.hv0 = rank * HV;
  p.hv_total = HV * world;
  p.chained = chained ? 1 : 0;
  bar.status = status;
  bar.epoch = epoch_counter;
  bar.timeout_ns = 1000ull * (timeout_us ? timeout_us : 1000000u);
  bar.rank = rank;
  bar.world = world;
  LaunchFn fn = pick_scatter(default_shape(static_cast<long long>(B) * HV, 1), p.l2norm != 0);
  if (!fn) return GDN_ERR_SHAPE;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fn(p, st) != cudaSuccess) return GDN_ERR_LAUNCH;
  // the barrier: a programmatic dependent of the decode grid (it waits for that grid)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tp_barrier_kernel, bar) == cudaSuccess ? GDN_OK
                                                                           : GDN_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int gdn_decode_tp(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state,
                  const float* A_log, const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
                  double scale, gdn_bf16* const* peer_outputs, uint32_t* const* peer_signals,
                  uint32_t* epoch_counter, int32_t* status, uint32_t timeout_us, int rank,
                  int world, int B, int H, int HV, int K, int V, int use_qk_l2norm,
                  void* stream) {
  return tp_step(q, k, v, state, A_log, a, dt_bias, b, scale, peer_outputs, peer_signals,
                 epoch_counter, status, timeout_us, rank, world, B, H, HV, K, V, use_qk_l2norm,
                 0, stream);
}

int gdn_decode_tp_chained(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state,
                          const float* A_log, const gdn_bf16* a, const float* dt_bias,
                          const gdn_bf16* b, double scale, gdn_bf16* const* peer_outputs,
                          uint32_t* const* peer_signals, uint32_t* epoch_counter,
                          int32_t* status, uint32_t timeout_us, int rank, int world, int B, int H,
                          int HV, int K, int V, int use_qk_l2norm, void* stream) {
  return tp_step(q, k, v, state, A_log, a, dt_bias, b, scale, peer_outputs, peer_signals,
                 epoch_counter, status, timeout_us, rank, world, B, H, HV, K, V, use_qk_l2norm,
                 1, stream);
}

}  // extern "C"

// ---- allocation-free tensor-parallel step --------------------------------------
//
// Callers that cannot allocate device memory where they run a decode step (a
// serving runtime that reserves all of HBM for its own pool at start-up, code that
// runs while a CUDA graph is being captured, a plain-C host with no allocator of its
// own) still have to give gdn_decode_tp an epoch counter.  gdn_decode_tp_static
// keeps those counters in a fixed array inside this library instead: one uint32 per
// "channel", kStaticChannels channels, resident on every GPU that loads the library
// until the process exits.
namespace {

constexpr int kStaticChannels = 64;
constexpr int kMaxDevices = 64;

// Epoch counters of gdn_decode_tp_static, one per channel (zero when the library is
// loaded).  Host code only ever sees a stand-in for this name: its device address
// comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) uint32_t g_tp_static_epochs[kStaticChannels];

std::mutex g_static_mutex;
uint32_t* g_static_epochs_dev[kMaxDevices];  // device address per device, null until set up

// Device address of g_tp_static_epochs on the current device, looked up (with that
// device current) on the first call for the device and cached for the life of the
// process (a cudaDeviceReset unloads the module; the header forbids use after one).
int static_epochs(uint32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return GDN_ERR_LIMIT;
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (g_static_epochs_dev[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_tp_static_epochs) != cudaSuccess) return GDN_ERR_LAUNCH;
    g_static_epochs_dev[dev] = static_cast<uint32_t*>(ptr);
  }
  *out = g_static_epochs_dev[dev];
  return GDN_OK;
}

}  // namespace

extern "C" {

int gdn_decode_tp_static(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state,
                         const float* A_log, const gdn_bf16* a, const float* dt_bias,
                         const gdn_bf16* b, double scale, gdn_bf16* const* peer_outputs,
                         uint32_t* const* peer_signals, int32_t* status, uint32_t timeout_us,
                         int channel, int rank, int world, int B, int H, int HV, int K, int V,
                         int use_qk_l2norm, void* stream) {
  if (channel < 0 || channel >= kStaticChannels) return GDN_ERR_LIMIT;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return GDN_ERR_ARG;
  if (!peer_outputs || !peer_signals || !status) return GDN_ERR_NULL;
  uint32_t* epochs = nullptr;
  const int rc = static_epochs(&epochs);
  if (rc != GDN_OK) return rc;
  return gdn_decode_tp(q, k, v, state, A_log, a, dt_bias, b, scale, peer_outputs, peer_signals,
                       epochs + channel, status, timeout_us, rank, world, B, H, HV, K, V,
                       use_qk_l2norm, stream);
}

int gdn_decode_gated_norm(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, float* state,
                          const float* A_log, const gdn_bf16* a, const float* dt_bias,
                          const gdn_bf16* b, double scale, const gdn_bf16* z,
                          const gdn_bf16* norm_weight, double eps, gdn_bf16* output, int B, int H,
                          int HV, int K, int V, int use_qk_l2norm, void* stream) {
  const int rc = check_common(q, k, v, state, A_log, a, dt_bias, b, output, B, 1, H, HV, K, V, B);
  if (rc == kNothingToDo) return GDN_OK;
  if (rc != GDN_OK) return rc;
  if (!z || !norm_weight) return GDN_ERR_NULL;
  if (!aligned(z, 2) || !aligned(norm_weight, 2)) return GDN_ERR_ALIGN;
  if (!(eps >= 0.0)) return GDN_ERR_ARG;
  StepArgs p = make_args(q, k, v, state, state, A_log, a, dt_bias, b, scale, output, B, 1, H, HV,
                         K, B, use_qk_l2norm);
  p.z = z;
  p.norm_w = norm_weight;
  p.eps = static_cast<float>(eps);
  const cudaError_t e = p.l2norm ? launch_gated_norm<true>(p, static_cast<cudaStream_t>(stream))
                                 : launch_gated_norm<false>(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_prefill_tuned(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* state,
                      const float* A_log, const gdn_bf16* a, const float* dt_bias,
                      const gdn_bf16* b, const int32_t* cu_seqlens, double scale,
                      gdn_bf16* output, float* new_state, int num_seqs, int total_tokens, int H,
                      int HV, int K, int V, int use_qk_l2norm, int lanes_per_row,
                      int rows_per_lane, int warps_per_cta, void* stream) {
  if (K != kDim || V != kDim) return GDN_ERR_SHAPE;
  if (num_seqs < 0 || total_tokens < 0 || H < 1 || HV < 1 || HV % H != 0) return GDN_ERR_SHAPE;
  if (static_cast<long long>(num_seqs) * HV * kDim > 0x7fffffffLL) return GDN_ERR_SHAPE;
  if (static_cast<long long>(total_tokens) * H > 0x7fffffffLL / kDim) return GDN_ERR_SHAPE;
  if (static_cast<long long>(total_tokens) * HV > 0x7fffffffLL / kDim) return GDN_ERR_SHAPE;
  if (num_seqs == 0) return GDN_OK;
  if (!cu_seqlens || !new_state || !A_log || !dt_bias) return GDN_ERR_NULL;
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !output)) return GDN_ERR_NULL;
  if (!aligned(new_state, 16) || !aligned(state, 16) || !aligned(q, 8) || !aligned(k, 8) ||
      !aligned(v, 2) || !aligned(a, 2) || !aligned(b, 2) || !aligned(output, 2) ||
      !aligned(A_log, 4) || !aligned(dt_bias, 4) || !aligned(cu_seqlens, 4))
    return GDN_ERR_ALIGN;
  const size_t bytes = static_cast<size_t>(num_seqs) * HV * kHeadElems * sizeof(float);
  if (state && state != new_state && overlaps(state, bytes, new_state, bytes)) return GDN_ERR_ALIAS;
  StepArgs p = make_args(q, k, v, state, new_state, A_log, a, dt_bias, b, scale, output, num_seqs,
                         1, H, HV, K, num_seqs, use_qk_l2norm);
  p.cu = cu_seqlens;
  p.total = total_tokens;
  LaunchShape s = prefill_shape(static_cast<long long>(num_seqs) * HV);
  if (lanes_per_row > 0) s.lpr = lanes_per_row;
  if (rows_per_lane > 0) s.rg = rows_per_lane;
  if (warps_per_cta > 0) s.warps = warps_per_cta;
  LaunchFn fn = pick_prefill(s, p.l2norm != 0);
  if (!fn) return GDN_ERR_SHAPE;
  return fn(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int gdn_prefill_ws(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* state,
                   const float* A_log, const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
                   const int32_t* cu_seqlens, double scale, gdn_bf16* output, float* new_state,
                   void* workspace, size_t workspace_bytes, int num_seqs, int total_tokens, int H,
                   int HV, int K, int V, int use_qk_l2norm, void* stream) {
  // Sequences of 32 tokens or more on average go to the chunked tensor-core path (one
  // chunk costs about what 15-25 dependent token updates cost in the register-resident
  // loop); shorter ones, the q/k L2-norm option and inputs without 16-byte alignment stay
  // on the token loop.  Among the chunked forms, sequences of 256 tokens or more on
  // average (4+ chunks) take the two-launch form when a workspace is given (its parallel
  // first launch pays off once each sequence has several chunks; B200 timings at 16/32
  // heads: 64 x 64 tokens 224 us one-launch vs 281 us two-launch, 16 x 256 tokens
  // 177 vs 175 us, 2 x 2048 tokens 301 vs 182 us).  All compute the same recurrence.
  if (!use_qk_l2norm && num_seqs > 0 && total_tokens >= 32LL * num_seqs &&
      aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(output, 16)) {
    if (total_tokens >= 256LL * num_seqs && workspace != nullptr && aligned(workspace, 16) &&
        workspace_bytes >= gdn_prefill_workspace_bytes(num_seqs, total_tokens, HV))
      return gdn_prefill_wy(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                            new_state, nullptr, workspace, workspace_bytes, num_seqs,
                            total_tokens, H, HV, K, V, stream);
    return gdn_prefill_chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                               new_state, nullptr, num_seqs, total_tokens, H, HV, K, V, stream);
  }
  return gdn_prefill_tuned(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                           new_state, num_seqs, total_tokens, H, HV, K, V, use_qk_l2norm, 0, 0, 0,
                           stream);
}

int gdn_prefill(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v, const float* state,
                const float* A_log, const gdn_bf16* a, const float* dt_bias, const gdn_bf16* b,
                const int32_t* cu_seqlens, double scale, gdn_bf16* output, float* new_state,
                int num_seqs, int total_tokens, int H, int HV, int K, int V, int use_qk_l2norm,
                void* stream) {
  const bool chunked = !use_qk_l2norm && num_seqs > 0 && total_tokens >= 256LL * num_seqs &&
                       H >= 1 && HV >= 1 && aligned(q, 16) && aligned(k, 16) && aligned(v, 16) &&
                       aligned(output, 16);
  const size_t need = chunked ? gdn_prefill_workspace_bytes(num_seqs, total_tokens, HV) : 0;
  if (need > 0) {
    // stream-ordered workspace (capturable; freed after the launches that use it)
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* ws = nullptr;
    if (cudaMallocAsync(&ws, need, st) == cudaSuccess) {
      const int rc = gdn_prefill_ws(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
                                    output, new_state, ws, need, num_seqs, total_tokens, H, HV,
                                    K, V, use_qk_l2norm, stream);
      const cudaError_t fe = cudaFreeAsync(ws, st);
      return (rc == GDN_OK && fe != cudaSuccess) ? GDN_ERR_LAUNCH : rc;
    }
    (void)cudaGetLastError();   // clear the failed allocation; run without a workspace
  }
  return gdn_prefill_ws(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                        new_state, nullptr, 0, num_seqs, total_tokens, H, HV, K, V,
                        use_qk_l2norm, stream);
}

int gdn_interleave_heads(const gdn_bf16* gathered, gdn_bf16* output, int world, int rows, int HVl,
                         int V, void* stream) {
  if (!gathered || !output) return GDN_ERR_NULL;
  if (world < 1 || rows < 0 || HVl < 1 || V < 4 || V % 4 != 0) return GDN_ERR_SHAPE;
  if (!aligned(gathered, 8) || !aligned(output, 8)) return GDN_ERR_ALIGN;
  const size_t n = static_cast<size_t>(world) * rows * HVl * V;
  if (overlaps(gathered, n * 2, output, n * 2)) return GDN_ERR_ALIAS;
  if (rows == 0) return GDN_OK;
  const size_t words = n / 4;
  const int threads = 256;
  size_t blocks = (words + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  interleave_heads_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                            static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint2*>(gathered), reinterpret_cast<uint2*>(output), world, rows, HVl,
      V / 4);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // extern "C"
