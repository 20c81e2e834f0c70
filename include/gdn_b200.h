/*
 * gdn_b200.h — C ABI of the B200 (sm_100a) Gated DeltaNet decode library.
 *
 * One library, libgdn_b200.so, holds every kernel of the GDN decode path:
 * the fused T=1 decode step, the pooled-state (continuous batching) step,
 * the multi-token (speculative verify) step, the bf16-state variant, the
 * tensor-parallel step that stores its outputs into every rank's buffer
 * over NVLink, and the head interleave used after an NCCL all-gather.  No
 * function here allocates memory: the caller owns every buffer.  No
 * function synchronises the host: work is enqueued on the given stream
 * (NULL = the legacy default stream).
 *
 * Data layout (all tensors contiguous, row-major):
 *   q, k        [B, T, H,  K]   bf16
 *   v           [B, T, HV, V]   bf16
 *   a, b        [B, T, HV]      bf16   (decay input, update-gate input)
 *   A_log       [HV]            fp32
 *   dt_bias     [HV]            fp32
 *   state       [S, HV, V, K]   fp32   "k-last": K is the contiguous axis
 *                                      (bf16 in gdn_decode_bf16_state)
 *   output      [B, T, HV, V]   bf16
 * with K == V == 128, HV % H == 0 (v-head hv reads q/k head hv / (HV/H)).
 *
 * Per (batch, v-head) and token, with x = a + dt_bias:
 *   g    = exp(-exp(A_log) * softplus(x))   softplus(x) = x if x > 20
 *   beta = sigmoid(b)
 *   S    = g * S + k (beta * (v - k.(g S)))^T     (delta rule, rank 1)
 *   o    = scale * S^T q
 * Optional q/k L2 normalisation: x * rsqrt(sum(x^2) + 1e-6).
 *
 * Return value: GDN_OK (0) or a negative GDN_ERR_* code.  Argument errors
 * are detected before anything is enqueued; GDN_ERR_LAUNCH reports a
 * failed kernel launch (cudaGetLastError after the launch).
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bf16 values travel as their 16-bit pattern. */
typedef uint16_t gdn_bf16;

/* Exported symbols stay visible when the library is built with
 * -fvisibility=hidden. */
#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#define GDN_OK 0
#define GDN_ERR_NULL (-1)        /* a required pointer is NULL            */
#define GDN_ERR_SHAPE (-2)       /* unsupported or inconsistent sizes     */
#define GDN_ERR_ALIGN (-3)       /* a pointer is not suitably aligned     */
#define GDN_ERR_LAUNCH (-4)      /* the CUDA launch failed                */
#define GDN_ERR_ALIAS (-5)       /* in/out buffers overlap illegally      */
#define GDN_ERR_ARG (-6)         /* invalid argument value                */
#define GDN_ERR_LIMIT (-7)       /* beyond a fixed, built-in maximum      */

#define GDN_ABI_VERSION 1

/* Version of this ABI (GDN_ABI_VERSION of the build). */
GDN_API int gdn_abi_version(void);

/* Human-readable text for a GDN_* return code (static storage). */
GDN_API const char* gdn_strerror(int code);

/*
 * Fused T=1 decode step, destination-passing form.
 *
 * Replaces the reference's TVM-FFI exports `kernel_cuda` / `kernel_cuda_v4`
 * (solution/cuda/kernel.cu:216-254 and :405-443, bound in Python by
 * solution/cuda/binding.py:35-60) and the Triton entry `kernel_fla_recurrent`
 * (solution/triton/kernel.py:150-197): same tensors, same argument order.
 * `state` is read, `new_state` is written; they may be the same buffer
 * (in-place update, the usual case) or fully disjoint.  scale == 0 selects
 * 1/sqrt(K) (solution/cuda/binding.py:38-41).  `use_qk_l2norm` != 0 also
 * L2-normalises q and k (the reference path passes False).
 * Sizes: state/new_state hold B slots, T == 1.
 */
GDN_API int gdn_decode(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
               const float* state, const float* A_log, const gdn_bf16* a,
               const float* dt_bias, const gdn_bf16* b, double scale,
               gdn_bf16* output, float* new_state,
               int B, int H, int HV, int K, int V,
               int use_qk_l2norm, void* stream);

/*
 * Pooled-state T=1 decode (continuous batching), updating the pool in place.
 *
 * Replaces the float32 pool path of FlashInfer's
 * gated_delta_rule_decode_pretranspose(initial_state=..., initial_state_indices=...,
 * output_state_indices=...) (flashinfer/gdn_decode.py:118-195, kernel side
 * flashinfer/gdn_kernels/gdn_decode_pretranspose.py:136-160), which the
 * reference calls from kernel_fi_baseline (solution/triton/kernel.py:124-147).
 * Batch entry i reads slot state_indices[i] of `state_pool` [pool_size,HV,V,K].
 *  - state_indices[i] < 0: entry skipped, pool untouched, output rows zero.
 *  - state_indices[i] >= pool_size: treated like -1 and counted in
 *    *bad_index_count (device int32, may be NULL) so a caller can detect it.
 *  - output_state_indices (may be NULL = same slot): the updated state is
 *    written to slot output_state_indices[i]; a negative value redirects the
 *    write to slot 0 (FlashInfer's null-buffer convention); a value >=
 *    pool_size skips the write and is counted in *bad_index_count.
 * Active read slots must be distinct, and so must active write slots: two
 * entries sharing a slot race.
 */
GDN_API int gdn_decode_pooled(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                      float* state_pool, int pool_size,
                      const int32_t* state_indices,
                      const int32_t* output_state_indices,
                      const float* A_log, const gdn_bf16* a,
                      const float* dt_bias, const gdn_bf16* b, double scale,
                      gdn_bf16* output, int B, int H, int HV, int K, int V,
                      int use_qk_l2norm, int32_t* bad_index_count,
                      void* stream);

/*
 * Multi-token (T >= 1) sequential decode for speculative verification.
 *
 * Replaces FlashInfer's gated_delta_rule_mtp (flashinfer/gdn_decode.py:557-700);
 * the per-token recurrence is the reference's kernel_prefill_reference inner
 * loop (solution/triton/prefill_kernel.py:142-181) applied to T tokens.
 * Entry i starts from slot s = state_indices ? state_indices[i] : i of
 * `state_pool` [pool_size,HV,V,K] and runs tokens t = 0..T-1 of q/k/v/a/b
 * ([B,T,...]).  After token t the state is written to
 * intermediate_states[i, t] ([B, cache_steps, HV, V, K], cache_steps >= T,
 * indexed by batch entry like FlashInfer's kernel,
 * flashinfer/gdn_kernels/gdn_decode_mtp.py:645) when that pointer is
 * non-NULL.  Unless disable_state_update != 0 the final state is written
 * back to slot s.  Slots < 0 (or >= pool_size, counted in *bad_index_count)
 * are skipped with zero outputs and untouched intermediates.
 */
GDN_API int gdn_decode_mtp(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                   float* state_pool, int pool_size,
                   const int32_t* state_indices,
                   const float* A_log, const gdn_bf16* a,
                   const float* dt_bias, const gdn_bf16* b, double scale,
                   gdn_bf16* output, float* intermediate_states,
                   int cache_steps, int disable_state_update,
                   int B, int T, int H, int HV, int K, int V,
                   int use_qk_l2norm, int32_t* bad_index_count,
                   void* stream);

/*
 * Decode with the state stored in bf16 (T >= 1, optional pool), updated in place.
 *
 * Replaces the bf16-state backend of FlashInfer's k-last decode, which
 * gated_delta_rule_decode_pretranspose selects for a bf16 state with K = V = 128
 * (flashinfer/gdn_decode.py:255-261; kernels in
 * flashinfer/gdn_kernels/gdn_decode_bf16_state.py, T = 1 and multi-token, with
 * split read/write pool slots at :124-172).  The reference's own decode keeps
 * an fp32 state; this variant halves the state bytes, which dominate the traffic.
 * Arithmetic is fp32 as in the other entries: the state is widened on load,
 * and rounded to bf16 (nearest even) only when stored.
 *  - state_pool [pool_size, HV, V, K] bf16; entry i uses slot
 *    state_indices[i] (NULL: slot i, pool_size >= B), writes slot
 *    output_state_indices[i] if given (NULL: the read slot; requires
 *    state_indices).  Index rules as gdn_decode_pooled: a negative read index
 *    skips the entry with zero outputs (FlashInfer's bf16 backend instead
 *    redirects it to a reserved slot 0 and leaves the output undefined; callers
 *    that reserve slot 0 see no difference), out-of-range indices are skipped
 *    and counted in *bad_index_count.
 *  - T tokens run in order per entry; intermediate_states [B, cache_steps, HV,
 *    V, K] bf16 (may be NULL) receives the state after each token; the final
 *    state is written back unless disable_state_update != 0.
 *  - q and k must be 16-byte aligned (16-byte chunks of 8 values are loaded).
 */
GDN_API int gdn_decode_bf16_state(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                                  gdn_bf16* state_pool, int pool_size,
                                  const int32_t* state_indices,
                                  const int32_t* output_state_indices,
                                  const float* A_log, const gdn_bf16* a,
                                  const float* dt_bias, const gdn_bf16* b, double scale,
                                  gdn_bf16* output, gdn_bf16* intermediate_states,
                                  int cache_steps, int disable_state_update,
                                  int B, int T, int H, int HV, int K, int V,
                                  int use_qk_l2norm, int32_t* bad_index_count,
                                  void* stream);

/*
 * Launch-shape tuning entry (no counterpart in the reference, whose launch
 * shapes are fixed: solution/cuda/kernel.cu:234-235, :423-424).  Same step
 * as gdn_decode_mtp without intermediates (T == 1: gdn_decode_pooled with
 * state_indices, or gdn_decode in place when state_indices is NULL), with
 * an explicit work split: lanes_per_row in {8,16,32} lanes share one 512-byte
 * state row, rows_per_lane in {1,2,4}, warps_per_cta in {1,2,4,8}; 0 keeps
 * the library's default for that field.  With state_indices or use_qk_l2norm
 * only the default shapes (8/1/4 and 8/4/1) are built; any other shape returns
 * GDN_ERR_SHAPE.  Used by the benchmark's sweeps.
 */
GDN_API int gdn_decode_tuned(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                     float* state_pool, int pool_size,
                     const int32_t* state_indices,
                     const float* A_log, const gdn_bf16* a,
                     const float* dt_bias, const gdn_bf16* b, double scale,
                     gdn_bf16* output, int B, int T, int H, int HV, int K,
                     int V, int use_qk_l2norm, int lanes_per_row,
                     int rows_per_lane, int warps_per_cta, void* stream);

/*
 * Fused T=1 decode step plus the decode layer's gated RMSNorm, state in place.
 *
 * The decode step of gdn_decode (state [B, HV, V, K] updated in place; the
 * reference's step, solution/triton/kernel.py:95-114) followed, inside the same
 * kernel, by the gated RMSNorm that Qwen3-Next applies to the step's output
 * before the output projection (the layer the reference's contest shapes come
 * from, CLAUDE.md:67-84; transformers models/qwen3_next/modeling_qwen3_next.py:73-82
 * and :693-697), per (batch entry, v-head) over the V = 128 outputs o (bf16):
 *   x   = bf16(o * rsqrt(mean(o^2) + eps))
 *   y   = bf16(norm_weight * x)
 *   out = bf16(y * silu(z))
 * z [B, 1, HV, V] bf16 is the layer's gate projection, norm_weight [V] bf16.
 * `output` [B, 1, HV, V] receives the normalised values (the raw o is not
 * stored).  One CTA holds a whole head, so the norm needs no second kernel.
 * eps must be >= 0 (GDN_ERR_ARG otherwise).
 */
GDN_API int gdn_decode_gated_norm(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                                  float* state, const float* A_log, const gdn_bf16* a,
                                  const float* dt_bias, const gdn_bf16* b, double scale,
                                  const gdn_bf16* z, const gdn_bf16* norm_weight, double eps,
                                  gdn_bf16* output, int B, int H, int HV, int K, int V,
                                  int use_qk_l2norm, void* stream);

/*
 * Variable-length prefill (a batch of prompts of different lengths).
 *
 * Replaces the reference's prefill entries for gdn_prefill_qk4_v8_d128_k_last:
 * the destination-passing kernel_prefill_fla_chunk / kernel_prefill_fi_baseline
 * (solution/triton/prefill_kernel.py:11-54, :57-83) with the semantics of
 * kernel_prefill_reference (:85-183).  Flat token-major inputs:
 *   q, k [total_tokens, H, K], v [total_tokens, HV, V], a, b [total_tokens, HV]
 *   cu_seqlens [num_seqs + 1] int32: sequence s owns tokens cu[s] .. cu[s+1]-1
 *   state [num_seqs, HV, V, K] fp32 initial states, or NULL for zeros
 *   output [total_tokens, HV, V] bf16, new_state [num_seqs, HV, V, K] fp32
 * Each sequence runs its tokens in order through the decode recurrence.  When
 * the sequences average 32 tokens or more (and q, k, v, output are 16-byte
 * aligned, use_qk_l2norm == 0) the call runs the chunked tensor-core form of the
 * same recurrence: gdn_prefill_wy (two launches) for 256 tokens or more on
 * average, with a workspace it allocates stream-ordered (cudaMallocAsync /
 * cudaFreeAsync on `stream`; if that allocation fails, gdn_prefill_chunked), else
 * the one-launch gdn_prefill_chunked.  Shorter sequences run a token loop whose
 * state stays in registers for the whole sequence (read once, written once).
 * gdn_prefill_ws takes the workspace from the caller instead.
 * A sequence with no tokens gets a zero final state (the reference's
 * zero-initialised new_state).  Sequence bounds are clamped to
 * [0, total_tokens] on the device, so malformed offsets cannot address memory
 * outside the inputs.  `state` and `new_state` may be the same buffer or
 * disjoint.  scale == 0 selects 1/sqrt(K).
 */
GDN_API int gdn_prefill(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                        const float* state, const float* A_log, const gdn_bf16* a,
                        const float* dt_bias, const gdn_bf16* b,
                        const int32_t* cu_seqlens, double scale,
                        gdn_bf16* output, float* new_state,
                        int num_seqs, int total_tokens, int H, int HV, int K, int V,
                        int use_qk_l2norm, void* stream);

/*
 * gdn_prefill with a caller-provided device workspace (no allocation): sequences of
 * 256 tokens or more on average use gdn_prefill_wy when `workspace_bytes` >=
 * gdn_prefill_workspace_bytes(num_seqs, total_tokens, HV), the other chunked cases
 * gdn_prefill_chunked; the token loop uses none (workspace may then be NULL).  `workspace` must be 16-byte aligned.  Same
 * reference interface as gdn_prefill.
 */
GDN_API int gdn_prefill_ws(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                           const float* state, const float* A_log, const gdn_bf16* a,
                           const float* dt_bias, const gdn_bf16* b,
                           const int32_t* cu_seqlens, double scale,
                           gdn_bf16* output, float* new_state, void* workspace,
                           size_t workspace_bytes, int num_seqs, int total_tokens, int H,
                           int HV, int K, int V, int use_qk_l2norm, void* stream);

/*
 * Device workspace bytes gdn_prefill_wy needs: (num_seqs + ceil(total_tokens / 64))
 * chunk slots of HV records of 104 KB (0 for invalid sizes).  No counterpart in the
 * reference.
 */
GDN_API size_t gdn_prefill_workspace_bytes(int num_seqs, int total_tokens, int HV);

/*
 * Variable-length prefill by chunks of 64 tokens in two launches (tcgen05).
 *
 * Same operation, arguments and results as gdn_prefill (the reference's prefill
 * entries, solution/triton/prefill_kernel.py:11-83, with kernel_prefill_reference's
 * semantics, :85-183), in the chunked (WY) form of gdn_prefill_chunked, split where
 * the algebra allows: the first launch computes every chunk's state-independent
 * products (the triangular solve and the U, W and masked Q K^T tiles) for all chunks of
 * all sequences at once, one CTA per (chunk, v-head), into `workspace`; the second
 * runs each (sequence, v-head)'s chain of state-dependent products with the state in
 * tensor memory.  A long single prompt thus spreads its chunk-local work over the
 * whole GPU.  q, k, v, the output, the states and the workspace must be 16-byte
 * aligned; workspace_bytes >= gdn_prefill_workspace_bytes(num_seqs, total_tokens, HV).
 * Sequences must not overlap (non-decreasing cu_seqlens, as the reference assumes):
 * the chunks of overlapping sequences may share workspace records, which keeps every
 * access inside the workspace but leaves their results unspecified.  `status` as in
 * gdn_prefill_chunked.
 */
GDN_API int gdn_prefill_wy(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                           const float* state, const float* A_log, const gdn_bf16* a,
                           const float* dt_bias, const gdn_bf16* b,
                           const int32_t* cu_seqlens, double scale,
                           gdn_bf16* output, float* new_state, int32_t* status,
                           void* workspace, size_t workspace_bytes,
                           int num_seqs, int total_tokens, int H, int HV, int K, int V,
                           void* stream);

/*
 * Variable-length prefill by chunks of 64 tokens on the tensor cores (tcgen05), in
 * one launch and without a workspace.
 *
 * Same operation, arguments and results as gdn_prefill (the reference's prefill
 * entries, solution/triton/prefill_kernel.py:11-83, with kernel_prefill_reference's
 * semantics, :85-183), computed in the chunked (WY) form of the delta rule that the
 * reference's own prefill path uses (solution/triton/fla_prefill_code.py): per chunk
 * of 64 tokens a handful of matrix products (bf16 for the chunk's own q/k/v, tf32
 * against the fp32 state, fp32 accumulation) replace 64 dependent rank-1 updates.
 * One CTA per (sequence, v-head), state resident in tensor memory; q, k, v, the
 * output and the states must be 16-byte aligned.  Results agree with the token loop to within the
 * accuracy of the split-bf16 / tf32 products (about 1e-4 relative on the state),
 * not bit for bit.  `status` (device int32, may be NULL, never cleared here) is set
 * to 1 if a bounded wait for the tensor cores or a TMA load timed out.
 */
GDN_API int gdn_prefill_chunked(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                                const float* state, const float* A_log, const gdn_bf16* a,
                                const float* dt_bias, const gdn_bf16* b,
                                const int32_t* cu_seqlens, double scale,
                                gdn_bf16* output, float* new_state, int32_t* status,
                                int num_seqs, int total_tokens, int H, int HV, int K, int V,
                                void* stream);

/*
 * gdn_prefill with an explicit work split (no counterpart in the reference;
 * used by the benchmark's sweeps): lanes_per_row / rows_per_lane / warps_per_cta
 * among the built splits 8/1/1, 8/2/1, 8/4/1, 8/1/4, 16/1/1 (0 keeps the
 * default field); other splits return GDN_ERR_SHAPE.
 */
GDN_API int gdn_prefill_tuned(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                              const float* state, const float* A_log, const gdn_bf16* a,
                              const float* dt_bias, const gdn_bf16* b,
                              const int32_t* cu_seqlens, double scale,
                              gdn_bf16* output, float* new_state,
                              int num_seqs, int total_tokens, int H, int HV, int K, int V,
                              int use_qk_l2norm, int lanes_per_row, int rows_per_lane,
                              int warps_per_cta, void* stream);

/*
 * Tensor-parallel T=1 decode step with the output all-gather fused in.
 *
 * No counterpart in the reference (it runs on one GPU; its qk4/v8 contest shape
 * is itself a 4-way head split of Qwen3-Next).  Rank `rank` of `world` (<= 8)
 * holds H q/k heads, HV v-heads (v-heads [rank*HV, (rank+1)*HV) of world*HV),
 * their A_log/dt_bias/a/b and its own state [B, HV, V, K], updated in place.
 * The decode kernel stores each output row straight into every rank's output
 * buffer peer_outputs[r] ([B, 1, world*HV, V] bf16, rank r's buffer mapped into
 * this process, e.g. by CUDA IPC or symmetric memory) at this rank's head
 * offset, overlapping the NVLink traffic with the math; a one-CTA barrier
 * kernel enqueued after it (launched as a programmatic dependent of the decode
 * grid, it waits for that grid to complete) then synchronises the ranks through
 * signal words:
 * peer_signals[r] points to `world` uint32 words on rank r (zero before the
 * first call); this rank writes the step's epoch into word `rank` of every
 * rank's array and waits until all `world` words of its own array reach it.
 * When the barrier kernel has finished, peer_outputs[rank] holds all
 * world*HV heads.
 *  - epoch_counter: one uint32 in this GPU's memory, zero before the first
 *    call; the barrier kernel reads it, uses value+1 as the step's epoch and
 *    stores that back (wrapping past 2^32 is handled).  Because no per-call
 *    value is passed, the two kernels can be captured in a CUDA graph and
 *    replayed.
 *  - status: int32 in device memory; set to 1 (never cleared by the library)
 *    if the wait for some rank exceeded timeout_us (0 = 1 s); the barrier then
 *    returns instead of waiting forever, and that output is incomplete.
 *  - Two consecutive calls must not write the same output buffers (a fast rank
 *    could overwrite rows a slow rank is still reading): alternate two buffers.
 *    With two buffers the output of call n is valid only until this rank
 *    enqueues call n+1: another rank's call n+2 writes the same buffer as soon
 *    as this rank's barrier n+1 has signalled, so work that reads output n
 *    must be enqueued on `stream` before call n+1 (or copy it out first).
 * Every rank must make the same sequence of calls with the same B, H, HV and
 * world.  Enqueues two kernels on `stream`.
 */
GDN_API int gdn_decode_tp(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                          float* state, const float* A_log, const gdn_bf16* a,
                          const float* dt_bias, const gdn_bf16* b, double scale,
                          gdn_bf16* const* peer_outputs, uint32_t* const* peer_signals,
                          uint32_t* epoch_counter, int32_t* status, uint32_t timeout_us,
                          int rank, int world, int B, int H, int HV, int K, int V,
                          int use_qk_l2norm, void* stream);

/*
 * gdn_decode_tp for the next step of a sequence of steps enqueued back to back on
 * one stream (no counterpart in the reference).  The decode kernel is launched as
 * a programmatic dependent of the previous call's barrier kernel: its CTAs load
 * their state while that barrier still waits for the other ranks, and wait for
 * the barrier grid (griddepcontrol.wait) before reading any other input or
 * storing any output.  Requires that the kernel enqueued on `stream` right
 * before this call is the barrier of a previous gdn_decode_tp /
 * gdn_decode_tp_chained call (that barrier lets this step launch only after its
 * own decode kernel has completed, so every state those steps wrote is
 * complete), and that nothing that writes `state` runs between them.  Results
 * are identical to gdn_decode_tp.
 */
GDN_API int gdn_decode_tp_chained(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                                  float* state, const float* A_log, const gdn_bf16* a,
                                  const float* dt_bias, const gdn_bf16* b, double scale,
                                  gdn_bf16* const* peer_outputs, uint32_t* const* peer_signals,
                                  uint32_t* epoch_counter, int32_t* status, uint32_t timeout_us,
                                  int rank, int world, int B, int H, int HV, int K, int V,
                                  int use_qk_l2norm, void* stream);

/*
 * Allocation-free variant of gdn_decode_tp.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory where they run the decode
 * step: a serving runtime that reserves all of HBM for its own pool at
 * start-up, code that runs while a CUDA graph is being captured (cudaMalloc is
 * not allowed there), a plain-C host without an allocator of its own.  The one
 * piece of scratch gdn_decode_tp needs besides the caller's inputs, outputs and
 * signal words is its epoch counter; here it comes from a fixed array inside
 * the library: 64 uint32 "channels" (GDN_ERR_LIMIT outside 0..63), present on
 * every GPU that loads the library until the process exits.  Nothing is
 * allocated: no cudaMalloc, no cudaFree, no allocating library call.
 *  - The first call on a device looks up the array's device address with that
 *    device current (cudaGetSymbolAddress, checked); make that first call
 *    before any stream capture on the device.
 *  - A channel starts at zero when the library is loaded and keeps counting
 *    across calls (the barrier's epoch continues; nothing is cleared per
 *    call).  Use a channel with one set of signal words only (zero before its
 *    first call on that channel), and the same channel number on every rank.
 *  - Every call on a channel shares its counter: calls on the same channel
 *    that overlap on the GPU (different streams, no ordering) race.
 *  - The device address is cached per device ordinal for the life of the
 *    process.  Do not call this entry after cudaDeviceReset on that device
 *    (the reset unloads the module and the cached address goes stale).
 * Other arguments and results as gdn_decode_tp.
 */
GDN_API int gdn_decode_tp_static(const gdn_bf16* q, const gdn_bf16* k, const gdn_bf16* v,
                                 float* state, const float* A_log, const gdn_bf16* a,
                                 const float* dt_bias, const gdn_bf16* b, double scale,
                                 gdn_bf16* const* peer_outputs,
                                 uint32_t* const* peer_signals, int32_t* status,
                                 uint32_t timeout_us, int channel, int rank, int world,
                                 int B, int H, int HV, int K, int V, int use_qk_l2norm,
                                 void* stream);

/*
 * Head interleave after a tensor-parallel output all-gather.
 *
 * No counterpart in the reference (it runs on one GPU only).  Rank r of W
 * owns v-heads [r*HVl, (r+1)*HVl); an all-gather of the per-rank outputs
 * [rows, HVl, V] yields `gathered` [W, rows, HVl, V]; this writes
 * `output` [rows, W*HVl, V] (rows = B*T).
 */
GDN_API int gdn_interleave_heads(const gdn_bf16* gathered, gdn_bf16* output,
                         int world, int rows, int HVl, int V, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
