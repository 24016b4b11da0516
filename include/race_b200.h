/*
 * race_b200.h -- C ABI of the B200-native causal RACE attention operator.
 *
 * Plain pointers, sizes and an explicit cudaStream_t (passed as void*); no
 * torch types.  Every entry point returns a status code (RACE_OK == 0) and
 * never allocates: callers size the workspace with race_workspace_bytes().
 * Launches go on the given stream and use the calling thread's current CUDA
 * device (the library links the shared CUDA runtime, so a caller's
 * cudaSetDevice / torch device guard applies).
 *
 * Notation: N independent streams (batch x heads), T tokens, D head_dim,
 * L hash tables, P hyperplanes per table, R = 2^P corners, S = L*R buckets.
 * Tensors are dense, row-major:
 *   Q, K, V, out, dO, dQ, dK, dV : [N, T, D]           (dtype: RACE_F32/RACE_BF16)
 *   probsK, probsQ, gradients    : [N, T, S]  float32  (bucket s = l*R + r)
 *   planes_T                     : [D, L*P]   float32  (column l*P + p)
 *   state A / B                  : [N, S] / [N, S, D] float32
 * Bucket/corner order and plane layout are the reference's
 * (scaling/race_common.py:14-33).  The math of every entry point is
 *   out_t = sum_s pq[t,s] * B_t[s,:] / (A_t[s] + eps),
 *   A_t = A0 + sum_{tau<=t} pk[tau,s],  B_t = B0 + sum_{tau<=t} pk[tau,s] V[tau,:]
 * (scaling/race_common.py:76-90), with pq/pk the soft hash of Q/K
 * (scaling/race_common.py:36-73): softmax over the R corners of
 * sum_p tanh(x . planes_T[:, l*P+p]) * logit_scale * (+-1).
 */
#ifndef RACE_B200_H
#define RACE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define RACE_OK 0
#define RACE_ERR_ARG 1          /* NULL pointer or invalid scalar argument   */
#define RACE_ERR_SHAPE 2        /* dimensions out of range / inconsistent    */
#define RACE_ERR_DTYPE 3        /* dtype enum not supported                  */
#define RACE_ERR_ALIGN 4        /* pointer alignment not met                 */
#define RACE_ERR_WORKSPACE 5    /* workspace NULL or smaller than required   */
#define RACE_ERR_CUDA 6         /* CUDA runtime / launch error               */
#define RACE_ERR_TIMEOUT 7      /* a bounded device-side wait expired        */
#define RACE_ERR_UNSUPPORTED 8  /* configuration has no kernel               */

/* ---- dtypes of the [N,T,D] activations ------------------------------------ */
#define RACE_F32 0
#define RACE_BF16 1

/* ---- operation ids for race_workspace_bytes ------------------------------ */
#define RACE_OP_FWD_PROBS 0
#define RACE_OP_BWD_PROBS 1
#define RACE_OP_FWD_QKV 2
#define RACE_OP_BWD_QKV 3
#define RACE_OP_STATE 4
#define RACE_OP_BWD_SPLIT 5  /* race_bwd_local + race_bwd_finish (one workspace) */
#define RACE_OP_FWD_SPLIT 6  /* race_fwd_local + race_fwd_finish (one workspace) */
#define RACE_OP_ACE_FWD 7    /* race_ace_fwd (non-causal)                      */
#define RACE_OP_ACE_BWD 8    /* race_ace_bwd (non-causal)                      */

/* Library ABI version (bumped on any signature change). */
int race_abi_version(void);

/* Human-readable text of a status code; race_last_error() gives the detail of
 * the most recent failure on the calling thread (empty if none). */
const char *race_status_string(int status);
const char *race_last_error(void);

/* Diagnostic: number of kernel launches this library has issued in this
 * process (host-side counter; used to report launches per benchmark step).
 * One process-wide counter: launches from every thread and stream add to it. */
unsigned long long race_launch_counter(void);

/* Diagnostic (no counterpart in the reference): device time of the tcgen05
 * kernels.  While enabled, CUDA events are recorded on the launch stream
 * around every launch of the kernels below; race_kernel_time() waits for the
 * events recorded so far and returns the totals since the last enable.
 * Enabling clears the totals.  Not for use inside stream capture.  The event
 * lists and totals are process-wide (one set for all threads, streams and
 * devices, guarded by a mutex): time one stream at a time, or the totals mix
 * the launches of every stream that ran while timing was on.  The compute
 * entry points keep no data between calls (their only shared settings are the
 * process-wide wait controls below). */
#define RACE_KT_FWD_TOTALS 0   /* fused K-hash + segment totals / chunk states */
#define RACE_KT_FWD_READOUT 1  /* forward readout                              */
#define RACE_KT_BWD_REV 2      /* backward reverse walk (segment-local grads)  */
#define RACE_KT_SCAN 3         /* segment prefix / suffix scans                */
#define RACE_KT_BWD_FIX 4      /* backward suffix fix-up (dK, dV, dQ)          */
#define RACE_KT_ACE_TILE 5     /* non-causal per-token tile kernel             */
#define RACE_KT_COUNT 6
int race_kernel_timing(int enable);
int race_kernel_time(int kernel, double *total_ms, long long *launches);
/* (The timing state is process-wide: one event list per kernel id, shared by
 * every host thread and stream.  Two threads timing at once mix their totals;
 * it is a measurement aid for one timing thread, not a per-stream facility.) */

/* Bounded device-side waits (no counterpart in the reference, whose kernels
 * launch with no error check: kernels/gpu/forward_kernel.cu:128-135).  Every
 * wait of the tcgen05 kernels on an mbarrier gives up after a poll limit.  A
 * kernel whose wait gave up stops working (every thread still takes every
 * barrier step), waits for its own tensor-core work in flight, frees its
 * tensor memory, returns, and leaves a non-zero status word at the head of
 * the call's workspace; that call's outputs are then invalid.  These settings
 * are process-wide and apply to calls made after them, from any thread.
 *
 * race_set_wait_limit: polls before a wait gives up (0 restores the default,
 *   2^26 polls, about a second on a B200; waits that sleep between polls, up
 *   to 1 us each, count each poll as 32).
 * race_set_status_check: 1 makes every later tcgen05-path call wait for its
 *   stream, read the status word and return RACE_ERR_TIMEOUT when a wait gave
 *   up (this synchronises, so not inside stream capture); 0 (the default)
 *   leaves the word for race_read_status.
 * race_read_status: waits for `stream`, then copies the status word of
 *   `workspace` to *status (0: every wait completed).
 * race_test_withhold_first_load: test hook.  1 makes the forward kernels
 *   issue no tile load for the first chunk of each segment, so their first
 *   waits expire with nothing in flight and the call reports a timeout. */
int race_set_wait_limit(unsigned int polls);
int race_set_status_check(int synchronous);
int race_read_status(const void *workspace, void *stream, int *status);
int race_test_withhold_first_load(int on);

/* Bytes of device workspace `op` needs for these sizes (pure host function).
 * chunk <= 0 selects the library default. */
int race_workspace_bytes(int op, int64_t N, int64_t T, int64_t S, int64_t D,
                         int64_t L, int64_t P, int dtype, int64_t chunk,
                         size_t *bytes);

/* The tcgen05 path's work split for N streams of T tokens on a device with `sms`
 * SMs (pure host function): *nseg segments of *seg_chunks 128-token chunks per
 * stream, one CTA each, and *max_nseg, the segment count the workspace from
 * race_workspace_bytes() has room for (a plan never exceeds it).  For
 * inspection and tests; the library plans by itself on the current device. */
int race_plan_segments(int64_t N, int64_t T, int64_t S, int sms, int *nseg, int *seg_chunks,
                       int *max_nseg);

/* ---- probability-level operator -----------------------------------------
 * Replaces race_fused_fwd (kernels/gpu/forward_kernel.cu:110-137), bound by
 * pybind at kernels/gpu/race_cuda_binding.cpp:12-17.  out[N,T,D] fp32 is fully
 * written (no pre-zeroing needed).  A_final/B_final may be NULL; otherwise they
 * receive the state after the last token (race_prefix_ref's A_final/B_final,
 * scaling/race_common.py:88-90). */
int race_fwd_probs(const float *probsK, const float *probsQ, const float *V2,
                   float *out, float *A_final, float *B_final,
                   int64_t N, int64_t T, int64_t S, int64_t D,
                   float eps, int64_t chunk,
                   void *workspace, size_t workspace_bytes, void *stream);

/* Replaces race_backward (kernels/gpu/backward_kernels.cu:174-215), bound at
 * kernels/gpu/race_cuda_binding.cpp:18-21: exact gradients w.r.t. probsK,
 * probsQ and V2 for upstream grad_out. */
int race_bwd_probs(const float *probsK, const float *probsQ, const float *V2,
                   const float *grad_out,
                   float *grad_probsK, float *grad_probsQ, float *grad_V2,
                   int64_t N, int64_t T, int64_t S, int64_t D,
                   float eps, int64_t chunk,
                   void *workspace, size_t workspace_bytes, void *stream);

/* ---- soft hash -------------------------------------------------------------
 * Replaces the probability half of soft_hash_probs
 * (scaling/race_common.py:36-73, share_planes layout): probs[N,T,S] fp32 of X. */
int race_soft_hash(const void *X, int dtype, const float *planes_T, float *probs,
                   int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                   float logit_scale, void *stream);

/* Gradient of soft_hash_probs w.r.t. X (autograd of
 * scaling/race_common.py:56-72): dX[N,T,D] (dtype) from dprobs[N,T,S] fp32. */
int race_soft_hash_bwd(const void *X, int dtype, const float *planes_T,
                       const float *dprobs, void *dX,
                       int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                       float logit_scale, void *stream);

/* ---- fused layer (soft hash + causal scan + readout) ---------------------
 * Replaces RaceCausalCuda.forward (scaling/race_causal_cuda.py:94-102), i.e.
 * soft_hash_probs + RaceCausalFn.forward without materialising the [N,T,S]
 * probabilities.  A0/B0 (may be NULL = zero) is a carried-in state: the prefix
 * of earlier sequence shards, or a decode cache.  A_final/B_final may be NULL. */
int race_fwd_qkv(const void *Q, const void *K, const void *V, int dtype,
                 const float *planes_T, void *out,
                 const float *A0, const float *B0,
                 float *A_final, float *B_final,
                 int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                 float eps, float logit_scale,
                 void *workspace, size_t workspace_bytes, void *stream);

/* Replaces RaceCausalFn.backward (scaling/race_causal_cuda.py:64-69) composed
 * with the autograd of soft_hash_probs.  gA_in/gB_in (may be NULL) is the
 * gradient reaching the final state from later sequence shards; dA0/dB0 (may
 * be NULL) receive the gradient w.r.t. the carried-in state A0/B0. */
int race_bwd_qkv(const void *Q, const void *K, const void *V, const void *dO,
                 int dtype, const float *planes_T,
                 void *dQ, void *dK, void *dV,
                 const float *A0, const float *B0,
                 const float *gA_in, const float *gB_in,
                 float *dA0, float *dB0,
                 int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                 float eps, float logit_scale,
                 void *workspace, size_t workspace_bytes, void *stream);

/* Forward that also keeps what the backward needs, and the backward that uses it
 * (no counterpart in the reference; the reference's autograd saves probsK/probsQ
 * instead, scaling/race_causal_cuda.py:57).  For the tcgen05 configurations
 * race_saved_bytes() gives the size of the caller-owned `saved` buffer (16-byte
 * aligned): the layer's state at every 128-token chunk start, A + eps fp32
 * [N, ceil(T/128), S] then B bf16 [N, ceil(T/128), S, D]; race_bwd_qkv_saved()
 * then skips the two passes that rebuild those states.  Pass the same
 * Q, K, V, planes, A0, B0, eps and logit_scale to both.  Elsewhere the size is 0
 * and the two calls are race_fwd_qkv / race_bwd_qkv. */
int race_saved_bytes(int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, int dtype, size_t *bytes);
int race_fwd_qkv_save(const void *Q, const void *K, const void *V, int dtype,
                      const float *planes_T, void *out, const float *A0, const float *B0,
                      float *A_final, float *B_final, void *saved, size_t saved_bytes,
                      int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps,
                      float logit_scale, void *workspace, size_t workspace_bytes, void *stream);
int race_bwd_qkv_saved(const void *Q, const void *K, const void *V, const void *dO, int dtype,
                       const float *planes_T, const void *saved, size_t saved_bytes,
                       void *dQ, void *dK, void *dV, const float *A0, const float *B0,
                       const float *gA_in, const float *gB_in, float *dA0, float *dB0,
                       int64_t N, int64_t T, int64_t D, int64_t L, int64_t P, float eps,
                       float logit_scale, void *workspace, size_t workspace_bytes, void *stream);

/* ---- state / decode (no reference counterpart: the reference's KV-cache
 * branch raises NotImplementedError, chat/nanochat/gpt.py:143-146) ---------- */

/* Prefill -> decode-state handoff, and phase A of the sequence-sharded forward:
 * A_out[N,S] = A0 + sum_t pk_t,  B_out[N,S,D] = B0 + sum_t pk_t V_t
 * (race_prefix_ref's A_final/B_final, scaling/race_common.py:88-90).
 * A0/B0 may be NULL. */
int race_state_from_prefill(const void *K, const void *V, int dtype,
                            const float *planes_T,
                            const float *A0, const float *B0,
                            float *A_out, float *B_out,
                            int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                            float logit_scale,
                            void *workspace, size_t workspace_bytes, void *stream);

/* One fused decode step for a batch of single tokens with grouped-query
 * sharing: q[Nq,D], k/v[Nkv,D] (Nq = Nkv*group, q head i reads kv stream
 * i/group).  Updates the persistent state A[Nkv,S], B[Nkv,S,D] in place with
 * this token's key, then writes out[Nq,D] = row t of the layer output.
 * A and B must be 16-byte aligned (the state streams in by 16-byte copies;
 * otherwise RACE_ERR_ALIGN, nothing launched). */
int race_decode_step(const void *q, const void *k, const void *v, int dtype,
                     const float *planes_T, float *A, float *B, void *out,
                     int64_t Nq, int64_t Nkv, int64_t D, int64_t L, int64_t P,
                     float eps, float logit_scale, void *stream);

/* Softmax grouped-query attention for one decode token over a bf16 KV cache,
 * for the softmax layers of a hybrid decoder whose other layers are RACE
 * (no reference counterpart; the hybrid decode configuration's softmax half).
 * q[B,Hq,64], k_new/v_new[B,Hkv,64], k_cache/v_cache[B,Hkv,Tmax,64], all bf16
 * and contiguous; *len (int32, device memory) = tokens already cached.  The
 * call stores (k_new, v_new) at cache position *len, then writes
 *   out[b,i] = softmax_j(softmax_scale * q[b,i].K[b,i/G,j]) V[b,i/G,j], j <= *len,
 * G = Hq/Hkv <= 8.  It does not advance *len (the caller does, once
 * per step for all layers), so one launch can be captured in a CUDA graph and
 * replayed every step.  workspace: race_gqa_decode_workspace_bytes(B, Hq, Hkv,
 * n_splits) bytes, zero-filled before its first use and reused as is (the
 * kernel leaves it ready for the next call); one workspace per concurrently
 * running call.  n_splits in [1,64] = key ranges per (b, kv head) processed in
 * parallel.  *len outside [0, Tmax) stores nothing, leaves out unwritten and
 * sets the workspace's last int32 to 1. */
size_t race_gqa_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int n_splits);
int race_gqa_decode_attn(const void *q, const void *k_new, const void *v_new,
                         void *k_cache, void *v_cache, const int32_t *len, void *out,
                         void *workspace, int64_t B, int64_t Hq, int64_t Hkv, int64_t Tmax,
                         int64_t D, int n_splits, float softmax_scale, void *stream);

/* ---- sequence-sharded phases (one rank's contiguous slice of T) ---------- */

/* The fused layer on activations laid out [B, T, H, D] (the layout attention modules
 * produce before any transpose; stream n = b*H + h, N = B*H), forward with the chunk
 * states kept in `saved` (race_saved_bytes(B*H, ...), may be NULL) and backward reusing
 * them.  Workspace sizes as race_fwd_qkv / race_bwd_qkv with N = B*H.  No reference
 * counterpart: chat/nanochat/gpt.py:133-139 transposes q, k, v to [B, H, T, D] and the
 * output back around the RACE call.  tcgen05 path only (bf16, D = 64, P = 4, L in {8, 16});
 * other configurations return RACE_ERR_UNSUPPORTED. */
int race_fwd_bthd(const void *Q, const void *K, const void *V, int dtype,
                  const float *planes_T, void *out, void *saved, size_t saved_bytes,
                  int64_t B, int64_t T, int64_t H, int64_t D, int64_t L, int64_t P,
                  float eps, float logit_scale,
                  void *workspace, size_t workspace_bytes, void *stream);
int race_bwd_bthd(const void *Q, const void *K, const void *V, const void *dO, int dtype,
                  const float *planes_T, const void *saved, size_t saved_bytes,
                  void *dQ, void *dK, void *dV,
                  int64_t B, int64_t T, int64_t H, int64_t D, int64_t L, int64_t P,
                  float eps, float logit_scale,
                  void *workspace, size_t workspace_bytes, void *stream);

/* Forward of a shard in two calls on ONE workspace (RACE_OP_FWD_SPLIT size):
 * race_fwd_local writes this shard's state totals A_tot[N,S], B_tot[N,S,D]
 * (what race_state_from_prefill with A0 = B0 = NULL writes) and keeps its
 * segment prefixes in the workspace; race_fwd_finish then writes `out`
 * given A0/B0 = the sum of the totals of all earlier shards (NULL: none),
 * without recomputing them.  `saved` (optional, race_saved_bytes) receives
 * the chunk states race_bwd_local/race_bwd_finish can reuse, as
 * race_fwd_qkv_save does.  Same K/V (and workspace) to both calls. */
int race_fwd_local(const void *K, const void *V, int dtype,
                   const float *planes_T, float *A_tot, float *B_tot,
                   int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                   float logit_scale,
                   void *workspace, size_t workspace_bytes, void *stream);
int race_fwd_finish(const void *Q, const void *K, const void *V, int dtype,
                    const float *planes_T, void *out, void *saved, size_t saved_bytes,
                    const float *A0, const float *B0,
                    int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                    float eps, float logit_scale,
                    void *workspace, size_t workspace_bytes, void *stream);

/* Backward of a shard in two calls on ONE workspace (RACE_OP_BWD_SPLIT size):
 * race_bwd_local writes this shard's gradient totals for its start state
 *   gA_tot[N,S]   = sum_t -pq[t,s] * G_t[s] / (A_t[s] + eps)^2,
 *                   G_t[s] = dO_t . B_t[s,:]
 *   gB_tot[N,S,D] = sum_t pq[t,s] * dO_t / (A_t[s] + eps)
 * given the carried-in forward prefix A0/B0 (and optionally the `saved`
 * chunk states of race_fwd_qkv_save), and keeps its local gradients in the
 * workspace; race_bwd_finish then writes dQ, dK, dV given gA_in/gB_in = the
 * sum of the totals of all later shards.  Same inputs to both calls. */
int race_bwd_local(const void *Q, const void *K, const void *V, const void *dO, int dtype,
                   const float *planes_T, const void *saved, size_t saved_bytes,
                   const float *A0, const float *B0, float *gA_tot, float *gB_tot,
                   int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                   float eps, float logit_scale,
                   void *workspace, size_t workspace_bytes, void *stream);
int race_bwd_finish(const void *Q, const void *K, const void *V, const void *dO, int dtype,
                    const float *planes_T, const void *saved, size_t saved_bytes,
                    const float *A0, const float *B0, const float *gA_in, const float *gB_in,
                    void *dQ, void *dK, void *dV,
                    int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                    float eps, float logit_scale,
                    void *workspace, size_t workspace_bytes, void *stream);

/* ---- allocation-free variant ----------------------------------------------
 * No counterpart in the reference.  Same math and outputs as race_fwd_probs
 * (without A_final/B_final), for callers that cannot give the library device
 * memory: a host that owns a fixed device pool and forbids side allocations,
 * a plugin callback that may only enqueue work on the stream it is handed,
 * or a launch loop that cannot afford cudaMalloc/cudaFree (cudaFree waits for
 * the whole device).  The scan's chunk records live in a library-owned static
 * device array of RACE_NOALLOC_SCRATCH_BYTES bytes, reserved on each GPU when
 * first used there and held until the process exits.  The first call on a
 * device looks up that array's address, so make it outside any stream
 * capture.  All calls share the array: calls whose GPU work overlaps race and
 * must be serialised.  Sizes whose per-stream records (4*ceil(T/32)*(S+S*D)
 * bytes) exceed the array return RACE_ERR_WORKSPACE. */
#define RACE_NOALLOC_SCRATCH_BYTES (32u << 20)
int race_fwd_probs_noalloc(const float *probsK, const float *probsQ, const float *V2,
                           float *out, int64_t N, int64_t T, int64_t S, int64_t D,
                           float eps, void *stream);

/* ---- non-causal RACE (BatchedACE with shared planes) --------------------------
 * Replaces the per-token products of the reference's non-causal module
 * (scaling/benchmark_time.py:129-161, misc/classification.py:282-308; its
 * autograd backward): every query reads the whole sequence's bucket summary,
 *   A = sum_t pk_t,  b = sum_t pk_t^T V_t,  out_t = pq_t (b / (A + eps)).
 * bf16 with D = 64, P = 4, L in {8, 16} (tcgen05 kernels; other configurations
 * return RACE_ERR_UNSUPPORTED).  No [N, T, S] tensor is formed.
 * race_ace_fwd writes out [N,T,64] and the summaries A [N,S], B (= b) [N,S,64]
 * fp32, which race_ace_bwd takes back to give dQ, dK, dV.  Workspace:
 * race_workspace_bytes(RACE_OP_ACE_FWD / RACE_OP_ACE_BWD, ...). */
int race_ace_fwd(const void *Q, const void *K, const void *V, int dtype,
                 const float *planes_T, void *out, float *A, float *B,
                 int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                 float eps, float logit_scale,
                 void *workspace, size_t workspace_bytes, void *stream);
int race_ace_bwd(const void *Q, const void *K, const void *V, const void *dO, int dtype,
                 const float *planes_T, const float *A, const float *B,
                 void *dQ, void *dK, void *dV,
                 int64_t N, int64_t T, int64_t D, int64_t L, int64_t P,
                 float eps, float logit_scale,
                 void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* RACE_B200_H */
