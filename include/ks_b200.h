/*
 * KernelSwift-B200: C ABI of the sm_100a operator library (libks_b200.so).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*, NULL = legacy default stream), launches
 * asynchronously on that stream and returns KS_OK or an error code; the message
 * of the last error on the calling thread is available from ks_last_error().
 * The caller owns all input, output and workspace memory.  Tensors are
 * row-major and contiguous unless a stride argument says otherwise.  bf16
 * tensors are passed as raw 16-bit storage.
 *
 * Kernels never spin without bound: a wait that runs out of its time budget
 * (KS_WAIT_BUDGET_MS in the environment, default 2000 ms) records an error in a
 * per-device status record (the code and where the first timeout happened) and
 * the kernel returns.  ks_device_status() reads and clears that record.
 */
#ifndef KS_B200_H
#define KS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KS_OK 0
#define KS_ERR_INVALID 1     /* bad pointer, shape or argument */
#define KS_ERR_UNSUPPORTED 2 /* valid call outside what the kernels implement */
#define KS_ERR_ALIGNMENT 3   /* pointer or stride not aligned as required */
#define KS_ERR_CUDA 4        /* a CUDA runtime call failed */
#define KS_ERR_WORKSPACE 5   /* workspace missing or too small */
#define KS_ERR_DEVICE 6      /* a kernel reported a timed-out wait or a bounds error */

#define KS_INT32 0
#define KS_INT64 1

/* Message of the last failing call on this thread ("" if none). */
const char* ks_last_error(void);

/* Library ABI version (major * 100 + minor). */
int ks_version(void);

/*
 * Sinkhorn normalisation of n_mats independent n x n fp32 matrices (x and out
 * are [n_mats, n, n], 16-byte aligned; x == out is allowed).
 * Semantics of baseline/sinkhorn.py:13-19: softmax over the last dim plus eps,
 * one column normalisation, then repeat-1 (row, column) normalisations, each
 * dividing by (sum + eps).  1 <= n <= 64.
 * Replaces sinkhorn_torch, optimized/sinkhorn_project/op_extension/sinkhorn_torch.cpp:18-56
 * (which accepted 4x4 only).
 */
int ks_sinkhorn(const float* x, float* out, int64_t n_mats, int32_t n, int32_t repeat, float eps,
                void* stream);

/*
 * Top-k sparse attention with a per-head sink logit, baseline/sparse_attention.py:5-42.
 *   q    bf16 [B, M, H, D]     kv bf16 [B, N, D] (shared by all heads: MQA / MLA latent)
 *   sink fp32 [H]              topk_idxs int32 [B, M, K]; entries < 0 are ignored,
 *                              repeated entries count once per occurrence; entries
 *                              >= N are ignored too and reported as a bounds error
 *                              by ks_device_status (the reference's gather raises)
 *   out  bf16 [B, M, H, dv]  = output columns [dv_begin, dv_begin + dv) of the
 *                              reference (V is kv[..., dv_begin : dv_begin + dv]).
 * Requirements: H <= 128, D % 64 == 0, D <= 576, dv % 64 == 0 (dv may be any
 * multiple of 64 up to 512), dv_begin % 64 == 0, dv_begin + dv <= D.
 * Replaces sparse_attn_megakernel_basic_torch,
 * optimized/sparse_attention/op_extension/sparse_attn_torch.cpp:96-160.
 */
int ks_sparse_attn(const void* q, const void* kv, const float* attn_sink,
                   const int32_t* topk_idxs, void* out, int64_t B, int64_t M, int64_t H,
                   int64_t D, int64_t N, int64_t K, int64_t dv_begin, int64_t dv,
                   float softmax_scale, void* stream);

/* Workspace bytes ks_indexer needs for B x S query rows over T keys. */
size_t ks_indexer_workspace_size(int64_t B, int64_t S, int64_t T);

/*
 * Lightning-indexer top-k, baseline/indexer.py:170-205 after the two projections:
 * RoPE on the last rope_dim dims of q, scores
 *   bf16( sum_h bf16( relu(bf16(q_h . k_t)) * w_h ) ),
 * causal mask (causal != 0: key t valid iff t < (pos0 + s + 1) / ratio),
 * top-min(topk, T) indices by value descending, ties by lower index, then
 * causal: invalid -> -1, else index + offset.
 *   q     bf16 [B, S, H, D], projected, before RoPE      (H in {16, 32, 64}, D in {64, 128})
 *   k     bf16 keys; batch b, key t at k + (b * k_batch_rows + t) * D   (t < T <= 65536)
 *   w     bf16 [B, S, H] head weights (already scaled by D^-0.5 H^-0.5)
 *   freqs fp32 [S, rope_dim / 2, 2] (cos, sin) at the positions of the S rows
 *   out   [B, S, min(topk, T)] int32 (out_dtype KS_INT32) or int64 (KS_INT64)
 *   pos0  sequence position of row s = 0 (0 for a whole prefill call; the
 *         first row of the shard when the rows are split)
 * topk <= 4096.  workspace >= ks_indexer_workspace_size(B, S, T), 256-byte aligned.
 * Replaces indexer_rope_torch, indexer_qk_reduce_torch and indexer_topk_torch,
 * optimized/indexer_project/op_extension/indexer_torch.cpp:100-268.
 */
int ks_indexer(const void* q, const void* k, int64_t k_batch_rows, const void* w,
               const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
               int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio, int32_t topk,
               int64_t offset, void* out, int32_t out_dtype, void* workspace,
               size_t workspace_bytes, void* stream);

/*
 * Score stage of ks_indexer alone: writes bf16 scores [B * S, score_ld] (row
 * b * S + s; columns >= the row's causal limit inside the last 128-key tile
 * hold -inf, columns beyond it are not written).  score_ld % 8 == 0, >= T.
 * Replaces indexer_rope_torch + indexer_qk_reduce_torch,
 * optimized/indexer_project/op_extension/indexer_torch.cpp:100-198.
 */
int ks_indexer_scores(const void* q, const void* k, int64_t k_batch_rows, const void* w,
                      const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
                      int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio,
                      void* scores, int64_t score_ld, void* stream);

/*
 * Top-k stage of ks_indexer alone over bf16 score rows [B * S, score_ld]
 * (only the valid prefix of each row is read).
 * Replaces indexer_topk_torch, optimized/indexer_project/op_extension/indexer_torch.cpp:232-268.
 */
int ks_topk_rows(const void* scores, int64_t score_ld, int64_t B, int64_t S, int64_t T,
                 int64_t pos0, int32_t causal, int32_t ratio, int32_t topk, int64_t offset,
                 void* out, int32_t out_dtype, void* stream);

/*
 * One DeepSeek-sparse-attention step over B x S query rows: the indexer
 * (exactly ks_indexer with out_dtype KS_INT32) selects top-min(topk, T) keys per
 * row, and sparse attention (exactly ks_sparse_attn with dv_begin = 0 and
 * K = min(topk, T)) attends to them.  The int32 indices go from the first stage
 * to the second in idx_out [B, S, min(topk, T)] (also a result), never as int64.
 *   q_ix, k_ix, w, freqs, rope_dim, pos0, causal, ratio, offset: as ks_indexer
 *   q_sa bf16 [B, S, H_sa, D_sa], kv bf16 [B, N, D_sa], attn_sink fp32 [H_sa]
 *   out  bf16 [B, S, H_sa, dv]
 * The indexer's output (index + offset, or -1) must address rows of kv: entries
 * >= N are skipped and reported by ks_device_status.  workspace >=
 * ks_indexer_workspace_size(B, S, T), 256-byte aligned.  T >= 1.
 * Composes baseline/indexer.py:195-205 (int64 indices) feeding
 * baseline/sparse_attention.py:16-17 (topk_idxs); the reference has no single
 * host op for the pair.
 */
int ks_dsa(const void* q_ix, const void* k_ix, int64_t k_batch_rows, const void* w,
           const float* freqs, int64_t B, int64_t S, int64_t H_ix, int64_t D_ix, int64_t T,
           int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio, int32_t topk,
           int64_t offset, const void* q_sa, const void* kv, int64_t N, const float* attn_sink,
           int64_t H_sa, int64_t D_sa, int64_t dv, float softmax_scale, int32_t* idx_out,
           void* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The indexer's projections with their follow-up arithmetic fused: the
 * producer of ks_indexer's q (rotated) and w (scaled) inputs.
 *   out[m, n] = bf16( sum_k a[m, k] * w[n, k] )            a bf16 [M, K], w bf16 [N, K]
 * (F.linear: fp32 accumulation, bf16 result), then
 *   rope_dim > 0: in every head_dim-wide group of columns the last rope_dim are
 *                 rotated as interleaved pairs with freqs[m % S] ([S, rope_dim/2, 2]
 *                 fp32 cos, sin), products and sums in fp32, result bf16
 *   apply_scale:  out = bf16( float(out) * scale )
 * Computes q = wq_b(qr) + RoPE (baseline/indexer.py:170-172, 114-129; then call
 * ks_indexer with rope_dim = 0) and weights = weights_proj(x) * scale
 * (baseline/indexer.py:173-175) on the tensor cores.  N % 16 == 0, K % 8 == 0,
 * pointers 16-byte aligned.  Replaces the reference's torch-side projections
 * and its RoPE op (optimized/indexer_project/indexer.py:196-200,
 * optimized/indexer_project/op_extension/indexer_torch.cpp:100-172).
 */
int ks_proj_rope(const void* a, const void* w, void* out, int64_t M, int64_t N, int64_t K,
                 int32_t head_dim, int32_t rope_dim, const float* freqs, int64_t S, float scale,
                 int32_t apply_scale, void* stream);

/*
 * e4m3 (fp8) quantisation of bf16 rows [rows, D] with one power-of-two scale
 * per row (the "ue8m0" scale format of ModelArgs, baseline/indexer.py:15):
 * scale[r] = the smallest power of two >= max(max_i |x[r,i]|, 1e-4) / 448 and
 * x8[r,i] = e4m3(x[r,i] / scale[r]) rounded to nearest even, saturating at +-448.
 * D % 4 == 0; x 8-byte aligned, x8 and scale 4-byte aligned.  Prepares the
 * queries (per token and head) and keys (per key) of ks_indexer_fp8.
 * The reference declares the FP8 option but implements no kernel for it.
 */
int ks_quant_fp8_rows(const void* x, void* x8, float* scale, int64_t rows, int32_t D,
                      void* stream);

/*
 * FP8 lightning indexer: ks_indexer with e4m3 queries and keys (ModelArgs.dtype
 * = "fp8", baseline/indexer.py:14; the bf16 baseline declares but does not use
 * it).  Scores
 *   bf16( k_scale[b,t] * sum_h( relu(q8[b,s,h,:] . k8[b,t,:]) * w[b,s,h] ) )
 * with the dot products from the tensor cores (fp32 accumulation), each
 * product and partial sum in fp32 rounded to nearest in head order; then the
 * causal mask, top-k and -1/offset post-processing of ks_indexer.
 *   q8 e4m3 [B, S, H, D] (rotated before quantisation: no RoPE here), D = 128
 *   k8 e4m3 keys; batch b, key t at k8 + (b * k_batch_rows + t) * D
 *   w  fp32 [B, S, H]  head weight x the query row's scale (x D^-0.5 H^-0.5)
 *   k_scale fp32 per key row, laid out like the rows of k8
 * out, workspace, pos0, causal, ratio, topk, offset: as ks_indexer.
 */
int ks_indexer_fp8(const void* q8, const void* k8, int64_t k_batch_rows, const float* w,
                   const float* k_scale, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
                   int64_t pos0, int32_t causal, int32_t ratio, int32_t topk, int64_t offset,
                   void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Score stage of ks_indexer_fp8 alone (bf16 scores laid out as ks_indexer_scores). */
int ks_indexer_fp8_scores(const void* q8, const void* k8, int64_t k_batch_rows, const float* w,
                          const float* k_scale, int64_t B, int64_t S, int64_t H, int64_t D,
                          int64_t T, int64_t pos0, int32_t causal, int32_t ratio, void* scores,
                          int64_t score_ld, void* stream);

/*
 * ks_indexer without a workspace argument, for callers that cannot allocate
 * device memory: processes whose device memory belongs to another allocator
 * (a framework's caching allocator or a fixed memory pool that must not be
 * bypassed), latency-critical paths that must not call cudaMalloc (it can
 * synchronise the device), and hosts such as FFI bindings or plugins that have
 * no device allocator to call.  It allocates nothing: the
 * score rows between the two kernels live in a fixed 32 MiB device array inside
 * the library, so B * S * round_up(T, 8) * 2 must not exceed 33554432 bytes
 * (larger calls are rejected with KS_ERR_WORKSPACE; split the rows over several
 * calls).  Every GPU that loads the library holds the array until the process
 * exits.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before
 * any stream capture.  All calls on a device share the one array, so calls that
 * overlap on the GPU (two streams, or two host threads) race on it: serialise
 * them.  The array keeps the last call's contents; nothing in it needs clearing.
 * Arguments and results are those of ks_indexer.  No counterpart in the
 * reference (its host op allocates its score buffer through torch).
 */
int ks_indexer_noalloc(const void* q, const void* k, int64_t k_batch_rows, const void* w,
                       const float* freqs, int64_t B, int64_t S, int64_t H, int64_t D, int64_t T,
                       int32_t rope_dim, int64_t pos0, int32_t causal, int32_t ratio,
                       int32_t topk, int64_t offset, void* out, int32_t out_dtype, void* stream);

/*
 * Synchronise `stream`, then read and clear the current device's status record:
 * KS_OK, or KS_ERR_DEVICE when a kernel reported a timed-out wait or a bounds
 * error since the last call (ks_last_error() then names the block, thread,
 * barrier and progress tag of the first timed-out wait).  No counterpart in the
 * reference.
 */
int ks_device_status(void* stream);

/*
 * Self-test of the bounded-wait path: launches one CTA that waits on a barrier
 * nobody completes, with the given budget; the wait gives up, records a
 * timeout in the status record and the kernel returns.  No counterpart in the
 * reference.
 */
int ks_selftest_wait_timeout(uint64_t budget_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KS_B200_H */
