/*
 * sparsedict_b200 — C ABI of the B200 (sm_100a) top-k sparse attention path.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * a dense row-major buffer, every size is an element count, `stream` is a
 * cudaStream_t passed as void* (NULL = the legacy default stream).  No call
 * synchronises the host or throws: each returns 0 (SDK_OK) or one of the
 * status codes below; sdk_status_string() names it.  No call allocates
 * device memory except sdk_topk_attn_fwd on the tensor-core path and
 * sdk_route_top1 (4 bytes per expert per 256 rows), which take stream-ordered
 * scratch from a memory pool of this library (kept for reuse);
 * sdk_topk_attn_fwd_ws is the same forward on the caller's scratch.
 *
 * Layout conventions (the reference's flattened layout,
 * kernels/fused_topk_attn.py:999-1001):
 *   q    [rows, d]        rows = slices * n (uniform) or offsets[slices]
 *   k    [slices, m, d]   keys of slice s start at k + s*m*d
 *   v    [slices, m, dv]
 *   out  [rows, dv], top_idx [rows, topk] int32, lse [rows]
 * Element types: SDK_DTYPE_* for q/k/v/out/dout/dq; lse, top_scores and the
 * gradient accumulators are float64 for SDK_DTYPE_F64 and float32 otherwise.
 */
#ifndef SPARSEDICT_B200_H_
#define SPARSEDICT_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SDK_DTYPE_F32 = 0,
  SDK_DTYPE_F64 = 1,
  SDK_DTYPE_BF16 = 2,
  SDK_DTYPE_F16 = 3,
};

enum {
  SDK_OK = 0,
  SDK_ERR_INVALID_ARGUMENT = 1, /* a size, pointer or dtype the call cannot accept */
  SDK_ERR_UNSUPPORTED = 2,      /* valid request outside the library's kernels (e.g. k too large) */
  SDK_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
  SDK_ERR_NO_DEVICE = 4,        /* no sm_100 device is current */
  SDK_ERR_TOO_LARGE = 5,        /* request exceeds the fixed scratch of sdk_topk_attn_bwd_noalloc */
};

/* Library version, (major << 16) | minor. */
int sdk_version(void);

/* Human-readable name of a status code returned by any sdk_* call. */
const char* sdk_status_string(int status);

/* Text of the last CUDA error recorded by this thread (empty if none). */
const char* sdk_last_cuda_error(void);

/* Largest top-k the fused kernels accept for `dtype` and feature width `d`. */
int sdk_max_topk(int32_t dtype, int32_t d);

/* Reads the device status word of the current device into *bits (bit 1: an
 * index outside [0, m) was met and skipped; bit 2: a bounded wait gave up),
 * clearing it when `clear` is nonzero.  Synchronises `stream`.  A forward
 * whose wait gave up writes NaN outputs and LSE and index -1 for the rows it
 * could not finish; callers that must not consume those poll this after a
 * forward. */
int sdk_device_status(unsigned int* bits, int32_t clear, void* stream);

/* Bound, in nanoseconds, of every pipeline wait of the tensor-core forward
 * (launches made after the call; process-wide).  0 restores the default of
 * 2 s; values above 60 s are refused.  A wait that runs out makes its CTA
 * stop, let its in-flight copies land (those waits keep the 2 s bound), mark
 * its rows as given up and raise device status bit 2: the kernel returns and
 * the context stays usable.  No counterpart in the reference (Triton kernels
 * have no bounded waits); used to check that path without a GPU fault. */
int sdk_set_wait_limit(uint64_t ns);

/*
 * Fused forward, stages 1-3: scaled affinity q·kᵀ, per-row top-k selection
 * (NaN first, larger score first, lower key index on ties), softmax over the
 * selected scores and the weighted sum of the gathered value rows.
 *
 * Replaces FusedTopKAttentionFunction.forward (kernels/fused_topk_attn.py:989-1094)
 * and _hybrid_topk_attention_with_aux (kernels/hybrid_topk.py:153-290), whose
 * outputs (top_scores, top_indices int32, lse, out) it writes.
 *   scale       score multiplier 1/(temperature*sqrt(d)) (fused_topk_attn.py:997)
 *   score_grid  0, or G > 0 for the tie-stress affinity rint(G*dot/root)/G with
 *               root = float(1/scale)
 *   row_offsets nullable: when set, slice s owns rows [row_offsets[s],
 *               row_offsets[s+1]) and n is the total row count (grouped /
 *               routed dictionaries)
 *   row_index   nullable: logical row r reads q/writes out at physical row
 *               row_index[r] (a routing permutation); top_idx/lse/top_scores
 *               stay in logical order
 *   top_scores  nullable
 */
int sdk_topk_attn_fwd(const void* q, const void* k, const void* v, void* out, int32_t* top_idx,
                      void* lse, void* top_scores, const int32_t* row_offsets,
                      const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d,
                      int32_t dv, int32_t topk, double scale, int32_t score_grid, int32_t dtype,
                      void* stream);

/*
 * Scratch of the forward: the bf16/fp16 tensor-core path (d = dv = 64,
 * topk <= 64, m <= 65536, score_grid 0, uniform slices) hands each query row's
 * candidate list (192 two-byte keys and four counts) from its streaming
 * kernel to its finishing kernel.  Returns the bytes for `rows` query rows
 * (slices*n, or the grouped row count), 0 when the call will not take that
 * path.  `grouped` (row_offsets or row_index will be passed) does not change
 * the size: grouped slices take the same path with the same scratch per row.
 * The reference's
 * wrapper allocates its intermediate top-k buffers with torch
 * (fused_topk_attn.py:1012-1017); callers that own their memory allocate this
 * and pass it to sdk_topk_attn_fwd_ws.
 */
size_t sdk_topk_attn_fwd_workspace_size(int64_t rows, int64_t m, int32_t d, int32_t dv, int32_t topk,
                                        int32_t score_grid, int32_t grouped, int32_t dtype);

/*
 * sdk_topk_attn_fwd on caller scratch: `workspace` (16-byte aligned, at least
 * sdk_topk_attn_fwd_workspace_size bytes) is used instead of the library pool;
 * SDK_ERR_INVALID_ARGUMENT when it is too small or misaligned.  May be NULL
 * with workspace_bytes 0 (then as sdk_topk_attn_fwd).  The workspace must not
 * be reused by another call until this call's launches on `stream` are done.
 */
int sdk_topk_attn_fwd_ws(const void* q, const void* k, const void* v, void* out, int32_t* top_idx,
                         void* lse, void* top_scores, const int32_t* row_offsets,
                         const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d,
                         int32_t dv, int32_t topk, double scale, int32_t score_grid, int32_t dtype,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Sparse backward on the saved support (replaces
 * FusedTopKAttentionFunction.backward, kernels/fused_topk_attn.py:1096-1201,
 * i.e. kernels B1 _backward_dq :609-846 and B2 _backward_dkv :848-977):
 *   dq      = scale * sum_j dS_ij k_j               (written, dtype)
 *   dk_acc += scale * dS_ij q_i  at row top_idx_ij  (accumulator dtype)
 *   dv_acc += P_ij dout_i        at row top_idx_ij  (accumulator dtype)
 * with P = exp(S - lse), G = dout·v_j, dS = P (G - sum_j P G).  The
 * accumulators are zeroed first unless `accumulate` is nonzero; dk_acc and
 * dv_acc may alias (keys and values that are the same dictionary).  For
 * SDK_DTYPE_F32/F64 the accumulators can be the dK/dV outputs themselves.
 */
int sdk_topk_attn_bwd(const void* q, const void* k, const void* v, const void* dout,
                      const int32_t* top_idx, const void* lse, void* dq, void* dk_acc,
                      void* dv_acc, const int32_t* row_offsets, const int32_t* row_index,
                      int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv, int32_t topk,
                      double scale, int32_t score_grid, int32_t accumulate, int32_t dtype,
                      void* stream);

/*
 * Forward with a per-query number of selected keys (adaptive k): logical row
 * r attends over its min(max(row_k[r], 1), topk) best keys, with the
 * softmax, LSE and output over those alone; the remaining slots of its index
 * row are -1 (and -inf in top_scores), which every backward entry point
 * treats as empty.  SparseDict predicts a per-token k_i and collapses it to
 * one budget before selection (models/moe_topk_restorer.py:333-338,
 * _effective_top_k; per-token k is listed future work, observations.md:63-65);
 * this keeps each token's own k.  row_k: device int32 [rows]; topk is the
 * largest k of the call.  Otherwise as sdk_topk_attn_fwd.
 */
int sdk_topk_attn_fwd_adaptive(const void* q, const void* k, const void* v, void* out, int32_t* top_idx,
                               void* lse, void* top_scores, const int32_t* row_offsets,
                               const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d,
                               int32_t dv, int32_t topk, double scale, int32_t score_grid,
                               const int32_t* row_k, int32_t dtype, void* stream);

/*
 * Forward with an additive score bias per (query row, key segment): the gate
 * fold of DualDomainMoEDictionary._mixture
 * (models/modules/dual_domain_moe.py:158-173), which adds log(max(g, tiny))
 * of token n's gate for expert e to the scores of expert e's atoms (-inf
 * where g == 0) before the top-k over the flat E*M atom axis.  Same as
 * sdk_topk_attn_fwd with
 *   score(r, j) = scale * q_r·k_j + seg_bias[r * segs + j / seg_len]
 * for logical row r; seg_bias is float (double for SDK_DTYPE_F64) and
 * seg_len * segs >= m.  Selection, lse and top_scores use the biased scores.
 * bf16/fp16 with d = dv = 64 and segments of whole 64-key tile quarters run on
 * the tensor cores, other shapes on the CUDA-core kernel.
 */
int sdk_topk_attn_fwd_biased(const void* q, const void* k, const void* v, void* out, int32_t* top_idx,
                             void* lse, void* top_scores, const int32_t* row_offsets,
                             const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d,
                             int32_t dv, int32_t topk, double scale, int32_t score_grid,
                             const void* seg_bias, int64_t seg_len, int32_t segs, int32_t dtype,
                             void* stream);

/*
 * Backward of sdk_topk_attn_fwd_biased (the score bias enters the recomputed
 * S).  dseg_bias (nullable, rows * segs, accumulator dtype) receives, per row
 * and segment, the sum of dS over the row's selected keys of that segment —
 * the gradient of the bias, from which the caller forms the gate gradient
 * dS_sum / g (models/modules/dual_domain_moe.py:164-166 under autograd).  It is
 * zeroed with the accumulators unless `accumulate` is nonzero.
 */
int sdk_topk_attn_bwd_biased(const void* q, const void* k, const void* v, const void* dout,
                             const int32_t* top_idx, const void* lse, void* dq, void* dk_acc,
                             void* dv_acc, const int32_t* row_offsets, const int32_t* row_index,
                             int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv,
                             int32_t topk, double scale, int32_t score_grid, int32_t accumulate,
                             const void* seg_bias, void* dseg_bias, int64_t seg_len, int32_t segs,
                             int32_t dtype, void* stream);

/*
 * Scratch bytes of sdk_topk_attn_bwd_direct for `rows` query rows (slices*n,
 * or the grouped row count with `grouped` nonzero), assuming 16-byte aligned
 * tensors: the key-major kernels' per-row statistics and per-key row lists
 * when the shape takes them (bf16/fp16, d = dv = 64, topk <= 64,
 * m <= 16384, at most 65535 rows per slice — grouped: in all, score_grid 0),
 * else fp32 (fp64) dK/dV accumulators.  0 for invalid sizes.
 */
size_t sdk_topk_attn_bwd_workspace_size(int64_t rows, int64_t slices, int64_t m, int32_t d, int32_t dv,
                                        int32_t topk, int32_t score_grid, int32_t grouped, int32_t dtype);

/*
 * The backward written straight into output-dtype gradients: dq [rows, d],
 * dk [slices, m, d] and dv [slices, m, dv_dim], all in `dtype` (the
 * reference returns dq·scale, dk·scale and dv in the input dtype,
 * kernels/fused_topk_attn.py:1195-1201).  dk == dv is allowed (d == dv_dim):
 * it then receives dK + dV (keys and values that are one dictionary).
 *
 * On the shapes of sdk_topk_attn_bwd_workspace_size's key-major case it runs
 * the deterministic key-major kernels: dq by a gathered contraction per query
 * row, dK/dV per key over the rows that selected it, in ascending row order —
 * no atomics, so the result is bit-identical from run to run, and every
 * element is written once (keys no row selected get zeros).  Other shapes
 * run the scatter kernel of sdk_topk_attn_bwd into accumulators in the
 * workspace and convert.  `workspace`: 256-byte aligned, at least
 * sdk_topk_attn_bwd_workspace_size bytes; SDK_ERR_INVALID_ARGUMENT otherwise.
 * Index -1 (a forward row given up on) contributes nothing.
 */
int sdk_topk_attn_bwd_direct(const void* q, const void* k, const void* v, const void* dout,
                             const int32_t* top_idx, const void* lse, void* dq, void* dk, void* dv,
                             const int32_t* row_offsets, const int32_t* row_index, int64_t slices,
                             int64_t n, int64_t m, int32_t d, int32_t dv_dim, int32_t topk, double scale,
                             int32_t score_grid, int32_t dtype, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Capacity, in fp32 elements (16 MiB), of the library-owned scratch array
 * that sdk_topk_attn_bwd_noalloc accumulates dK and dV in. */
#define SDK_NOALLOC_SCRATCH_FLOATS (4u * 1024u * 1024u)

/*
 * Backward without device allocation.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory — code running under
 * a memory budget owned by someone else (a host framework's pool, another
 * runtime that reserved the device) or on a latency-critical path where
 * cudaMalloc, which may synchronise the device, is not allowed — and so
 * cannot pass the accumulator buffers sdk_topk_attn_bwd needs.
 *
 * Computes the same gradients as sdk_topk_attn_bwd followed by
 * sdk_finalize_grad (uniform slices, no routing, score_grid 0), writing dq,
 * dk [slices, m, d] and dv [slices, m, dv_dim] in `dtype` (F32, BF16 or F16).
 * The fp32 accumulators live in a file-scope device array of
 * SDK_NOALLOC_SCRATCH_FLOATS elements that every GPU loading the library
 * holds until the process exits; a request needing more than
 * slices*m*(d+dv_dim) <= SDK_NOALLOC_SCRATCH_FLOATS is refused with
 * SDK_ERR_TOO_LARGE before anything runs.  The call allocates nothing.
 *
 * Every call looks up that array's device address (cudaGetSymbolAddress,
 * with the call's device current) before it launches anything; the first
 * call on a device also loads the library's device code there, so make that
 * first call before any stream capture.  All calls share the one array: each clears the
 * part it uses before accumulating, and calls that overlap on the GPU (on
 * different streams or from different host threads) race on it.
 */
int sdk_topk_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* dout,
                              const int32_t* top_idx, const float* lse, void* dq, void* dk, void* dv,
                              int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv_dim, int32_t topk,
                              double scale, int32_t dtype, void* stream);

/* Converts `count` accumulator elements (float32; float64 for F64) into
 * `dtype`, multiplying by `multiplier`.  `out` may alias `acc` only when the
 * element sizes match. */
int sdk_finalize_grad(const void* acc, void* out, int64_t count, double multiplier, int32_t dtype,
                      void* stream);

/*
 * Stage 1 alone: dense scores[n, m] (float32) = q[n, d] · k[m, d]ᵀ, with
 * row strides in elements.  Replaces tiled_affinity
 * (kernels/fused_topk_attn.py:227-287); dtype F32 or F16.
 */
int sdk_affinity(const void* q, const void* k, float* scores, int64_t n, int64_t m, int32_t d,
                 int64_t q_row_stride, int64_t k_row_stride, int32_t dtype, void* stream);

/*
 * Stage 2 alone: per-row top-k of scores[rows, m] (row stride in elements),
 * writing values (input dtype) and int64 indices.  Replaces tiled_topk
 * (kernels/fused_topk_attn.py:290-336, F32 or F16 there) and the torch.topk of
 * models/modules/topk_select.py:94-103 (any float dtype: F32, F16, BF16, F64).
 */
int sdk_topk_select(const void* scores, void* top_values, int64_t* top_idx, int64_t rows, int64_t m,
                    int64_t row_stride, int32_t topk, int32_t dtype, void* stream);

/*
 * Stage 3 alone: out[rows, dv] (float32) = softmax(top_scores) · values[top_idx].
 * Replaces tiled_topk_aggregate (kernels/fused_topk_attn.py:339-408).
 * score_dtype / value_dtype: F32 or F16; idx_bits: 32 or 64.  Indices outside
 * [0, m) contribute nothing and set device status bit 1.
 */
int sdk_topk_aggregate(const void* top_scores, const void* top_idx, const void* values, float* out,
                       int64_t rows, int32_t topk, int64_t m, int32_t dv, int64_t score_row_stride,
                       int64_t idx_row_stride, int64_t value_row_stride, int32_t score_dtype,
                       int32_t idx_bits, int32_t value_dtype, void* stream);

/*
 * Top-1 routing for the routed-dictionary configuration: expert[i] =
 * argmax_e logits[i, e] (lowest e on ties; models/modules/router.py:139-145),
 * then a stable counting sort: order[] lists rows grouped by expert and
 * offsets[e] .. offsets[e+1] delimits expert e's rows in it.
 * offsets needs experts+1 entries.  logits are float32; experts <= 16.
 * Three launches (per-block counts, their scan, placement); the block counts
 * live in stream-ordered scratch from the library pool.
 */
int sdk_route_top1(const float* logits, int64_t n, int32_t experts, int32_t* expert,
                   int32_t* order, int32_t* offsets, void* stream);

/*
 * Sparse top-k attention over given dense scores, after the selection
 * (sdk_topk_select): the body of sparse_topk_attention
 * (models/modules/topk_select.py:146-161).  For each of `rows` score rows with
 * selected scores top_scores[r, j] at keys top_idx[r, j] (int64, j < topk):
 *   out[r]           = sum_j softmax(top_scores[r])_j values[b, top_idx[r, j]]
 *   weights[r, :]    = 0 except the softmax weights at the selected keys
 *   masked_scores[r] = -inf except the selected scores at the selected keys
 * with values [batches, m, dv] and b = r / rows_per_batch (rows_per_batch 0:
 * one shared [m, dv] matrix).  top_scores, weights and masked_scores are in
 * score_dtype; values and out in out_dtype, which is score_dtype or the wider
 * of the two float types (F32 for F16/BF16 scores, F64).  topk <= 256.
 */
int sdk_sparse_topk_attn_fwd(const void* top_scores, const int64_t* top_idx, const void* values, void* out,
                             void* weights, void* masked_scores, int64_t rows, int64_t rows_per_batch,
                             int32_t topk, int64_t m, int32_t dv, int32_t score_dtype, int32_t out_dtype,
                             void* stream);

/*
 * Gradient of sdk_sparse_topk_attn_fwd with respect to the dense scores and
 * the values, given the gradients of out (grad_out, out_dtype) and, nullable,
 * of weights and masked_scores (dense, score_dtype).  grad_scores [rows, m]
 * (score_dtype) is written in full (zero off the selection); the values'
 * gradient is added to grad_values_acc [batches, m, dv] (float32, float64
 * when out_dtype is F64), which the caller zeroes first.
 */
int sdk_sparse_topk_attn_bwd(const void* top_scores, const int64_t* top_idx, const void* values,
                             const void* grad_out, const void* grad_weights, const void* grad_masked,
                             void* grad_scores, void* grad_values_acc, int64_t rows, int64_t rows_per_batch,
                             int32_t topk, int64_t m, int32_t dv, int32_t score_dtype, int32_t out_dtype,
                             void* stream);

/*
 * dst[r, :] = fill, then dst[r, idx[r, j]] = src[r, j] for rows r < rows,
 * j < k (idx int64, dst [rows, m], src [rows, k], both `dtype`): the hard
 * top-k mask (fill -inf, topk_select.py:94-103) and the straight-through
 * gradient of the selected scores (fill 0, :33-45).
 */
int sdk_fill_scatter(const void* src, const int64_t* idx, void* dst, int64_t rows, int32_t k, int64_t m,
                     double fill, int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSEDICT_B200_H_ */
