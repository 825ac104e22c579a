// Internal launch descriptors shared by the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/sparsedict_b200.h"

namespace sdk {

constexpr size_t kMaxDynamicSmem = 227 * 1024;

inline int next_pow2_host(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

struct FwdLaunch {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int32_t* top_idx;
  void* lse;
  void* top_scores;
  const int32_t* row_offsets;
  const int32_t* row_index;
  int64_t slices, n, m;
  int d, dv, topk;
  double scale;
  int score_grid;
  int dtype;
  unsigned int* status;
  cudaStream_t stream;
  // Optional additive score bias per (logical query row, key segment):
  // score(r, j) += seg_bias[r * segs + j / seg_len], after the scale.  In the
  // accumulator type (double for fp64 inputs, float otherwise).
  const void* seg_bias = nullptr;
  int64_t seg_len = 0;
  int segs = 0;
  // Optional per-row number of selected keys (adaptive k): logical row r keeps
  // its min(max(row_k[r], 1), topk) best keys; the other slots of its index row
  // are -1 (and -inf in top_scores).  Null: topk for every row.
  const int32_t* row_k = nullptr;
  // Scratch of the tensor-core forward (fwd_tensorcore_workspace bytes, 16-byte
  // aligned); null: stream-ordered scratch from this library's memory pool.
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
};

struct BwdLaunch {
  const void* q;
  const void* k;
  const void* v;
  const void* dout;
  const int32_t* top_idx;
  const void* lse;
  void* dq;
  void* dk_acc;
  void* dv_acc;
  const int32_t* row_offsets;
  const int32_t* row_index;
  int64_t slices, n, m;
  int d, dv, topk;
  double scale;
  int score_grid;
  int dtype;
  unsigned int* status;
  cudaStream_t stream;
  // Optional score bias as in FwdLaunch; dseg_bias (nullable, zeroed by the
  // caller, rows * segs) receives the sum of dS over each row's selected keys
  // of each segment.
  const void* seg_bias = nullptr;
  void* dseg_bias = nullptr;
  int64_t seg_len = 0;
  int segs = 0;
};

// Bound of each pipeline wait of the tensor-core forward, in ns
// (sdk_set_wait_limit; default sm100::kWaitLimitNs).  Defined in capi.cu.
uint64_t wait_limit_ns();

// Records a CUDA error for sdk_last_cuda_error(); returns SDK_ERR_CUDA (or
// SDK_OK for cudaSuccess).  Defined in capi.cu.
int record_cuda_error(cudaError_t err);

// CUDA-core fused forward (fwd_generic.cu).
int fwd_generic(const FwdLaunch& L);
int max_topk_generic(int dtype, int d);

// Tensor-core (tcgen05) bf16/fp16 forward (fwd_tc.cu); returns
// SDK_ERR_UNSUPPORTED for shapes it does not take.
int fwd_tensorcore(const FwdLaunch& L);
bool fwd_tensorcore_supports(const FwdLaunch& L);
// Scratch bytes the tensor-core forward needs for `rows` query rows when the
// shape takes that path (bf16/fp16, d = dv = 64, topk <= 64, m <= 65536,
// score_grid 0, not grouped or routed), else 0.
size_t fwd_tensorcore_workspace(int64_t rows, int64_t m, int d, int dv, int topk, int score_grid, bool grouped,
                                int dtype);

// Sparse backward (bwd.cu).
int bwd_sparse(const BwdLaunch& L);

// Deterministic key-major backward (bwd_km.cu): bf16/fp16, d = dv = 64,
// topk <= 64, m <= 16384, at most 65535 rows per slice.  Writes dq and dk/dv
// (input dtype, or fp32 accumulators when out_acc; dk == dv sums both) with
// no atomics; `ws` holds bwd_keymajor_workspace bytes (256-byte aligned).
bool bwd_keymajor_supports(const BwdLaunch& L);
size_t bwd_keymajor_workspace(int64_t rows, int64_t slices, int64_t m, int topk);
int bwd_keymajor(const BwdLaunch& L, void* dk, void* dv, int out_acc, int accumulate, void* ws);
int finalize_grad(const void* acc, void* out, int64_t count, double multiplier, int dtype,
                  cudaStream_t stream);

// Dense fp16 affinity on the tensor cores (affinity_tc.cu): fp16, d >= 64,
// 16-byte aligned rows; `affinity` routes such calls there.
bool affinity_tensorcore_supports(const void* q, const void* k, int64_t n, int64_t m, int d, int64_t q_stride,
                                  int64_t k_stride, int dtype);
int affinity_tensorcore(const void* q, const void* k, float* scores, int64_t n, int64_t m, int d,
                        int64_t q_stride, int64_t k_stride, cudaStream_t stream);

// Stage ops (stages.cu).
int affinity(const void* q, const void* k, float* scores, int64_t n, int64_t m, int d,
             int64_t q_stride, int64_t k_stride, int dtype, cudaStream_t stream);
int topk_select(const void* scores, void* top_values, int64_t* top_idx, int64_t rows, int64_t m,
                int64_t row_stride, int topk, int dtype, cudaStream_t stream);
int topk_aggregate(const void* top_scores, const void* top_idx, const void* values, float* out,
                   int64_t rows, int topk, int64_t m, int dv, int64_t score_stride,
                   int64_t idx_stride, int64_t value_stride, int score_dtype, int idx_bits,
                   int value_dtype, unsigned int* status, cudaStream_t stream);
int route_top1(const float* logits, int64_t n, int experts, int32_t* expert, int32_t* order,
               int32_t* offsets, cudaStream_t stream);

// Sparse top-k attention over given dense scores (select_attn.cu).
int sparse_attn_forward(const void* sel, const int64_t* idx, const void* values, void* out, void* weights,
                        void* masked, int64_t rows, int64_t rows_per_batch, int k, int64_t m, int dv, int score_dtype,
                        int out_dtype, unsigned int* status, cudaStream_t stream);
int sparse_attn_backward(const void* sel, const int64_t* idx, const void* values, const void* g_out,
                         const void* g_weights, const void* g_masked, void* g_scores, void* g_values, int64_t rows,
                         int64_t rows_per_batch, int k, int64_t m, int dv, int score_dtype, int out_dtype,
                         unsigned int* status, cudaStream_t stream);
int fill_scatter(const void* src, const int64_t* idx, void* dst, int64_t rows, int k, int64_t m, double fill,
                 int dtype, unsigned int* status, cudaStream_t stream);

}  // namespace sdk
