// extern "C" entry points of libsparsedict_b200.so (declared in
// include/sparsedict_b200.h).  Each validates its arguments, picks the
// kernel for the dtype/shape and launches on the caller's stream.  No
// exceptions cross this boundary.  The only device memory the library takes
// itself is the tensor-core forward's stream-ordered scratch when the caller
// passes no workspace (fwd_tc.cu) and the no-allocation backward's static
// array (bwd_noalloc.cu).
#include <atomic>
#include <cstdio>
#include <cstring>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace sdk {

__device__ unsigned int g_device_status;

namespace {
thread_local char g_last_cuda_error[256] = "";
std::atomic<uint64_t> g_wait_limit_ns{0};  // 0: the default bound

int record(cudaError_t err) {
  if (err == cudaSuccess) return SDK_OK;
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(err),
                cudaGetErrorString(err));
  return SDK_ERR_CUDA;
}

int finish(int rc) {
  if (rc == SDK_ERR_CUDA) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) record(err);
  }
  return rc;
}

bool dtype_ok(int32_t dtype) {
  return dtype == SDK_DTYPE_F32 || dtype == SDK_DTYPE_F64 || dtype == SDK_DTYPE_BF16 || dtype == SDK_DTYPE_F16;
}

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return SDK_ERR_NO_DEVICE;
  }
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
    cudaGetLastError();
    return SDK_ERR_NO_DEVICE;
  }
  return major == 10 ? SDK_OK : SDK_ERR_NO_DEVICE;
}
}  // namespace

int record_cuda_error(cudaError_t err) { return record(err); }

uint64_t wait_limit_ns() {
  const uint64_t v = g_wait_limit_ns.load(std::memory_order_relaxed);
  return v ? v : 2000000000ull;
}

// Device address of this library's status word in the current device's
// context (looked up on every call: a cheap host-side query, and no address
// outlives the context it was taken in).
unsigned int* device_status_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return static_cast<unsigned int*>(p);
}

// Stream-ordered scratch (the tensor-core forward's candidate buffer, the
// router's block counts): a memory pool of this library per device that keeps
// what it has reserved (no release at synchronisation), so repeated calls
// reuse the same device memory.
cudaMemPool_t scratch_pool() {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) return nullptr;
    uint64_t keep = ~0ull;
    if (cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess) return nullptr;
    pools[dev] = pool;
  }
  return pools[dev];
}

}  // namespace sdk

using namespace sdk;

extern "C" {

int sdk_version(void) { return (0 << 16) | 1; }

const char* sdk_status_string(int status) {
  switch (status) {
    case SDK_OK: return "ok";
    case SDK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SDK_ERR_UNSUPPORTED: return "unsupported by the library's kernels";
    case SDK_ERR_CUDA: return "CUDA error";
    case SDK_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    case SDK_ERR_TOO_LARGE: return "request exceeds the fixed scratch capacity of the no-allocation entry point";
    default: return "unknown status";
  }
}

const char* sdk_last_cuda_error(void) { return g_last_cuda_error; }

int sdk_max_topk(int32_t dtype, int32_t d) {
  if (!dtype_ok(dtype) || d <= 0) return 0;
  return max_topk_generic(dtype, d);
}

int sdk_set_wait_limit(uint64_t ns) {
  if (ns > 60000000000ull) return SDK_ERR_INVALID_ARGUMENT;
  g_wait_limit_ns.store(ns, std::memory_order_relaxed);
  return SDK_OK;
}

int sdk_device_status(unsigned int* bits, int32_t clear, void* stream) {
  if (!bits) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  unsigned int* p = device_status_ptr();
  if (!p) return record(cudaErrorInvalidSymbol);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = record(cudaMemcpyAsync(bits, p, sizeof(unsigned int), cudaMemcpyDeviceToHost, st))) return rc;
  if (clear)
    if (int rc = record(cudaMemsetAsync(p, 0, sizeof(unsigned int), st))) return rc;
  return record(cudaStreamSynchronize(st));
}

}  // extern "C"

namespace {

int fwd_impl(const void* q, const void* k, const void* v, void* out, int32_t* top_idx, void* lse, void* top_scores,
             const int32_t* row_offsets, const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d,
             int32_t dv, int32_t topk, double scale, int32_t score_grid, const void* seg_bias, int64_t seg_len,
             int32_t segs, int32_t dtype, void* stream, void* workspace = nullptr, size_t workspace_bytes = 0,
             const int32_t* row_k = nullptr) {
  if (!q || !k || !v || !out || !top_idx || !lse) return SDK_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype) || slices <= 0 || n < 0 || m <= 0 || d <= 0 || dv <= 0) return SDK_ERR_INVALID_ARGUMENT;
  if (topk < 1 || topk > m || m > 0x7ffffffe || !(scale > 0) || score_grid < 0) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  if (topk > max_topk_generic(dtype, d)) return SDK_ERR_UNSUPPORTED;
  FwdLaunch L{q, k, v, out, top_idx, lse, top_scores, row_offsets, row_index, slices, n, m, d, dv, topk,
              scale, score_grid, dtype, device_status_ptr(), static_cast<cudaStream_t>(stream)};
  L.seg_bias = seg_bias;
  L.seg_len = seg_len;
  L.segs = segs;
  L.workspace = workspace;
  L.workspace_bytes = workspace_bytes;
  L.row_k = row_k;
  if (fwd_tensorcore_supports(L)) return finish(fwd_tensorcore(L));
  return finish(fwd_generic(L));
}

int bwd_impl(const void* q, const void* k, const void* v, const void* dout, const int32_t* top_idx, const void* lse,
             void* dq, void* dk_acc, void* dv_acc, const int32_t* row_offsets, const int32_t* row_index,
             int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv, int32_t topk, double scale,
             int32_t score_grid, int32_t accumulate, const void* seg_bias, void* dseg_bias, int64_t seg_len,
             int32_t segs, int32_t dtype, void* stream) {
  if (!q || !k || !v || !dout || !top_idx || !lse || !dq || !dk_acc || !dv_acc) return SDK_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype) || slices <= 0 || n < 0 || m <= 0 || d <= 0 || dv <= 0) return SDK_ERR_INVALID_ARGUMENT;
  if (topk < 1 || topk > m || !(scale > 0) || score_grid < 0) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t acc_sz = dtype == SDK_DTYPE_F64 ? 8 : 4;
  if (!accumulate) {
    if (int rc = record(cudaMemsetAsync(dk_acc, 0, (size_t)slices * m * d * acc_sz, st))) return rc;
    if (dv_acc != dk_acc)
      if (int rc = record(cudaMemsetAsync(dv_acc, 0, (size_t)slices * m * dv * acc_sz, st))) return rc;
    if (dseg_bias) {
      const int64_t rows = row_offsets ? n : slices * n;
      if (int rc = record(cudaMemsetAsync(dseg_bias, 0, (size_t)rows * segs * acc_sz, st))) return rc;
    }
  }
  BwdLaunch L{q, k, v, dout, top_idx, lse, dq, dk_acc, dv_acc, row_offsets, row_index, slices, n, m, d, dv, topk,
              scale, score_grid, dtype, device_status_ptr(), st};
  L.seg_bias = seg_bias;
  L.dseg_bias = dseg_bias;
  L.seg_len = seg_len;
  L.segs = segs;
  return finish(bwd_sparse(L));
}

// Backward into output-dtype dK/dV: the key-major kernels when the shape
// takes them, else the scatter kernel into fp32 (fp64) accumulators carved
// from the workspace, then one conversion.  Returns the bytes needed.
size_t bwd_direct_bytes(int64_t rows, int64_t slices, int64_t m, int32_t d, int32_t dv, int32_t topk,
                        int32_t score_grid, bool grouped, int32_t dtype, int64_t n, bool alias, bool aligned) {
  BwdLaunch probe{};
  probe.dtype = dtype;
  probe.d = d;
  probe.dv = dv;
  probe.topk = topk;
  probe.score_grid = score_grid;
  probe.m = m;
  probe.n = n;
  probe.slices = slices;
  probe.row_offsets = grouped ? reinterpret_cast<const int32_t*>(16) : nullptr;
  const void* p16 = reinterpret_cast<const void*>(aligned ? 256 : 1);
  probe.q = probe.k = probe.v = probe.dout = p16;
  probe.dq = const_cast<void*>(p16);
  if (bwd_keymajor_supports(probe)) return bwd_keymajor_workspace(rows, slices, m, topk);
  const size_t acc = dtype == SDK_DTYPE_F64 ? 8 : 4;
  return (size_t)slices * (size_t)m * (size_t)(d + (alias ? 0 : dv)) * acc + 256;
}

bool segments_ok(const void* seg_bias, int64_t seg_len, int32_t segs, int64_t m) {
  return seg_bias && seg_len >= 1 && segs >= 1 && seg_len * (int64_t)segs >= m;
}

}  // namespace

extern "C" {

int sdk_topk_attn_fwd(const void* q, const void* k, const void* v, void* out, int32_t* top_idx, void* lse,
                      void* top_scores, const int32_t* row_offsets, const int32_t* row_index, int64_t slices,
                      int64_t n, int64_t m, int32_t d, int32_t dv, int32_t topk, double scale, int32_t score_grid,
                      int32_t dtype, void* stream) {
  return fwd_impl(q, k, v, out, top_idx, lse, top_scores, row_offsets, row_index, slices, n, m, d, dv, topk, scale,
                  score_grid, nullptr, 0, 0, dtype, stream);
}

int sdk_topk_attn_fwd_adaptive(const void* q, const void* k, const void* v, void* out, int32_t* top_idx, void* lse,
                               void* top_scores, const int32_t* row_offsets, const int32_t* row_index,
                               int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv, int32_t topk,
                               double scale, int32_t score_grid, const int32_t* row_k, int32_t dtype, void* stream) {
  if (!row_k) return SDK_ERR_INVALID_ARGUMENT;
  return fwd_impl(q, k, v, out, top_idx, lse, top_scores, row_offsets, row_index, slices, n, m, d, dv, topk, scale,
                  score_grid, nullptr, 0, 0, dtype, stream, nullptr, 0, row_k);
}

size_t sdk_topk_attn_fwd_workspace_size(int64_t rows, int64_t m, int32_t d, int32_t dv, int32_t topk,
                                        int32_t score_grid, int32_t grouped, int32_t dtype) {
  return fwd_tensorcore_workspace(rows, m, d, dv, topk, score_grid, grouped != 0, dtype);
}

int sdk_topk_attn_fwd_ws(const void* q, const void* k, const void* v, void* out, int32_t* top_idx, void* lse,
                         void* top_scores, const int32_t* row_offsets, const int32_t* row_index, int64_t slices,
                         int64_t n, int64_t m, int32_t d, int32_t dv, int32_t topk, double scale,
                         int32_t score_grid, int32_t dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace && workspace_bytes) return SDK_ERR_INVALID_ARGUMENT;
  return fwd_impl(q, k, v, out, top_idx, lse, top_scores, row_offsets, row_index, slices, n, m, d, dv, topk, scale,
                  score_grid, nullptr, 0, 0, dtype, stream, workspace, workspace_bytes);
}

int sdk_topk_attn_bwd(const void* q, const void* k, const void* v, const void* dout, const int32_t* top_idx,
                      const void* lse, void* dq, void* dk_acc, void* dv_acc, const int32_t* row_offsets,
                      const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv,
                      int32_t topk, double scale, int32_t score_grid, int32_t accumulate, int32_t dtype,
                      void* stream) {
  return bwd_impl(q, k, v, dout, top_idx, lse, dq, dk_acc, dv_acc, row_offsets, row_index, slices, n, m, d, dv, topk,
                  scale, score_grid, accumulate, nullptr, nullptr, 0, 0, dtype, stream);
}

int sdk_topk_attn_fwd_biased(const void* q, const void* k, const void* v, void* out, int32_t* top_idx, void* lse,
                             void* top_scores, const int32_t* row_offsets, const int32_t* row_index,
                             int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv, int32_t topk,
                             double scale, int32_t score_grid, const void* seg_bias, int64_t seg_len,
                             int32_t segs, int32_t dtype, void* stream) {
  if (!segments_ok(seg_bias, seg_len, segs, m)) return SDK_ERR_INVALID_ARGUMENT;
  return fwd_impl(q, k, v, out, top_idx, lse, top_scores, row_offsets, row_index, slices, n, m, d, dv, topk, scale,
                  score_grid, seg_bias, seg_len, segs, dtype, stream);
}

int sdk_topk_attn_bwd_biased(const void* q, const void* k, const void* v, const void* dout, const int32_t* top_idx,
                             const void* lse, void* dq, void* dk_acc, void* dv_acc, const int32_t* row_offsets,
                             const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv,
                             int32_t topk, double scale, int32_t score_grid, int32_t accumulate,
                             const void* seg_bias, void* dseg_bias, int64_t seg_len, int32_t segs, int32_t dtype,
                             void* stream) {
  if (!segments_ok(seg_bias, seg_len, segs, m)) return SDK_ERR_INVALID_ARGUMENT;
  return bwd_impl(q, k, v, dout, top_idx, lse, dq, dk_acc, dv_acc, row_offsets, row_index, slices, n, m, d, dv, topk,
                  scale, score_grid, accumulate, seg_bias, dseg_bias, seg_len, segs, dtype, stream);
}

size_t sdk_topk_attn_bwd_workspace_size(int64_t rows, int64_t slices, int64_t m, int32_t d, int32_t dv,
                                        int32_t topk, int32_t score_grid, int32_t grouped, int32_t dtype) {
  if (rows < 0 || slices <= 0 || m <= 0 || d <= 0 || dv <= 0 || topk < 1 || !dtype_ok(dtype)) return 0;
  // the per-slice row limit of the key-major kernels is checked against the
  // largest slice: rows (grouped) or rows / slices (uniform)
  const int64_t n = grouped ? rows : rows / slices;
  return bwd_direct_bytes(rows, slices, m, d, dv, topk, score_grid, grouped != 0, dtype, n, false, true);
}

int sdk_topk_attn_bwd_direct(const void* q, const void* k, const void* v, const void* dout, const int32_t* top_idx,
                             const void* lse, void* dq, void* dk, void* dv, const int32_t* row_offsets,
                             const int32_t* row_index, int64_t slices, int64_t n, int64_t m, int32_t d,
                             int32_t dv_dim, int32_t topk, double scale, int32_t score_grid, int32_t dtype,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !dout || !top_idx || !lse || !dq || !dk || !dv) return SDK_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype) || slices <= 0 || n < 0 || m <= 0 || d <= 0 || dv_dim <= 0) return SDK_ERR_INVALID_ARGUMENT;
  if (topk < 1 || topk > m || !(scale > 0) || score_grid < 0) return SDK_ERR_INVALID_ARGUMENT;
  if (dk == dv && d != dv_dim) return SDK_ERR_INVALID_ARGUMENT;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255)) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = row_offsets ? n : slices * n;
  BwdLaunch L{q, k, v, dout, top_idx, lse, dq, nullptr, nullptr, row_offsets, row_index, slices, n, m, d, dv_dim, topk,
              scale, score_grid, dtype, device_status_ptr(), st};
  const bool alias = dk == dv;
  if (bwd_keymajor_supports(L)) {
    if (workspace_bytes < bwd_keymajor_workspace(rows, slices, m, topk)) return SDK_ERR_INVALID_ARGUMENT;
    return finish(bwd_keymajor(L, dk, dv, 0, 0, workspace));
  }
  const size_t acc_sz = dtype == SDK_DTYPE_F64 ? 8 : 4;
  const size_t dk_bytes = (size_t)slices * m * d * acc_sz;
  const size_t need = dk_bytes + (alias ? 0 : (size_t)slices * m * dv_dim * acc_sz);
  if (workspace_bytes < need) return SDK_ERR_INVALID_ARGUMENT;
  L.dk_acc = workspace;
  L.dv_acc = alias ? workspace : static_cast<uint8_t*>(workspace) + dk_bytes;
  if (int rc = record(cudaMemsetAsync(workspace, 0, need, st))) return rc;
  int rc = bwd_sparse(L);
  if (rc == SDK_OK) rc = finalize_grad(L.dk_acc, dk, slices * m * d, 1.0, dtype, st);
  if (rc == SDK_OK && !alias) rc = finalize_grad(L.dv_acc, dv, slices * m * dv_dim, 1.0, dtype, st);
  return finish(rc);
}

int sdk_finalize_grad(const void* acc, void* out, int64_t count, double multiplier, int32_t dtype, void* stream) {
  if (!acc || !out || count < 0 || !dtype_ok(dtype)) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  return finish(finalize_grad(acc, out, count, multiplier, dtype, static_cast<cudaStream_t>(stream)));
}

int sdk_affinity(const void* q, const void* k, float* scores, int64_t n, int64_t m, int32_t d, int64_t q_row_stride,
                 int64_t k_row_stride, int32_t dtype, void* stream) {
  if (!q || !k || !scores || n <= 0 || m <= 0 || d <= 0 || q_row_stride < d || k_row_stride < d)
    return SDK_ERR_INVALID_ARGUMENT;
  if (dtype != SDK_DTYPE_F32 && dtype != SDK_DTYPE_F16) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  return finish(affinity(q, k, scores, n, m, d, q_row_stride, k_row_stride, dtype, static_cast<cudaStream_t>(stream)));
}

int sdk_topk_select(const void* scores, void* top_values, int64_t* top_idx, int64_t rows, int64_t m,
                    int64_t row_stride, int32_t topk, int32_t dtype, void* stream) {
  if (!scores || !top_values || !top_idx || rows <= 0 || m <= 0 || row_stride < m) return SDK_ERR_INVALID_ARGUMENT;
  if (topk < 1 || topk > m || m > 0x7ffffffe) return SDK_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype)) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  return finish(topk_select(scores, top_values, top_idx, rows, m, row_stride, topk, dtype,
                            static_cast<cudaStream_t>(stream)));
}

int sdk_topk_aggregate(const void* top_scores, const void* top_idx, const void* values, float* out, int64_t rows,
                       int32_t topk, int64_t m, int32_t dv, int64_t score_row_stride, int64_t idx_row_stride,
                       int64_t value_row_stride, int32_t score_dtype, int32_t idx_bits, int32_t value_dtype,
                       void* stream) {
  if (!top_scores || !top_idx || !values || !out || rows <= 0 || topk <= 0 || m <= 0 || dv <= 0)
    return SDK_ERR_INVALID_ARGUMENT;
  if (score_row_stride < topk || idx_row_stride < topk || value_row_stride < dv) return SDK_ERR_INVALID_ARGUMENT;
  if (idx_bits != 32 && idx_bits != 64) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  return finish(topk_aggregate(top_scores, top_idx, values, out, rows, topk, m, dv, score_row_stride,
                               idx_row_stride, value_row_stride, score_dtype, idx_bits, value_dtype,
                               device_status_ptr(), static_cast<cudaStream_t>(stream)));
}

int sdk_sparse_topk_attn_fwd(const void* top_scores, const int64_t* top_idx, const void* values, void* out,
                             void* weights, void* masked_scores, int64_t rows, int64_t rows_per_batch, int32_t topk,
                             int64_t m, int32_t dv, int32_t score_dtype, int32_t out_dtype, void* stream) {
  if (!top_scores || !top_idx || !values || !out || !weights || !masked_scores) return SDK_ERR_INVALID_ARGUMENT;
  if (rows < 0 || rows_per_batch < 0 || topk < 1 || topk > 256 || topk > m || dv < 1) return SDK_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(score_dtype) || !dtype_ok(out_dtype)) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  if (rows == 0) return SDK_OK;
  return finish(sparse_attn_forward(top_scores, top_idx, values, out, weights, masked_scores, rows, rows_per_batch,
                                    topk, m, dv, score_dtype, out_dtype, device_status_ptr(),
                                    static_cast<cudaStream_t>(stream)));
}

int sdk_sparse_topk_attn_bwd(const void* top_scores, const int64_t* top_idx, const void* values, const void* grad_out,
                             const void* grad_weights, const void* grad_masked, void* grad_scores,
                             void* grad_values_acc, int64_t rows, int64_t rows_per_batch, int32_t topk, int64_t m,
                             int32_t dv, int32_t score_dtype, int32_t out_dtype, void* stream) {
  if (!top_scores || !top_idx || !values || !grad_out || !grad_scores || !grad_values_acc)
    return SDK_ERR_INVALID_ARGUMENT;
  if (rows < 0 || rows_per_batch < 0 || topk < 1 || topk > 256 || topk > m || dv < 1) return SDK_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(score_dtype) || !dtype_ok(out_dtype)) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  if (rows == 0) return SDK_OK;
  return finish(sparse_attn_backward(top_scores, top_idx, values, grad_out, grad_weights, grad_masked, grad_scores,
                                     grad_values_acc, rows, rows_per_batch, topk, m, dv, score_dtype, out_dtype,
                                     device_status_ptr(), static_cast<cudaStream_t>(stream)));
}

int sdk_fill_scatter(const void* src, const int64_t* idx, void* dst, int64_t rows, int32_t k, int64_t m, double fill,
                     int32_t dtype, void* stream) {
  if (!src || !idx || !dst || rows < 0 || k < 1 || m < 1 || !dtype_ok(dtype)) return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  if (rows == 0) return SDK_OK;
  return finish(fill_scatter(src, idx, dst, rows, k, m, fill, dtype, device_status_ptr(),
                             static_cast<cudaStream_t>(stream)));
}

int sdk_route_top1(const float* logits, int64_t n, int32_t experts, int32_t* expert, int32_t* order,
                   int32_t* offsets, void* stream) {
  if (!logits || !expert || !order || !offsets || n <= 0 || n > 0x7fffffff || experts <= 0)
    return SDK_ERR_INVALID_ARGUMENT;
  if (int rc = check_device()) return rc;
  return finish(route_top1(logits, n, experts, expert, order, offsets, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
