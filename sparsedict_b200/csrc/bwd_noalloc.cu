// Sparse backward for callers that cannot allocate device memory.
//
// sdk_topk_attn_bwd needs fp32 dK/dV accumulator buffers from the caller.
// Some callers cannot provide them: code that runs under a device-memory
// budget owned by someone else (a host framework's memory pool, another
// runtime that has reserved the device), or code on a latency-critical path
// where cudaMalloc, which may synchronise the device, is not acceptable.
// sdk_topk_attn_bwd_noalloc serves them: its accumulators live in one
// fixed-size array of device memory that belongs to this library, so the
// caller passes only inputs and outputs.
//
// The array is `g_noalloc_scratch` below: SDK_NOALLOC_SCRATCH_FLOATS fp32
// elements (16 MiB), held on every GPU that loads the library until the
// process exits.  Its name is only a host-side stand-in in host code; the
// device address is looked up with cudaGetSymbolAddress on every call, with
// the call's device current (a cheap host-side query), so no address outlives
// the context it was taken in (a cudaDeviceReset between calls included).

#include "common.cuh"
#include "kernels.h"

namespace sdk {
namespace {

static __device__ __align__(256) float g_noalloc_scratch[SDK_NOALLOC_SCRATCH_FLOATS];

// Device address of the scratch array in the current device's context.
int noalloc_scratch(float** out) {
  void* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (err != cudaSuccess) return record_cuda_error(err);
  *out = static_cast<float*>(p);
  return SDK_OK;
}

}  // namespace
}  // namespace sdk

using namespace sdk;

extern "C" int sdk_topk_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* dout,
                                         const int32_t* top_idx, const float* lse, void* dq, void* dk, void* dv,
                                         int64_t slices, int64_t n, int64_t m, int32_t d, int32_t dv_dim,
                                         int32_t topk, double scale, int32_t dtype, void* stream) {
  if (!q || !k || !v || !dout || !top_idx || !lse || !dq || !dk || !dv) return SDK_ERR_INVALID_ARGUMENT;
  if (slices <= 0 || n < 0 || m <= 0 || d <= 0 || dv_dim <= 0) return SDK_ERR_INVALID_ARGUMENT;
  if (topk < 1 || topk > m || !(scale > 0)) return SDK_ERR_INVALID_ARGUMENT;
  if (dtype != SDK_DTYPE_F32 && dtype != SDK_DTYPE_BF16 && dtype != SDK_DTYPE_F16) return SDK_ERR_UNSUPPORTED;
  const int64_t dk_elems = slices * m * d, dv_elems = slices * m * dv_dim;
  if (dk_elems > (int64_t)SDK_NOALLOC_SCRATCH_FLOATS - dv_elems) return SDK_ERR_TOO_LARGE;
  int major = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10) {
    cudaGetLastError();
    return SDK_ERR_NO_DEVICE;
  }
  float* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's sums: clear the part this call uses
  cudaError_t err = cudaMemsetAsync(scratch, 0, (size_t)(dk_elems + dv_elems) * sizeof(float), st);
  if (err != cudaSuccess) return record_cuda_error(err);
  BwdLaunch L{q, k, v, dout, top_idx, lse, dq, scratch, scratch + dk_elems, nullptr, nullptr, slices, n, m, d,
              dv_dim, topk, scale, 0, dtype, device_status_ptr(), st};
  int rc = bwd_sparse(L);
  if (rc == SDK_OK) rc = finalize_grad(scratch, dk, dk_elems, 1.0, dtype, st);
  if (rc == SDK_OK) rc = finalize_grad(scratch + dk_elems, dv, dv_elems, 1.0, dtype, st);
  if (rc == SDK_ERR_CUDA) {
    err = cudaGetLastError();
    if (err != cudaSuccess) record_cuda_error(err);
  }
  return rc;
}
