// Sparse top-k attention over given dense scores: the body of
// sparse_topk_attention (models/modules/topk_select.py:106-162) after the
// top-k selection, and its gradient, as warp-per-row kernels.
//
// For each score row r (of batch b = r / rows_per_batch; one shared value
// matrix when rows_per_batch is 0) with selected scores s_j at keys i_j:
//   p_j = softmax(s)_j                         (over the k selected scores)
//   out[r]         = sum_j p_j values[b, i_j]
//   weights[r, :]  = 0,   weights[r, i_j] = p_j
//   masked[r, :]   = -inf, masked[r, i_j] = s_j
// Backward, given the gradients of out, weights and masked:
//   G_j  = g_weights[r, i_j] + g_out[r]·values[b, i_j]
//   ds_j = p_j (G_j - sum_l p_l G_l) + g_masked[r, i_j]
//   g_scores[r, :] = 0, g_scores[r, i_j] = ds_j
//   g_values[b, i_j] += p_j g_out[r]           (fp32/fp64 atomics)
// A separate warp-per-row kernel fills a dense row with a constant and
// scatters k values into it (the gradient of the selected scores, the hard
// top-k mask).
#include "common.cuh"
#include "kernels.h"

namespace sdk {
namespace {

constexpr int SW = 8;   // warps per block
constexpr int NPL = 8;  // selected entries per lane (k <= 256)

__device__ __forceinline__ void atomic_add_acc(float* p, float x) { atomicAdd(p, x); }
__device__ __forceinline__ void atomic_add_acc(double* p, double x) { atomicAdd(p, x); }

template <typename T, typename Acc>
__device__ __forceinline__ T out_cast(Acc x) {
  if constexpr (std::is_same<T, double>::value) return (double)x;
  else return from_acc<T>((float)x);
}

template <typename T>
__device__ __forceinline__ auto in_cast(T x) {
  return to_acc(x);
}

// Fill row r of dst [rows, m] with `fill`, then dst[r, idx[r, j]] = src[r, j].
template <typename T>
__global__ void __launch_bounds__(SW * kWarp) fill_scatter_kernel(const T* __restrict__ src,
                                                                  const int64_t* __restrict__ idx, T* dst,
                                                                  int64_t rows, int k, int64_t m, T fill,
                                                                  unsigned int* status) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * SW + warp; r < rows; r += (int64_t)gridDim.x * SW) {
    T* row = dst + r * m;
    for (int64_t c = lane; c < m; c += kWarp) row[c] = fill;
    __syncwarp();
    for (int j = lane; j < k; j += kWarp) {
      const int64_t c = idx[r * k + j];
      if (c < 0 || c >= m) {
        raise_device_status(status, kStatusIndexOutOfRange);
        continue;
      }
      row[c] = src[r * k + j];
    }
    __syncwarp();
  }
}

// Softmax weights of one row's selected scores, lane j holding entries
// j, j + 32, ... (k <= 256: NPL per lane).
template <typename Acc, typename TS>
__device__ __forceinline__ void row_softmax(const TS* srow, int k, int lane, Acc (&p)[NPL]) {
  Acc mx = neg_inf<Acc>();
#pragma unroll
  for (int u = 0; u < NPL; ++u) {
    const int j = lane + kWarp * u;
    p[u] = j < k ? (Acc)in_cast(srow[j]) : neg_inf<Acc>();
    mx = mx > p[u] ? mx : p[u];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const Acc y = __shfl_xor_sync(0xffffffffu, mx, o);
    mx = mx > y ? mx : y;
  }
  Acc tot = 0;
#pragma unroll
  for (int u = 0; u < NPL; ++u) {
    const int j = lane + kWarp * u;
    p[u] = j < k ? exp_acc(p[u] - mx) : (Acc)0;  // all -inf: NaN, as a softmax gives
    tot += p[u];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
#pragma unroll
  for (int u = 0; u < NPL; ++u) p[u] = p[u] / tot;
}

template <typename TS, typename TO>
__global__ void __launch_bounds__(SW * kWarp) sparse_attn_fwd_kernel(
    const TS* __restrict__ sel, const int64_t* __restrict__ idx, const TO* __restrict__ values, TO* __restrict__ out,
    TS* weights, TS* masked, int64_t rows, int64_t rows_per_batch, int k, int64_t m, int dv, unsigned int* status) {
  using Acc = typename AccOf<TO>::type;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * SW + warp; r < rows; r += (int64_t)gridDim.x * SW) {
    const TO* vb = values + (rows_per_batch ? (r / rows_per_batch) * m * dv : 0);
    Acc p[NPL];
    row_softmax<Acc>(sel + r * k, k, lane, p);
    // dense weights and masked scores: fill, then the k entries
    for (int64_t c = lane; c < m; c += kWarp) {
      weights[r * m + c] = out_cast<TS, Acc>((Acc)0);
      masked[r * m + c] = out_cast<TS, Acc>(neg_inf<Acc>());
    }
    __syncwarp();
    int key[NPL];
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      const int j = lane + kWarp * u;
      key[u] = j < k ? (int)idx[r * k + j] : -1;
      if (j < k && (key[u] < 0 || key[u] >= m)) {
        raise_device_status(status, kStatusIndexOutOfRange);
        key[u] = -1;
      }
      if (key[u] >= 0) {
        weights[r * m + key[u]] = out_cast<TS, Acc>(p[u]);
        masked[r * m + key[u]] = sel[r * k + j];
      }
    }
    // out[r, f] = sum_j p_j values[i_j, f]: lanes over features, selections in order
    for (int f0 = 0; f0 < dv; f0 += kWarp) {
      const int f = f0 + lane;
      Acc acc = 0;
#pragma unroll
      for (int u = 0; u < NPL; ++u)
        for (int l = 0; l < kWarp && kWarp * u + l < k; ++l) {
          const int kj = __shfl_sync(0xffffffffu, key[u], l);
          const Acc pj = __shfl_sync(0xffffffffu, p[u], l);
          if (kj >= 0 && f < dv) acc += pj * (Acc)in_cast(vb[(int64_t)kj * dv + f]);
        }
      if (f < dv) out[r * dv + f] = out_cast<TO, Acc>(acc);
    }
  }
}

template <typename TS, typename TO>
__global__ void __launch_bounds__(SW * kWarp) sparse_attn_bwd_kernel(
    const TS* __restrict__ sel, const int64_t* __restrict__ idx, const TO* __restrict__ values,
    const TO* __restrict__ g_out, const TS* __restrict__ g_weights, const TS* __restrict__ g_masked, TS* g_scores,
    typename AccOf<TO>::type* g_values, int64_t rows, int64_t rows_per_batch, int k, int64_t m, int dv,
    unsigned int* status) {
  using Acc = typename AccOf<TO>::type;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * SW + warp; r < rows; r += (int64_t)gridDim.x * SW) {
    const int64_t boff = rows_per_batch ? (r / rows_per_batch) * m * dv : 0;
    const TO* vb = values + boff;
    Acc p[NPL];
    row_softmax<Acc>(sel + r * k, k, lane, p);
    int key[NPL];
    Acc G[NPL];
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      const int j = lane + kWarp * u;
      key[u] = j < k ? (int)idx[r * k + j] : -1;
      if (j < k && (key[u] < 0 || key[u] >= m)) {
        raise_device_status(status, kStatusIndexOutOfRange);
        key[u] = -1;
      }
      G[u] = (key[u] >= 0 && g_weights) ? (Acc)in_cast(g_weights[r * m + key[u]]) : (Acc)0;
    }
    // G_j += g_out[r]·values[i_j]: lanes over features, one warp sum per selection
#pragma unroll
    for (int u = 0; u < NPL; ++u)
      for (int l = 0; l < kWarp && kWarp * u + l < k; ++l) {
        const int kj = __shfl_sync(0xffffffffu, key[u], l);
        Acc part = 0;
        if (kj >= 0)
          for (int f = lane; f < dv; f += kWarp)
            part += (Acc)in_cast(g_out[r * dv + f]) * (Acc)in_cast(vb[(int64_t)kj * dv + f]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (l == lane) G[u] += part;
      }
    Acc delta = 0;
#pragma unroll
    for (int u = 0; u < NPL; ++u) delta += (key[u] >= 0) ? p[u] * G[u] : (Acc)0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) delta += __shfl_xor_sync(0xffffffffu, delta, o);
    for (int64_t c = lane; c < m; c += kWarp) g_scores[r * m + c] = out_cast<TS, Acc>((Acc)0);
    __syncwarp();
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      if (key[u] < 0) continue;
      Acc ds = p[u] * (G[u] - delta);
      if (g_masked) ds += (Acc)in_cast(g_masked[r * m + key[u]]);
      g_scores[r * m + key[u]] = out_cast<TS, Acc>(ds);
    }
    // g_values[b, i_j] += p_j g_out[r]
#pragma unroll
    for (int u = 0; u < NPL; ++u)
      for (int l = 0; l < kWarp && kWarp * u + l < k; ++l) {
        const int kj = __shfl_sync(0xffffffffu, key[u], l);
        const Acc pj = __shfl_sync(0xffffffffu, p[u], l);
        if (kj < 0) continue;
        for (int f = lane; f < dv; f += kWarp)
          atomic_add_acc(&g_values[boff + (int64_t)kj * dv + f], pj * (Acc)in_cast(g_out[r * dv + f]));
      }
  }
}

unsigned grid_for(int64_t rows) {
  const int64_t want = (rows + SW - 1) / SW;
  return (unsigned)(want < 148 * 64 ? want : 148 * 64);
}

template <typename TS, typename TO>
int fwd_t(const void* sel, const int64_t* idx, const void* values, void* out, void* weights, void* masked,
          int64_t rows, int64_t rpb, int k, int64_t m, int dv, unsigned int* status, cudaStream_t st) {
  sparse_attn_fwd_kernel<TS, TO><<<grid_for(rows), SW * kWarp, 0, st>>>(
      static_cast<const TS*>(sel), idx, static_cast<const TO*>(values), static_cast<TO*>(out),
      static_cast<TS*>(weights), static_cast<TS*>(masked), rows, rpb, k, m, dv, status);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

template <typename TS, typename TO>
int bwd_t(const void* sel, const int64_t* idx, const void* values, const void* g_out, const void* g_weights,
          const void* g_masked, void* g_scores, void* g_values, int64_t rows, int64_t rpb, int k, int64_t m, int dv,
          unsigned int* status, cudaStream_t st) {
  using Acc = typename AccOf<TO>::type;
  sparse_attn_bwd_kernel<TS, TO><<<grid_for(rows), SW * kWarp, 0, st>>>(
      static_cast<const TS*>(sel), idx, static_cast<const TO*>(values), static_cast<const TO*>(g_out),
      static_cast<const TS*>(g_weights), static_cast<const TS*>(g_masked), static_cast<TS*>(g_scores),
      static_cast<Acc*>(g_values), rows, rpb, k, m, dv, status);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

// The (score, output) dtype pairs torch's type promotion produces between the
// four float types, with values already in the output dtype.
template <template <typename, typename> class F, typename... A>
int dispatch(int ts, int to, A... args) {
  using bf = __nv_bfloat16;
  if (ts == to) {
    switch (ts) {
      case SDK_DTYPE_F32: return F<float, float>::run(args...);
      case SDK_DTYPE_F64: return F<double, double>::run(args...);
      case SDK_DTYPE_F16: return F<__half, __half>::run(args...);
      case SDK_DTYPE_BF16: return F<bf, bf>::run(args...);
    }
  } else if (to == SDK_DTYPE_F32) {
    if (ts == SDK_DTYPE_F16) return F<__half, float>::run(args...);
    if (ts == SDK_DTYPE_BF16) return F<bf, float>::run(args...);
  } else if (to == SDK_DTYPE_F64) {
    if (ts == SDK_DTYPE_F32) return F<float, double>::run(args...);
    if (ts == SDK_DTYPE_F16) return F<__half, double>::run(args...);
    if (ts == SDK_DTYPE_BF16) return F<bf, double>::run(args...);
  }
  return SDK_ERR_INVALID_ARGUMENT;
}

template <typename TS, typename TO> struct FwdRun {
  static int run(const void* sel, const int64_t* idx, const void* values, void* out, void* weights, void* masked,
                 int64_t rows, int64_t rpb, int k, int64_t m, int dv, unsigned int* status, cudaStream_t st) {
    return fwd_t<TS, TO>(sel, idx, values, out, weights, masked, rows, rpb, k, m, dv, status, st);
  }
};

template <typename TS, typename TO> struct BwdRun {
  static int run(const void* sel, const int64_t* idx, const void* values, const void* g_out, const void* g_weights,
                 const void* g_masked, void* g_scores, void* g_values, int64_t rows, int64_t rpb, int k, int64_t m,
                 int dv, unsigned int* status, cudaStream_t st) {
    return bwd_t<TS, TO>(sel, idx, values, g_out, g_weights, g_masked, g_scores, g_values, rows, rpb, k, m, dv,
                         status, st);
  }
};

template <typename T>
int fill_t(const void* src, const int64_t* idx, void* dst, int64_t rows, int k, int64_t m, double fill,
           unsigned int* status, cudaStream_t st) {
  // the fill value converted on the host (from_acc is device code)
  T f;
  if constexpr (std::is_same<T, double>::value) f = fill;
  else if constexpr (std::is_same<T, float>::value) f = (float)fill;
  else if constexpr (std::is_same<T, __half>::value) f = __float2half_rn((float)fill);
  else f = __float2bfloat16_rn((float)fill);
  fill_scatter_kernel<T><<<grid_for(rows), SW * kWarp, 0, st>>>(static_cast<const T*>(src), idx, static_cast<T*>(dst),
                                                                 rows, k, m, f, status);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

}  // namespace

int sparse_attn_forward(const void* sel, const int64_t* idx, const void* values, void* out, void* weights,
                        void* masked, int64_t rows, int64_t rows_per_batch, int k, int64_t m, int dv, int score_dtype,
                        int out_dtype, unsigned int* status, cudaStream_t stream) {
  return dispatch<FwdRun>(score_dtype, out_dtype, sel, idx, values, out, weights, masked, rows, rows_per_batch, k, m,
                          dv, status, stream);
}

int sparse_attn_backward(const void* sel, const int64_t* idx, const void* values, const void* g_out,
                         const void* g_weights, const void* g_masked, void* g_scores, void* g_values, int64_t rows,
                         int64_t rows_per_batch, int k, int64_t m, int dv, int score_dtype, int out_dtype,
                         unsigned int* status, cudaStream_t stream) {
  return dispatch<BwdRun>(score_dtype, out_dtype, sel, idx, values, g_out, g_weights, g_masked, g_scores, g_values,
                          rows, rows_per_batch, k, m, dv, status, stream);
}

int fill_scatter(const void* src, const int64_t* idx, void* dst, int64_t rows, int k, int64_t m, double fill,
                 int dtype, unsigned int* status, cudaStream_t stream) {
  switch (dtype) {
    case SDK_DTYPE_F32: return fill_t<float>(src, idx, dst, rows, k, m, fill, status, stream);
    case SDK_DTYPE_F64: return fill_t<double>(src, idx, dst, rows, k, m, fill, status, stream);
    case SDK_DTYPE_F16: return fill_t<__half>(src, idx, dst, rows, k, m, fill, status, stream);
    case SDK_DTYPE_BF16: return fill_t<__nv_bfloat16>(src, idx, dst, rows, k, m, fill, status, stream);
    default: return SDK_ERR_INVALID_ARGUMENT;
  }
}

}  // namespace sdk
