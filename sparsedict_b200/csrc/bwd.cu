// Sparse backward of top-k attention on the saved support.
//
// Restates the reference's B1 (_backward_dq, kernels/fused_topk_attn.py:609-846)
// and B2 (_backward_dkv, :848-977) as one kernel.  A warp owns one query
// row i and its k selected keys:
//   S_ij  = scale * q_i·k_j   (recomputed; the tie-stress grid re-quantises)
//   P_ij  = exp(S_ij - lse_i)
//   G_ij  = dout_i·v_j
//   delta = sum_j P_ij G_ij,  dS_ij = P_ij (G_ij - delta)
//   dq_i  = scale * sum_j dS_ij k_j                    (gathered contraction,
//                                                       written once, no atomics)
//   dk_j += scale * dS_ij q_i,  dv_j += P_ij dout_i    (scatter into the
//                                                       accumulators with
//                                                       vector reductions)
// The per-row recomputation reads the k selected key/value rows once each
// (lane j holds slot j), the dq contraction re-reads the key rows coalesced
// across features.
#include "common.cuh"
#include "kernels.h"

namespace sdk {
namespace {

constexpr int WARPS = 4;
constexpr int NT = WARPS * kWarp;

template <typename Acc> struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* dout;
  const int32_t* top_idx;
  const Acc* lse;
  void* dq;
  Acc* dk_acc;
  Acc* dv_acc;
  SliceGeometry geo;
  const int32_t* row_index;
  int64_t rows, m;
  int d, dv, topk;
  Acc scale, root, grid;
  unsigned int* status;
};

__device__ __forceinline__ int64_t slice_of_row(const SliceGeometry& g, int64_t r) {
  if (!g.row_offsets) return r / g.n;
  int64_t lo = 0, hi = g.slices - 1;
  while (lo < hi) {  // last slice whose first row is <= r
    const int64_t mid = (lo + hi + 1) >> 1;
    if ((int64_t)g.row_offsets[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void red_add(float* p, float x) { atomicAdd(p, x); }
__device__ __forceinline__ void red_add(double* p, double x) { atomicAdd(p, x); }

template <typename T>
__global__ void __launch_bounds__(NT) sparse_bwd(BwdArgs<typename AccOf<T>::type> a) {
  using Acc = typename AccOf<T>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // per warp: qv[d] dov[dv] pj[k] dsj[k] idx[k]
  const int per_warp = a.d + a.dv + 2 * a.topk;
  Acc* base = reinterpret_cast<Acc*>(smem_raw) + warp * per_warp;
  Acc* qv = base;
  Acc* dov = qv + a.d;
  Acc* pj = dov + a.dv;
  Acc* dsj = pj + a.topk;
  int* ij = reinterpret_cast<int*>(reinterpret_cast<Acc*>(smem_raw) + WARPS * per_warp) + warp * a.topk;

  const T* __restrict__ q = static_cast<const T*>(a.q);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);

  for (int64_t r = (int64_t)blockIdx.x * WARPS + warp; r < a.rows; r += (int64_t)gridDim.x * WARPS) {
    const int64_t slice = slice_of_row(a.geo, r);
    const int64_t pr = a.row_index ? (int64_t)a.row_index[r] : r;
    const T* __restrict__ kmat = static_cast<const T*>(a.k) + slice * a.m * a.d;
    const T* __restrict__ vmat = static_cast<const T*>(a.v) + slice * a.m * a.dv;
    Acc* dkm = a.dk_acc + slice * a.m * a.d;
    Acc* dvm = a.dv_acc + slice * a.m * a.dv;

    for (int f = lane; f < a.d; f += kWarp) qv[f] = to_acc(q[pr * a.d + f]);
    for (int f = lane; f < a.dv; f += kWarp) dov[f] = to_acc(dout[pr * a.dv + f]);
    __syncwarp();
    const Acc l = a.lse[r];

    Acc part = 0;
    for (int j = lane; j < a.topk; j += kWarp) {
      int key = a.top_idx[r * a.topk + j];
      Acc p = 0, g = 0;
      if (key < 0 || key >= a.m) {
        raise_device_status(a.status, kStatusIndexOutOfRange);
        key = -1;
      } else {
        const T* kr = kmat + (int64_t)key * a.d;
        const T* vr = vmat + (int64_t)key * a.dv;
        Acc s = 0;
        for (int f = 0; f < a.d; ++f) s = fma(qv[f], to_acc(kr[f]), s);
        s = (a.grid > 0) ? rint_acc((s * a.grid) / a.root) / a.grid : s * a.scale;
        p = exp_acc(s - l);
        for (int f = 0; f < a.dv; ++f) g = fma(dov[f], to_acc(vr[f]), g);
      }
      ij[j] = key;
      pj[j] = p;
      dsj[j] = g;
      part = fma(p, g, part);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const Acc delta = part;
    __syncwarp();
    for (int j = lane; j < a.topk; j += kWarp) dsj[j] = pj[j] * (dsj[j] - delta);
    __syncwarp();

    T* dqr = static_cast<T*>(a.dq) + pr * a.d;
    for (int f = lane; f < a.d; f += kWarp) {
      Acc acc = 0;
      for (int j = 0; j < a.topk; ++j) {
        const int key = ij[j];
        if (key >= 0) acc = fma(dsj[j], to_acc(kmat[(int64_t)key * a.d + f]), acc);
      }
      dqr[f] = cvt_out<T>(acc * a.scale);
    }
    for (int j = 0; j < a.topk; ++j) {
      const int key = ij[j];
      if (key < 0) continue;
      const Acc wk = dsj[j] * a.scale, wv = pj[j];
      for (int f = lane; f < a.d; f += kWarp) red_add(&dkm[(int64_t)key * a.d + f], wk * qv[f]);
      for (int f = lane; f < a.dv; f += kWarp) red_add(&dvm[(int64_t)key * a.dv + f], wv * dov[f]);
    }
    __syncwarp();
  }
}

template <typename T>
int launch(const BwdLaunch& L) {
  using Acc = typename AccOf<T>::type;
  BwdArgs<Acc> a;
  a.q = L.q; a.k = L.k; a.v = L.v; a.dout = L.dout; a.top_idx = L.top_idx;
  a.lse = static_cast<const Acc*>(L.lse);
  a.dq = L.dq;
  a.dk_acc = static_cast<Acc*>(L.dk_acc);
  a.dv_acc = static_cast<Acc*>(L.dv_acc);
  a.geo = SliceGeometry{L.row_offsets, L.slices, L.n};
  a.row_index = L.row_index;
  a.rows = L.row_offsets ? L.n : L.slices * L.n;
  a.m = L.m; a.d = L.d; a.dv = L.dv; a.topk = L.topk;
  a.scale = (Acc)L.scale;
  a.root = (Acc)(1.0 / L.scale);
  a.grid = (Acc)L.score_grid;
  a.status = L.status;
  const size_t smem = (size_t)WARPS * ((L.d + L.dv + 2 * L.topk) * sizeof(Acc) + L.topk * sizeof(int));
  if (smem > kMaxDynamicSmem) return SDK_ERR_UNSUPPORTED;
  if (a.rows <= 0) return SDK_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (a.rows + WARPS - 1) / WARPS;
  const int64_t cap = (int64_t)sms * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  auto kern = sparse_bwd<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SDK_ERR_CUDA;
  kern<<<grid, NT, smem, L.stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

template <typename T, typename Acc>
__global__ void finalize_kernel(const Acc* acc, T* out, int64_t count, Acc mult) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = cvt_out<T>(acc[i] * mult);
}

template <typename T>
int launch_finalize(const void* acc, void* out, int64_t count, double mult, cudaStream_t stream) {
  using Acc = typename AccOf<T>::type;
  if (count <= 0) return SDK_OK;
  const int64_t blocks = (count + 255) / 256;
  const unsigned grid = (unsigned)(blocks < 148 * 32 ? blocks : 148 * 32);
  finalize_kernel<T, Acc><<<grid, 256, 0, stream>>>(static_cast<const Acc*>(acc), static_cast<T*>(out),
                                                    count, (Acc)mult);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

}  // namespace

int bwd_sparse(const BwdLaunch& L) {
  switch (L.dtype) {
    case SDK_DTYPE_F32: return launch<float>(L);
    case SDK_DTYPE_F64: return launch<double>(L);
    case SDK_DTYPE_BF16: return launch<__nv_bfloat16>(L);
    case SDK_DTYPE_F16: return launch<__half>(L);
    default: return SDK_ERR_INVALID_ARGUMENT;
  }
}

int finalize_grad(const void* acc, void* out, int64_t count, double multiplier, int dtype,
                  cudaStream_t stream) {
  switch (dtype) {
    case SDK_DTYPE_F32: return launch_finalize<float>(acc, out, count, multiplier, stream);
    case SDK_DTYPE_F64: return launch_finalize<double>(acc, out, count, multiplier, stream);
    case SDK_DTYPE_BF16: return launch_finalize<__nv_bfloat16>(acc, out, count, multiplier, stream);
    case SDK_DTYPE_F16: return launch_finalize<__half>(acc, out, count, multiplier, stream);
    default: return SDK_ERR_INVALID_ARGUMENT;
  }
}

}  // namespace sdk
