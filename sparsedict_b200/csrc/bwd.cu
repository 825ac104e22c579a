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
  const Acc* seg_bias;  // nullable: score bias per (logical row, key segment)
  Acc* dseg_bias;       // nullable: per (row, segment) sum of dS over the selected keys
  int64_t seg_len;
  int segs;
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
        if (a.seg_bias) s += a.seg_bias[r * a.segs + key / a.seg_len];
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
    if (a.dseg_bias && lane == 0) {
      // the warp owns row r: one lane adds its dS per segment in selection
      // order (deterministic, no atomics; the buffer starts at zero)
      for (int j = 0; j < a.topk; ++j)
        if (ij[j] >= 0) a.dseg_bias[r * a.segs + ij[j] / a.seg_len] += dsj[j];
    }

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

// ------------------------------------------------ d = dv = 64 fast path ---
// bf16/fp16 rows of 64 features (128 bytes), k <= 64.  A warp owns one query
// row; lane L owns slots L and L+32:
//   pass 1  each lane reads its slots' key and value rows with 16-byte loads
//           and forms s, P = exp(s - lse) and G = dout·v against q and dout
//           broadcast from shared memory;
//   dq      each lane keeps its key rows in registers and adds dS·k into a
//           64-wide partial; the 32 partials are summed through a padded
//           shared-memory transpose (lane L finishes features 2L, 2L+1);
//   scatter lanes span the 64 features of one key row (two per lane) so each
//           warp-wide vector reduction covers a whole 256-byte fp32 row.
constexpr int F64W = 4;  // warps per block

__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int h = 0; h < 8; ++h) f[h] = to_acc(e[h]);
}

template <typename T>
__global__ void __launch_bounds__(F64W * kWarp) sparse_bwd_d64(BwdArgs<float> a) {
  __shared__ __align__(16) float sq[F64W][64];
  __shared__ __align__(16) float sdo[F64W][64];
  __shared__ float part[F64W][kWarp][65];
  __shared__ float swk[F64W][64], swv[F64W][64];
  __shared__ int skey[F64W][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T* __restrict__ q = static_cast<const T*>(a.q);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);

  for (int64_t r = (int64_t)blockIdx.x * F64W + warp; r < a.rows; r += (int64_t)gridDim.x * F64W) {
    const int64_t slice = slice_of_row(a.geo, r);
    const int64_t pr = a.row_index ? (int64_t)a.row_index[r] : r;
    const T* __restrict__ kmat = static_cast<const T*>(a.k) + slice * a.m * 64;
    const T* __restrict__ vmat = static_cast<const T*>(a.v) + slice * a.m * 64;
    sq[warp][2 * lane] = to_acc(q[pr * 64 + 2 * lane]);
    sq[warp][2 * lane + 1] = to_acc(q[pr * 64 + 2 * lane + 1]);
    sdo[warp][2 * lane] = to_acc(dout[pr * 64 + 2 * lane]);
    sdo[warp][2 * lane + 1] = to_acc(dout[pr * 64 + 2 * lane + 1]);
    __syncwarp();
    const float l = a.lse[r];

    uint4 kr[2][8];
    float p[2], g[2];
    int key[2];
#pragma unroll
    for (int sj = 0; sj < 2; ++sj) {
      const int j = lane + 32 * sj;
      p[sj] = 0.f;
      g[sj] = 0.f;
      key[sj] = -1;
#pragma unroll
      for (int c = 0; c < 8; ++c) kr[sj][c] = make_uint4(0, 0, 0, 0);
      if (j < a.topk) {
        int kk = a.top_idx[r * a.topk + j];
        if (kk < 0 || kk >= a.m) {
          raise_device_status(a.status, kStatusIndexOutOfRange);
        } else {
          key[sj] = kk;
          const uint4* krow = reinterpret_cast<const uint4*>(kmat + (int64_t)kk * 64);
          const uint4* vrow = reinterpret_cast<const uint4*>(vmat + (int64_t)kk * 64);
          uint4 vr[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            kr[sj][c] = __ldg(krow + c);
            vr[c] = __ldg(vrow + c);
          }
          float s = 0.f, gg = 0.f;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float kf[8], vf[8];
            unpack8<T>(kr[sj][c], kf);
            unpack8<T>(vr[c], vf);
            const float4 q0 = *reinterpret_cast<const float4*>(&sq[warp][8 * c]);
            const float4 q1 = *reinterpret_cast<const float4*>(&sq[warp][8 * c + 4]);
            const float4 d0 = *reinterpret_cast<const float4*>(&sdo[warp][8 * c]);
            const float4 d1 = *reinterpret_cast<const float4*>(&sdo[warp][8 * c + 4]);
            s = fmaf(q0.x, kf[0], s); s = fmaf(q0.y, kf[1], s); s = fmaf(q0.z, kf[2], s); s = fmaf(q0.w, kf[3], s);
            s = fmaf(q1.x, kf[4], s); s = fmaf(q1.y, kf[5], s); s = fmaf(q1.z, kf[6], s); s = fmaf(q1.w, kf[7], s);
            gg = fmaf(d0.x, vf[0], gg); gg = fmaf(d0.y, vf[1], gg); gg = fmaf(d0.z, vf[2], gg); gg = fmaf(d0.w, vf[3], gg);
            gg = fmaf(d1.x, vf[4], gg); gg = fmaf(d1.y, vf[5], gg); gg = fmaf(d1.z, vf[6], gg); gg = fmaf(d1.w, vf[7], gg);
          }
          p[sj] = expf(s * a.scale - l);
          g[sj] = gg;
        }
      }
    }
    float part_sum = p[0] * g[0] + p[1] * g[1];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part_sum += __shfl_xor_sync(0xffffffffu, part_sum, o);
    const float delta = part_sum;
    const float ds0 = p[0] * (g[0] - delta), ds1 = p[1] * (g[1] - delta);

    float dqp[64];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float k0[8], k1[8];
      unpack8<T>(kr[0][c], k0);
      unpack8<T>(kr[1][c], k1);
#pragma unroll
      for (int h = 0; h < 8; ++h) dqp[8 * c + h] = fmaf(ds0, k0[h], ds1 * k1[h]);
    }
#pragma unroll
    for (int f = 0; f < 64; ++f) part[warp][lane][f] = dqp[f];
#pragma unroll
    for (int sj = 0; sj < 2; ++sj) {
      const int j = lane + 32 * sj;
      if (j < 64) {
        skey[warp][j] = key[sj];
        swk[warp][j] = (sj ? ds1 : ds0) * a.scale;
        swv[warp][j] = p[sj];
      }
    }
    __syncwarp();
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 8
    for (int i = 0; i < kWarp; ++i) {
      acc0 += part[warp][i][2 * lane];
      acc1 += part[warp][i][2 * lane + 1];
    }
    T* dqr = static_cast<T*>(a.dq) + pr * 64;
    dqr[2 * lane] = cvt_out<T>(acc0 * a.scale);
    dqr[2 * lane + 1] = cvt_out<T>(acc1 * a.scale);

    const float q0 = sq[warp][2 * lane], q1 = sq[warp][2 * lane + 1];
    const float o0 = sdo[warp][2 * lane], o1 = sdo[warp][2 * lane + 1];
    float* dkm = a.dk_acc + slice * a.m * 64;
    float* dvm = a.dv_acc + slice * a.m * 64;
    for (int j = 0; j < a.topk; ++j) {
      const int kk = skey[warp][j];
      if (kk < 0) continue;
      const float wk = swk[warp][j], wv = swv[warp][j];
      red_add2(dkm + (int64_t)kk * 64 + 2 * lane, wk * q0, wk * q1);
      red_add2(dvm + (int64_t)kk * 64 + 2 * lane, wv * o0, wv * o1);
    }
    __syncwarp();
  }
}

template <typename T>
int launch_d64(const BwdLaunch& L) {
  BwdArgs<float> a;
  a.q = L.q; a.k = L.k; a.v = L.v; a.dout = L.dout; a.top_idx = L.top_idx;
  a.lse = static_cast<const float*>(L.lse);
  a.dq = L.dq;
  a.dk_acc = static_cast<float*>(L.dk_acc);
  a.dv_acc = static_cast<float*>(L.dv_acc);
  a.geo = SliceGeometry{L.row_offsets, L.slices, L.n};
  a.row_index = L.row_index;
  a.rows = L.row_offsets ? L.n : L.slices * L.n;
  a.m = L.m; a.d = L.d; a.dv = L.dv; a.topk = L.topk;
  a.scale = (float)L.scale;
  a.root = (float)(1.0 / L.scale);
  a.grid = 0.f;
  a.status = L.status;
  a.seg_bias = nullptr;
  a.dseg_bias = nullptr;
  a.seg_len = 0;
  a.segs = 0;
  if (a.rows <= 0) return SDK_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (a.rows + F64W - 1) / F64W;
  const int64_t cap = (int64_t)sms * 8;
  sparse_bwd_d64<T><<<(unsigned)(want < cap ? want : cap), F64W * kWarp, 0, L.stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool d64_supported(const BwdLaunch& L) {
  return (L.dtype == SDK_DTYPE_BF16 || L.dtype == SDK_DTYPE_F16) && L.d == 64 && L.dv == 64 && L.topk <= 64 &&
         L.score_grid == 0 && !L.seg_bias && !L.dseg_bias && aligned16(L.k) && aligned16(L.v) &&
         aligned16(L.dk_acc) && aligned16(L.dv_acc);
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
  a.seg_bias = static_cast<const Acc*>(L.seg_bias);
  a.dseg_bias = static_cast<Acc*>(L.dseg_bias);
  a.seg_len = L.seg_len;
  a.segs = L.segs;
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
  if (d64_supported(L)) return L.dtype == SDK_DTYPE_BF16 ? launch_d64<__nv_bfloat16>(L) : launch_d64<__half>(L);
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
