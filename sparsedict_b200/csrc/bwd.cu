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
// The generic kernel below serves every dtype and width; bf16/fp16 rows of
// 64 features take the grouped fast path further down.
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
        // -1 marks an empty slot (a row that keeps fewer keys, or one the
        // forward gave up on); anything else out of range is flagged
        if (key != -1) raise_device_status(a.status, kStatusIndexOutOfRange);
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
// row.  Its lanes form four groups of eight: group g takes slots g, g+4, g+8,
// ... and lane l of a group features 8l..8l+7, so each key or value row is one
// coalesced 128-byte access by eight lanes (four rows per load instruction).
//   pass 1  per slot: q·k and dout·v as 8-feature partials, summed over the
//           group by three butterfly steps (every lane of the group holds the
//           same sums); P = exp(s·scale - lse); P, G and the key go to shared
//           memory; delta = sum of P·G over the row;
//   pass 2  per slot: dS = P (G - delta); the key row is read again (an L1/L2
//           hit) for dq += dS·k; dK[key] += scale·dS·q and dV[key] += P·dout
//           are two 16-byte vector reductions per lane each, lane l taking
//           features 4l..4l+3 and 32+4l..32+4l+3 so that each reduction
//           instruction covers four rows' 128-byte halves.  (Whole-warp
//           8-byte reductions of one 256-byte row per instruction touch half
//           the L2 sectors but measured 7 % slower: twice the instructions.)
//   dq      the four groups' partials are summed by two butterfly steps and
//           group 0 writes the row once (no atomics).
constexpr int G8W = 8;  // warps per block

__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int h = 0; h < 8; ++h) f[h] = to_acc(e[h]);
}

template <typename T>
__device__ __forceinline__ void unpack4(const uint2& u, float* f) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int h = 0; h < 4; ++h) f[h] = to_acc(e[h]);
}

template <typename T>
__global__ void __launch_bounds__(G8W * kWarp, 4) sparse_bwd_d64(BwdArgs<float> a) {
  __shared__ float sp[G8W][64], sg[G8W][64];
  __shared__ int skey[G8W][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 3, l8 = lane & 7;
  const T* __restrict__ q = static_cast<const T*>(a.q);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);

  for (int64_t r = (int64_t)blockIdx.x * G8W + warp; r < a.rows; r += (int64_t)gridDim.x * G8W) {
    const int64_t slice = slice_of_row(a.geo, r);
    const int64_t pr = a.row_index ? (int64_t)a.row_index[r] : r;
    const uint4* __restrict__ kmat =
        reinterpret_cast<const uint4*>(static_cast<const T*>(a.k) + slice * a.m * 64) + l8;
    const uint4* __restrict__ vmat =
        reinterpret_cast<const uint4*>(static_cast<const T*>(a.v) + slice * a.m * 64) + l8;
    float qf[8], df[8];
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(q + pr * 64) + l8), qf);
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(dout + pr * 64) + l8), df);
    const float l = a.lse[r];
    int i0 = -1, i1 = -1;  // slots lane and lane + 32
    if (lane < a.topk) i0 = a.top_idx[r * a.topk + lane];
    if (lane + 32 < a.topk) i1 = a.top_idx[r * a.topk + lane + 32];
    // -1 marks an empty slot (a row that keeps fewer keys, or one the forward
    // gave up on); anything else out of range is flagged
    if ((lane < a.topk && (i0 < -1 || i0 >= a.m)) || (lane + 32 < a.topk && (i1 < -1 || i1 >= a.m)))
      raise_device_status(a.status, kStatusIndexOutOfRange);
    if (i0 < 0 || i0 >= a.m) i0 = -1;
    if (i1 < 0 || i1 >= a.m) i1 = -1;

    float part = 0.f;
#pragma unroll 4
    for (int it = 0; it < 16; ++it) {
      const int j = 4 * it + grp;
      const int key = __shfl_sync(0xffffffffu, it < 8 ? i0 : i1, j & 31);
      float s = 0.f, g = 0.f;
      if (key >= 0) {
        float kf[8], vf[8];
        unpack8<T>(__ldg(kmat + (int64_t)key * 8), kf);
        unpack8<T>(__ldg(vmat + (int64_t)key * 8), vf);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          s = fmaf(qf[h], kf[h], s);
          g = fmaf(df[h], vf[h], g);
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        g += __shfl_xor_sync(0xffffffffu, g, o);
      }
      const float p = key >= 0 ? expf(s * a.scale - l) : 0.f;
      if (l8 == 0) {
        sp[warp][j] = p;
        sg[warp][j] = g;
        skey[warp][j] = key;
      }
      part = fmaf(p, g, part);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 8);
    part += __shfl_xor_sync(0xffffffffu, part, 16);
    const float delta = part;
    __syncwarp();

    // q and dout again, features 4·l8..4·l8+3 and 32+4·l8..32+4·l8+3 (the
    // reduction layout)
    float qb[8], db[8];
    {
      const uint2* q2 = reinterpret_cast<const uint2*>(q + pr * 64);
      const uint2* d2 = reinterpret_cast<const uint2*>(dout + pr * 64);
      unpack4<T>(__ldg(q2 + l8), qb);
      unpack4<T>(__ldg(q2 + 8 + l8), qb + 4);
      unpack4<T>(__ldg(d2 + l8), db);
      unpack4<T>(__ldg(d2 + 8 + l8), db + 4);
    }
    float dq[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) dq[h] = 0.f;
    float* dkm = a.dk_acc + slice * a.m * 64 + 4 * l8;
    float* dvm = a.dv_acc + slice * a.m * 64 + 4 * l8;
#pragma unroll 4
    for (int it = 0; it < 16; ++it) {
      const int j = 4 * it + grp;
      const int key = skey[warp][j];
      if (key < 0) continue;
      const float p = sp[warp][j];
      const float ds = p * (sg[warp][j] - delta);
      float kf[8];
      unpack8<T>(__ldg(kmat + (int64_t)key * 8), kf);
#pragma unroll
      for (int h = 0; h < 8; ++h) dq[h] = fmaf(ds, kf[h], dq[h]);
      const float wk = ds * a.scale;
      float* dk = dkm + (int64_t)key * 64;
      float* dv = dvm + (int64_t)key * 64;
      red_add4(dk, wk * qb[0], wk * qb[1], wk * qb[2], wk * qb[3]);
      red_add4(dk + 32, wk * qb[4], wk * qb[5], wk * qb[6], wk * qb[7]);
      red_add4(dv, p * db[0], p * db[1], p * db[2], p * db[3]);
      red_add4(dv + 32, p * db[4], p * db[5], p * db[6], p * db[7]);
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      dq[h] += __shfl_xor_sync(0xffffffffu, dq[h], 8);
      dq[h] += __shfl_xor_sync(0xffffffffu, dq[h], 16);
    }
    if (grp == 0) {
      uint4 o;
      T* e = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int h = 0; h < 8; ++h) e[h] = cvt_out<T>(dq[h] * a.scale);
      reinterpret_cast<uint4*>(static_cast<T*>(a.dq) + pr * 64)[l8] = o;
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
  // One block per eight rows (not a resident grid-stride wave): blocks retire
  // as they go, so kernels on other streams (the gradient exchange of an
  // earlier bucket) get SMs while this one runs; measured no slower alone.
  // (the kernel walks its rows grid-stride, so a clamped grid stays correct)
  const int64_t want = (a.rows + G8W - 1) / G8W;
  const unsigned grid = (unsigned)(want < 0x7fffffff ? want : 0x7fffffff);
  sparse_bwd_d64<T><<<grid, G8W * kWarp, 0, L.stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool d64_supported(const BwdLaunch& L) {
  const int64_t rows = L.row_offsets ? L.n : L.slices * L.n;
  if (rows > 0x7fffff00) return false;  // row indices and row * topk stay in range
  return (L.dtype == SDK_DTYPE_BF16 || L.dtype == SDK_DTYPE_F16) && L.d == 64 && L.dv == 64 && L.topk <= 64 &&
         L.score_grid == 0 && !L.seg_bias && !L.dseg_bias && aligned16(L.q) && aligned16(L.k) &&
         aligned16(L.v) && aligned16(L.dout) && aligned16(L.dq) && aligned16(L.dk_acc) && aligned16(L.dv_acc);
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
