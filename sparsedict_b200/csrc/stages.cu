// Stand-alone stage ops of the top-k attention path and the top-1 router.
//
//   affinity   dense scores = q·kᵀ (fp32), reference tiled_affinity
//              (kernels/fused_topk_attn.py:227-287); fp16 rows with d >= 64
//              go to the tensor-core kernel of affinity_tc.cu
//   select     per-row top-k of a score matrix, reference tiled_topk
//              (kernels/fused_topk_attn.py:290-336)
//   aggregate  softmax over selected scores and weighted gather of value
//              rows, reference tiled_topk_aggregate
//              (kernels/fused_topk_attn.py:339-408)
//   route      top-1 expert per token and a stable grouping of tokens by
//              expert (models/modules/router.py:139-145); per-block counts
//              in stream-ordered scratch from the library pool
#include "common.cuh"
#include "kernels.h"

namespace sdk {
namespace {

// ------------------------------------------------------------ affinity ---
constexpr int A_BM = 64, A_BN = 64, A_FC = 16, A_NT = 256;

template <typename T>
__global__ void __launch_bounds__(A_NT) affinity_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                        float* __restrict__ s, int64_t n, int64_t m, int d,
                                                        int64_t qs, int64_t ks) {
  __shared__ __align__(16) float Qs[A_FC][A_BM];
  __shared__ __align__(16) float Ks[A_FC][A_BN];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t r0 = (int64_t)blockIdx.y * A_BM, c0 = (int64_t)blockIdx.x * A_BN;
  float acc[4][4] = {};
  for (int fc = 0; fc < d; fc += A_FC) {
    for (int e = tid; e < A_BM * A_FC; e += A_NT) {
      const int r = e / A_FC, f = e % A_FC;
      Qs[f][r] = (r0 + r < n && fc + f < d) ? to_acc(q[(r0 + r) * qs + fc + f]) : 0.f;
      Ks[f][r] = (c0 + r < m && fc + f < d) ? to_acc(k[(c0 + r) * ks + fc + f]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int f = 0; f < A_FC; ++f) {
      const float4 a = *reinterpret_cast<const float4*>(&Qs[f][4 * ty]);
      const float4 b = *reinterpret_cast<const float4*>(&Ks[f][4 * tx]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t r = r0 + 4 * ty + i, c = c0 + 4 * tx + j;
      if (r < n && c < m) s[r * m + c] = acc[i][j];
    }
}

// -------------------------------------------------------------- select ---
// One warp per row streams the row 32 keys at a time, keeps keys that beat
// the running k-th best in a shared-memory list and re-ranks the list with a
// warp bitonic sort when it could overflow.
// Comparisons run in the accumulator type (double for fp64 scores, float
// otherwise), which holds every input value exactly.
template <typename T>
__global__ void select_kernel(const T* __restrict__ s, T* __restrict__ vals_out, int64_t* __restrict__ idx_out,
                              int64_t rows, int64_t m, int64_t stride, int topk, int capp) {
  using Acc = typename AccOf<T>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  Acc* cv = reinterpret_cast<Acc*>(smem_raw) + warp * capp;
  int* ci = reinterpret_cast<int*>(reinterpret_cast<Acc*>(smem_raw) + warps * capp) + warp * capp;
  for (int64_t r = (int64_t)blockIdx.x * warps + warp; r < rows; r += (int64_t)gridDim.x * warps) {
    const T* row = s + r * stride;
    Acc tau = quiet_nan<Acc>();
    int cnt = 0;
    for (int64_t c0 = 0; c0 < m; c0 += kWarp) {
      const int64_t c = c0 + lane;
      const bool ok = c < m;
      const Acc x = ok ? to_acc(row[c]) : Acc(0);
      const bool pass = ok && !(x <= tau);
      const unsigned b = __ballot_sync(0xffffffffu, pass);
      if (pass) {
        const int pos = cnt + __popc(b & ((1u << lane) - 1u));
        cv[pos] = x;
        ci[pos] = (int)c;
      }
      cnt += __popc(b);
      __syncwarp();
      if (cnt > capp - kWarp) {
        const int P = next_pow2_dev(cnt);
        for (int i = cnt + lane; i < P; i += kWarp) { cv[i] = neg_inf<Acc>(); ci[i] = kPadIndex; }
        __syncwarp();
        warp_bitonic_sort(cv, ci, P, lane);
        cnt = topk;
        tau = cv[topk - 1];
      }
    }
    const int P = next_pow2_dev(cnt);
    for (int i = cnt + lane; i < P; i += kWarp) { cv[i] = neg_inf<Acc>(); ci[i] = kPadIndex; }
    __syncwarp();
    warp_bitonic_sort(cv, ci, P, lane);
    for (int j = lane; j < topk; j += kWarp) {
      vals_out[r * topk + j] = cvt_out<T>(cv[j]);
      idx_out[r * topk + j] = ci[j];
    }
    __syncwarp();
  }
}

// ----------------------------------------------------------- aggregate ---
template <typename TS, typename TI, typename TV>
__global__ void aggregate_kernel(const TS* __restrict__ ts, const TI* __restrict__ ti, const TV* __restrict__ vals,
                                 float* __restrict__ out, int64_t rows, int topk, int64_t m, int dv,
                                 int64_t ss, int64_t is, int64_t vs, unsigned int* status) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int64_t r = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * warps) {
    const TS* srow = ts + r * ss;
    const TI* irow = ti + r * is;
    float mx = neg_inf<float>();
    for (int j = lane; j < topk; j += kWarp) mx = fmaxf(mx, to_acc(srow[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.f;
    for (int j = lane; j < topk; j += kWarp) total += expf(to_acc(srow[j]) - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    for (int f0 = 0; f0 < dv; f0 += kWarp) {
      const int f = f0 + lane;
      float acc = 0.f;
      for (int j = 0; j < topk; ++j) {
        const int64_t key = (int64_t)irow[j];
        if (key < 0 || key >= m) {
          if (lane == 0 && f0 == 0) raise_device_status(status, kStatusIndexOutOfRange);
          continue;
        }
        const float w = expf(to_acc(srow[j]) - mx) / total;
        if (f < dv) acc = fmaf(w, to_acc(vals[key * vs + f]), acc);
      }
      if (f < dv) out[r * dv + f] = acc;
    }
  }
}

// --------------------------------------------------------------- route ---
// Three launches over blocks of RB tokens (one per thread):
//   count  each token's expert (the first maximum, NaN ranking highest, as
//          torch.argmax) and the block's per-expert counts;
//   scan   one block: for each expert, the exclusive sum of the counts over
//          the blocks before each block, plus the expert offsets;
//   place  each token's position: its expert's offset + the block's prefix
//          + its rank among the block's tokens of that expert (warp
//          match/popc, then a prefix over the block's warps), so the order
//          within an expert is ascending token index (a stable sort).
constexpr int R_NT = 256, R_MAXE = 16, R_WARPS = R_NT / kWarp;

__global__ void __launch_bounds__(R_NT) route_count(const float* __restrict__ logits, int64_t n, int experts,
                                                    int32_t* __restrict__ expert, int32_t* __restrict__ counts) {
  __shared__ int wc[R_WARPS][R_MAXE];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t i = (int64_t)blockIdx.x * R_NT + t;
  int best = -1;
  if (i < n) {
    const float* row = logits + i * experts;
    float v[R_MAXE];
#pragma unroll
    for (int x = 0; x < R_MAXE; ++x) v[x] = x < experts ? __ldg(row + x) : 0.f;
    best = 0;
    float bv = v[0];
#pragma unroll
    for (int x = 1; x < R_MAXE; ++x)
      if (x < experts && ranks_above(v[x], x, bv, best)) { bv = v[x]; best = x; }
    expert[i] = best;
  }
  for (int x = 0; x < experts; ++x) {
    const unsigned b = __ballot_sync(0xffffffffu, best == x);
    if (lane == 0) wc[warp][x] = __popc(b);
  }
  __syncthreads();
  if (t < experts) {
    int c = 0;
#pragma unroll
    for (int w = 0; w < R_WARPS; ++w) c += wc[w][t];
    counts[(int64_t)blockIdx.x * experts + t] = c;
  }
}

// One block of R_NT threads: thread x < experts scans expert x's column of
// the block counts (in place, exclusive); then the expert offsets.
__global__ void __launch_bounds__(R_NT) route_scan(int32_t* __restrict__ counts, int64_t blocks, int experts,
                                                   int32_t* __restrict__ offsets) {
  __shared__ int tot[R_MAXE];
  const int t = threadIdx.x;
  if (t < experts) {
    int run = 0;
    for (int64_t b = 0; b < blocks; ++b) {
      const int c = counts[b * experts + t];
      counts[b * experts + t] = run;
      run += c;
    }
    tot[t] = run;
  }
  __syncthreads();
  if (t == 0) {
    int run = 0;
    for (int x = 0; x < experts; ++x) {
      offsets[x] = run;
      run += tot[x];
    }
    offsets[experts] = run;
  }
}

__global__ void __launch_bounds__(R_NT) route_place(const int32_t* __restrict__ expert, int64_t n, int experts,
                                                    const int32_t* __restrict__ counts,
                                                    const int32_t* __restrict__ offsets, int32_t* __restrict__ order) {
  __shared__ int wc[R_WARPS][R_MAXE];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t i = (int64_t)blockIdx.x * R_NT + t;
  const int x = i < n ? expert[i] : -1;
  const unsigned same = __match_any_sync(0xffffffffu, x);
  const int rank = __popc(same & ((1u << lane) - 1u));
  for (int y = 0; y < experts; ++y)
    if (lane == 0) wc[warp][y] = 0;
  __syncwarp();
  if (x >= 0 && rank == 0) wc[warp][x] = __popc(same);
  __syncthreads();
  if (x >= 0) {
    int pos = offsets[x] + counts[(int64_t)blockIdx.x * experts + x] + rank;
    for (int w = 0; w < warp; ++w) pos += wc[w][x];
    order[pos] = (int32_t)i;
  }
}

template <typename TS, typename TI>
int aggregate_v(const void* ts, const void* ti, const void* v, float* out, int64_t rows, int topk, int64_t m,
                int dv, int64_t ss, int64_t is, int64_t vs, int vdt, unsigned int* status, cudaStream_t st,
                unsigned grid) {
  if (vdt == SDK_DTYPE_F32)
    aggregate_kernel<TS, TI, float><<<grid, 128, 0, st>>>(static_cast<const TS*>(ts), static_cast<const TI*>(ti),
                                                         static_cast<const float*>(v), out, rows, topk, m, dv,
                                                         ss, is, vs, status);
  else if (vdt == SDK_DTYPE_F16)
    aggregate_kernel<TS, TI, __half><<<grid, 128, 0, st>>>(static_cast<const TS*>(ts), static_cast<const TI*>(ti),
                                                          static_cast<const __half*>(v), out, rows, topk, m, dv,
                                                          ss, is, vs, status);
  else
    return SDK_ERR_INVALID_ARGUMENT;
  return SDK_OK;
}

}  // namespace

int affinity(const void* q, const void* k, float* scores, int64_t n, int64_t m, int d, int64_t qs, int64_t ks,
             int dtype, cudaStream_t stream) {
  if (affinity_tensorcore_supports(q, k, n, m, d, qs, ks, dtype))
    return affinity_tensorcore(q, k, scores, n, m, d, qs, ks, stream);
  const dim3 grid((unsigned)((m + A_BN - 1) / A_BN), (unsigned)((n + A_BM - 1) / A_BM));
  if (grid.y > 65535u) return SDK_ERR_UNSUPPORTED;
  if (dtype == SDK_DTYPE_F32)
    affinity_kernel<float><<<grid, A_NT, 0, stream>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                                       scores, n, m, d, qs, ks);
  else if (dtype == SDK_DTYPE_F16)
    affinity_kernel<__half><<<grid, A_NT, 0, stream>>>(static_cast<const __half*>(q), static_cast<const __half*>(k),
                                                        scores, n, m, d, qs, ks);
  else
    return SDK_ERR_INVALID_ARGUMENT;
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

template <typename T>
int launch_select(const void* scores, void* top_values, int64_t* top_idx, int64_t rows, int64_t m, int64_t stride,
                  int topk, cudaStream_t stream) {
  using Acc = typename AccOf<T>::type;
  const int capp = next_pow2_host(topk + kWarp);
  const size_t per_warp = (size_t)capp * (sizeof(Acc) + sizeof(int));
  int warps = 4;
  while (warps > 1 && warps * per_warp > kMaxDynamicSmem) warps >>= 1;
  const size_t smem = warps * per_warp;
  if (smem > kMaxDynamicSmem) return SDK_ERR_UNSUPPORTED;
  const int64_t want = (rows + warps - 1) / warps;
  const unsigned grid = (unsigned)(want < 148 * 64 ? want : 148 * 64);
  auto kern = select_kernel<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SDK_ERR_CUDA;
  kern<<<grid, warps * kWarp, smem, stream>>>(static_cast<const T*>(scores), static_cast<T*>(top_values), top_idx,
                                              rows, m, stride, topk, capp);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

int topk_select(const void* scores, void* top_values, int64_t* top_idx, int64_t rows, int64_t m, int64_t stride,
                int topk, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case SDK_DTYPE_F32: return launch_select<float>(scores, top_values, top_idx, rows, m, stride, topk, stream);
    case SDK_DTYPE_F16: return launch_select<__half>(scores, top_values, top_idx, rows, m, stride, topk, stream);
    case SDK_DTYPE_BF16:
      return launch_select<__nv_bfloat16>(scores, top_values, top_idx, rows, m, stride, topk, stream);
    case SDK_DTYPE_F64: return launch_select<double>(scores, top_values, top_idx, rows, m, stride, topk, stream);
    default: return SDK_ERR_INVALID_ARGUMENT;
  }
}

int topk_aggregate(const void* ts, const void* ti, const void* v, float* out, int64_t rows, int topk, int64_t m,
                   int dv, int64_t ss, int64_t is, int64_t vs, int sdt, int idx_bits, int vdt, unsigned int* status,
                   cudaStream_t stream) {
  const int64_t want = (rows + 3) / 4;
  const unsigned grid = (unsigned)(want < 148 * 64 ? want : 148 * 64);
  int rc;
  if (sdt == SDK_DTYPE_F32 && idx_bits == 32)
    rc = aggregate_v<float, int32_t>(ts, ti, v, out, rows, topk, m, dv, ss, is, vs, vdt, status, stream, grid);
  else if (sdt == SDK_DTYPE_F32 && idx_bits == 64)
    rc = aggregate_v<float, int64_t>(ts, ti, v, out, rows, topk, m, dv, ss, is, vs, vdt, status, stream, grid);
  else if (sdt == SDK_DTYPE_F16 && idx_bits == 32)
    rc = aggregate_v<__half, int32_t>(ts, ti, v, out, rows, topk, m, dv, ss, is, vs, vdt, status, stream, grid);
  else if (sdt == SDK_DTYPE_F16 && idx_bits == 64)
    rc = aggregate_v<__half, int64_t>(ts, ti, v, out, rows, topk, m, dv, ss, is, vs, vdt, status, stream, grid);
  else
    return SDK_ERR_INVALID_ARGUMENT;
  if (rc != SDK_OK) return rc;
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

int route_top1(const float* logits, int64_t n, int experts, int32_t* expert, int32_t* order, int32_t* offsets,
               cudaStream_t stream) {
  if (experts < 1 || experts > R_MAXE) return SDK_ERR_UNSUPPORTED;
  const int64_t blocks = (n + R_NT - 1) / R_NT;
  if (blocks > 0x7fffffff) return SDK_ERR_UNSUPPORTED;
  // per-block counts: stream-ordered scratch from the library pool
  cudaMemPool_t pool = scratch_pool();
  if (!pool) return SDK_ERR_CUDA;
  void* scratch = nullptr;
  if (cudaMallocFromPoolAsync(&scratch, (size_t)blocks * experts * sizeof(int32_t), pool, stream) != cudaSuccess)
    return SDK_ERR_CUDA;
  int32_t* counts = static_cast<int32_t*>(scratch);
  route_count<<<(unsigned)blocks, R_NT, 0, stream>>>(logits, n, experts, expert, counts);
  route_scan<<<1, R_NT, 0, stream>>>(counts, blocks, experts, offsets);
  route_place<<<(unsigned)blocks, R_NT, 0, stream>>>(expert, n, experts, counts, offsets, order);
  int rc = cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
  if (cudaFreeAsync(scratch, stream) != cudaSuccess) rc = SDK_ERR_CUDA;
  return rc;
}

}  // namespace sdk
