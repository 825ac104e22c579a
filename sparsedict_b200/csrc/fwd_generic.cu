// Fused top-k attention forward, CUDA-core (FFMA/DFMA) path.
//
// One CTA owns BQ=32 query rows of one slice and streams that slice's keys
// in tiles of BK=64:
//   stage 1  affinity tile 32x64 from shared-memory Q/K chunks, 4x4 register
//            micro-tiles per thread, exact fp32 (fp64) accumulation;
//   stage 2  per-row threshold selection: warp w owns rows 8w..8w+7, keeps
//            every key scoring above the row's running k-th best score in a
//            shared-memory candidate list, and re-ranks the list with a warp
//            bitonic sort whenever it could overflow, which raises the
//            threshold; nothing of the score row reaches global memory;
//   stage 3  the final sort gives the top-k in reference order, then LSE,
//            softmax and the weighted sum of the gathered value rows.
//
// This kernel serves float32/float64 inputs (where the affinity must be exact
// fp32/fp64, kernels/fused_topk_attn.py:474-503 computes it with ieee dots)
// and any bf16/fp16 shape the tensor-core kernel does not take.
#include "common.cuh"
#include "kernels.h"

namespace sdk {
namespace {

constexpr int BQ = 32;
constexpr int BK = 64;
constexpr int FC = 32;
constexpr int NT = 128;
constexpr int KS = BK + 4;  // row stride of the key chunk (16-byte aligned rows)
constexpr int SS = BK + 1;  // row stride of the score tile

template <typename Acc> struct FwdArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int32_t* top_idx;
  Acc* lse;
  Acc* top_scores;
  SliceGeometry geo;
  const int32_t* row_index;
  int64_t m;
  int d, dv, topk, capp;
  Acc scale, root, grid;
  unsigned int* status;
  const Acc* seg_bias;  // nullable: score bias per (logical row, key segment)
  int64_t seg_len;
  int segs;
  const int32_t* row_k;  // nullable: per logical row, the number of keys to keep
};

template <typename Acc>
__device__ __forceinline__ void load4(const Acc* p, Acc (&r)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&r)[4]) {
  const float4 t = *reinterpret_cast<const float4*>(p);
  r[0] = t.x; r[1] = t.y; r[2] = t.z; r[3] = t.w;
}
template <>
__device__ __forceinline__ void load4<double>(const double* p, double (&r)[4]) {
  const double2 a = *reinterpret_cast<const double2*>(p);
  const double2 b = *reinterpret_cast<const double2*>(p + 2);
  r[0] = a.x; r[1] = a.y; r[2] = b.x; r[3] = b.y;
}

template <typename T>
__global__ void __launch_bounds__(NT) fused_fwd_generic(FwdArgs<typename AccOf<T>::type> a) {
  using Acc = typename AccOf<T>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];

  int64_t slice, row0;
  int rows;
  locate_tile(a.geo, blockIdx.x, BQ, &slice, &row0, &rows);
  if (rows <= 0) return;

  const T* __restrict__ q = static_cast<const T*>(a.q);
  const T* __restrict__ kmat = static_cast<const T*>(a.k) + slice * a.m * a.d;
  const T* __restrict__ vmat = static_cast<const T*>(a.v) + slice * a.m * a.dv;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ty = tid >> 4, tx = tid & 15;
  const int dpad = (a.d + FC - 1) / FC * FC;
  const int capp = a.capp;

  Acc* Qs = reinterpret_cast<Acc*>(smem_raw);  // [dpad][BQ]
  Acc* Ks = Qs + dpad * BQ;                     // [FC][KS]
  Acc* Ss = Ks + FC * KS;                       // [BQ][SS]
  Acc* cv = Ss + BQ * SS;                       // [BQ][capp]
  Acc* tau = cv + BQ * capp;                    // [BQ]
  int* ci = reinterpret_cast<int*>(tau + BQ);   // [BQ][capp]
  int* cnt = ci + BQ * capp;                    // [BQ]

  for (int e = tid; e < BQ * dpad; e += NT) {
    const int r = e / dpad, f = e - r * dpad;
    Acc val = 0;
    if (r < rows && f < a.d) {
      const int64_t lr = row0 + r;
      const int64_t pr = a.row_index ? (int64_t)a.row_index[lr] : lr;
      val = to_acc(q[pr * a.d + f]);
    }
    Qs[f * BQ + r] = val;
  }
  if (tid < BQ) {
    tau[tid] = quiet_nan<Acc>();  // "no threshold yet": !(s <= NaN) admits every key
    cnt[tid] = 0;
  }

  for (int64_t kt = 0; kt < a.m; kt += BK) {
    const int kvalid = (int)((a.m - kt) < BK ? (a.m - kt) : BK);
    Acc acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0;

    for (int fc = 0; fc < dpad; fc += FC) {
      __syncthreads();
      for (int e = tid; e < BK * FC; e += NT) {
        const int key = e / FC, f = e - key * FC;
        Acc val = 0;
        if (key < kvalid && fc + f < a.d) val = to_acc(kmat[(kt + key) * a.d + fc + f]);
        Ks[f * KS + key] = val;
      }
      __syncthreads();
#pragma unroll 4
      for (int f = 0; f < FC; ++f) {
        Acc qa[4], kb[4];
        load4(&Qs[(fc + f) * BQ + 4 * ty], qa);
        load4(&Ks[f * KS + 4 * tx], kb);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fma(qa[i], kb[j], acc[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Acc s = acc[i][j];
        s = (a.grid > 0) ? rint_acc((s * a.grid) / a.root) / a.grid : s * a.scale;
        if (a.seg_bias && 4 * ty + i < rows && 4 * tx + j < kvalid)
          s += a.seg_bias[(row0 + 4 * ty + i) * a.segs + (kt + 4 * tx + j) / a.seg_len];
        Ss[(4 * ty + i) * SS + 4 * tx + j] = s;
      }
    __syncthreads();

    for (int rr = 0; rr < BQ / 4; ++rr) {
      const int r = warp * (BQ / 4) + rr;
      if (r >= rows) break;
      const Acc t = tau[r];
      int c0 = cnt[r];
      Acc* rv = cv + r * capp;
      int* ri = ci + r * capp;
#pragma unroll
      for (int cb = 0; cb < BK; cb += kWarp) {
        const int c = cb + lane;
        const bool ok = c < kvalid;
        const Acc s = ok ? Ss[r * SS + c] : Acc(0);
        const bool pass = ok && !(s <= t);
        const unsigned b = __ballot_sync(0xffffffffu, pass);
        if (pass) {
          const int pos = c0 + __popc(b & ((1u << lane) - 1u));
          rv[pos] = s;
          ri[pos] = (int)(kt + c);
        }
        c0 += __popc(b);
      }
      __syncwarp();
      if (c0 > capp - BK) c0 = compact_row(rv, ri, c0, a.topk, &tau[r], lane);
      if (lane == 0) cnt[r] = c0;
      __syncwarp();
    }
  }

  // Final ranking, LSE, softmax and value aggregation (one warp per row).
  for (int rr = 0; rr < BQ / 4; ++rr) {
    const int r = warp * (BQ / 4) + rr;
    if (r >= rows) break;
    Acc* rv = cv + r * capp;
    int* ri = ci + r * capp;
    compact_row(rv, ri, cnt[r], a.topk, &tau[r], lane);
    const int64_t lr = row0 + r;
    // the row keeps its kr best (the list is in reference order); the other
    // index slots are -1 (adaptive k)
    const int kr = a.row_k ? min(max(a.row_k[lr], 1), a.topk) : a.topk;
    // softmax shift: the row maximum, or 0 when it is not finite (all
    // selected scores -inf gives LSE -inf)
    const Acc mx = isfinite(rv[0]) ? rv[0] : Acc(0);
    Acc part = 0;
    for (int j = lane; j < kr; j += kWarp) part += exp_acc(rv[j] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const Acc total = part;
    for (int j = lane; j < a.topk; j += kWarp) {
      a.top_idx[lr * a.topk + j] = j < kr ? ri[j] : -1;
      if (a.top_scores) a.top_scores[lr * a.topk + j] = j < kr ? rv[j] : neg_inf<Acc>();
    }
    if (lane == 0) a.lse[lr] = mx + log_acc(total);
    __syncwarp();
    for (int j = lane; j < kr; j += kWarp) rv[j] = exp_acc(rv[j] - mx) / total;
    __syncwarp();
    const int64_t pr = a.row_index ? (int64_t)a.row_index[lr] : lr;
    T* orow = static_cast<T*>(a.out) + pr * a.dv;
    for (int f = lane; f < a.dv; f += kWarp) {
      Acc o = 0;
      for (int j = 0; j < kr; ++j) o = fma(rv[j], to_acc(vmat[(int64_t)ri[j] * a.dv + f]), o);
      orow[f] = cvt_out<T>(o);
    }
  }
}

template <typename T>
size_t smem_bytes(int d, int capp) {
  using Acc = typename AccOf<T>::type;
  const int dpad = (d + FC - 1) / FC * FC;
  return sizeof(Acc) * ((size_t)dpad * BQ + FC * KS + BQ * SS + (size_t)BQ * capp + BQ) +
         sizeof(int) * ((size_t)BQ * capp + BQ);
}

template <typename T>
int launch(const FwdLaunch& L) {
  using Acc = typename AccOf<T>::type;
  const int capp = next_pow2_host(L.topk + BK);
  const size_t smem = smem_bytes<T>(L.d, capp);
  if (smem > kMaxDynamicSmem) return SDK_ERR_UNSUPPORTED;
  FwdArgs<Acc> a;
  a.q = L.q; a.k = L.k; a.v = L.v; a.out = L.out; a.top_idx = L.top_idx;
  a.lse = static_cast<Acc*>(L.lse);
  a.top_scores = static_cast<Acc*>(L.top_scores);
  a.geo = SliceGeometry{L.row_offsets, L.slices, L.n};
  a.row_index = L.row_index;
  a.m = L.m; a.d = L.d; a.dv = L.dv; a.topk = L.topk; a.capp = capp;
  a.scale = (Acc)L.scale;
  a.root = (Acc)(1.0 / L.scale);
  a.grid = (Acc)L.score_grid;
  a.status = L.status;
  a.seg_bias = static_cast<const Acc*>(L.seg_bias);
  a.seg_len = L.seg_len;
  a.segs = L.segs;
  a.row_k = L.row_k;
  const int64_t tiles = L.row_offsets ? (L.n + BQ - 1) / BQ + L.slices : L.slices * ((L.n + BQ - 1) / BQ);
  if (tiles <= 0) return SDK_OK;
  auto kern = fused_fwd_generic<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SDK_ERR_CUDA;
  kern<<<(unsigned)tiles, NT, smem, L.stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

}  // namespace

int max_topk_generic(int dtype, int d) {
  // The candidate list of a row holds capp = next_pow2(topk + BK) entries.
  int best = 0;
  for (int capp = 2 * BK; capp <= (1 << 16); capp <<= 1) {
    const size_t smem = dtype == SDK_DTYPE_F64 ? smem_bytes<double>(d, capp) : smem_bytes<float>(d, capp);
    if (smem > kMaxDynamicSmem) break;
    best = capp - BK;
  }
  return best;
}

int fwd_generic(const FwdLaunch& L) {
  switch (L.dtype) {
    case SDK_DTYPE_F32: return launch<float>(L);
    case SDK_DTYPE_F64: return launch<double>(L);
    case SDK_DTYPE_BF16: return launch<__nv_bfloat16>(L);
    case SDK_DTYPE_F16: return launch<__half>(L);
    default: return SDK_ERR_INVALID_ARGUMENT;
  }
}

}  // namespace sdk
