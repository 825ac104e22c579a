// Shared device helpers for the top-k sparse attention kernels.
//
// The selection order everywhere is the reference comparator of
// kernels/fused_topk_attn.py:67-89 (SparseDict): NaN ranks above every
// number (two NaNs: lower key index first), otherwise larger score first and,
// on equal scores, lower key index first.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sparsedict_b200.h"

namespace sdk {

constexpr int kWarp = 32;

// ---------------------------------------------------------------- dtypes ---
template <typename T> struct AccOf { using type = float; };
template <> struct AccOf<double> { using type = double; };

__device__ __forceinline__ float to_acc(float x) { return x; }
__device__ __forceinline__ double to_acc(double x) { return x; }
__device__ __forceinline__ float to_acc(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_acc(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_acc(float x);
template <> __device__ __forceinline__ float from_acc<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_acc<__half>(float x) { return __float2half_rn(x); }
__device__ __forceinline__ double from_acc_d(double x) { return x; }

template <typename T> __device__ __forceinline__ T cvt_out(typename AccOf<T>::type x) { return from_acc<T>(x); }
template <> __device__ __forceinline__ double cvt_out<double>(double x) { return x; }

template <typename V> __device__ __forceinline__ V quiet_nan();
template <> __device__ __forceinline__ float quiet_nan<float>() { return __int_as_float(0x7fc00000); }
template <> __device__ __forceinline__ double quiet_nan<double>() { return __longlong_as_double(0x7ff8000000000000LL); }

template <typename V> __device__ __forceinline__ V neg_inf();
template <> __device__ __forceinline__ float neg_inf<float>() { return __int_as_float(0xff800000); }
template <> __device__ __forceinline__ double neg_inf<double>() { return __longlong_as_double(0xfff0000000000000LL); }

__device__ __forceinline__ float exp_acc(float x) { return expf(x); }
__device__ __forceinline__ double exp_acc(double x) { return exp(x); }
__device__ __forceinline__ float log_acc(float x) { return logf(x); }
__device__ __forceinline__ double log_acc(double x) { return log(x); }
__device__ __forceinline__ float rint_acc(float x) { return rintf(x); }
__device__ __forceinline__ double rint_acc(double x) { return rint(x); }

// ------------------------------------------------------------ comparator ---
// True when (va, ia) ranks strictly above (vb, ib).
template <typename V>
__device__ __forceinline__ bool ranks_above(V va, int ia, V vb, int ib) {
  const bool na = va != va, nb = vb != vb;
  if (na | nb) return na && (!nb || ia < ib);
  return va > vb || (va == vb && ia < ib);
}

// Sentinel that ranks below every real entry, -inf scores included.
constexpr int kPadIndex = 0x7fffffff;

// Bitonic sort of P (power of two, >= 2) entries held in shared memory by one
// warp, best-ranked first.  Each lane owns P/64 compare-exchange pairs per
// step; the network is data independent.
template <typename V>
__device__ void warp_bitonic_sort(V* vals, int* idx, int P, int lane) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = lane; t < (P >> 1); t += kWarp) {
        const int i = 2 * t - (t & (stride - 1));
        const int j = i + stride;
        const bool best_first = (i & size) == 0;
        const V vi = vals[i], vj = vals[j];
        const int ii = idx[i], ij = idx[j];
        const bool swap = best_first ? ranks_above(vj, ij, vi, ii) : ranks_above(vi, ii, vj, ij);
        if (swap) {
          vals[i] = vj; vals[j] = vi;
          idx[i] = ij; idx[j] = ii;
        }
      }
      __syncwarp();
    }
  }
}

__device__ __forceinline__ int next_pow2_dev(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Sort the first `count` candidates of one row (padding to a power of two
// with sentinels) and keep the best min(count, topk).  Sets the row's
// threshold once topk candidates are held.
template <typename Acc>
__device__ int compact_row(Acc* vals, int* idx, int count, int topk, Acc* tau, int lane) {
  const int P = next_pow2_dev(count);
  for (int i = count + lane; i < P; i += kWarp) {
    vals[i] = neg_inf<Acc>();
    idx[i] = kPadIndex;
  }
  __syncwarp();
  warp_bitonic_sort(vals, idx, P, lane);
  const int kept = count < topk ? count : topk;
  if (kept == topk && lane == 0) *tau = vals[topk - 1];
  __syncwarp();
  return kept;
}

// --------------------------------------------------------- device status ---
// Bits set by kernels when they meet data they refuse to act on (an index
// outside [0, M) handed to the aggregate op, for example).  Read and cleared
// by sdk_device_status().
__device__ __forceinline__ void raise_device_status(unsigned int* status, unsigned int bit) {
  if (status) atomicOr(status, bit);
}

enum DeviceStatusBits : unsigned int {
  kStatusIndexOutOfRange = 1u,
  kStatusWaitTimeout = 2u,
};

unsigned int* device_status_ptr();  // defined in capi.cu
cudaMemPool_t scratch_pool();       // this library's stream-ordered scratch pool (capi.cu)

// ------------------------------------------------------ launch geometry ---
struct SliceGeometry {
  // Rows of slice s are [row_begin(s), row_begin(s+1)) in the logical row
  // order.  Uniform slices have n rows each; grouped slices read offsets.
  const int32_t* row_offsets;  // nullable, slices+1 entries
  int64_t slices;
  int64_t n;  // rows per slice when uniform, total rows when grouped
};

__device__ __forceinline__ int64_t slice_row_begin(const SliceGeometry& g, int64_t s) {
  return g.row_offsets ? (int64_t)g.row_offsets[s] : s * g.n;
}

// The slice that holds logical row r (grouped: the last slice whose first
// row is <= r, which skips empty slices).
__device__ __forceinline__ int64_t slice_of_row(const SliceGeometry& g, int64_t r) {
  if (!g.row_offsets) return r / g.n;
  int64_t lo = 0, hi = g.slices - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if ((int64_t)g.row_offsets[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Map a CTA's tile id to (slice, first row, row count) for tiles of `tile`
// rows.  Grouped geometry launches ceil(total/tile)+slices CTAs; surplus
// CTAs get count 0.
__device__ __forceinline__ void locate_tile(const SliceGeometry& g, int64_t tile_id, int tile,
                                            int64_t* slice, int64_t* row0, int* count) {
  if (!g.row_offsets) {
    const int64_t per = (g.n + tile - 1) / tile;
    *slice = tile_id / per;
    const int64_t local = (tile_id % per) * tile;
    *row0 = *slice * g.n + local;
    const int64_t left = g.n - local;
    *count = (int)(left < tile ? left : tile);
    return;
  }
  int64_t before = 0;
  for (int64_t s = 0; s < g.slices; ++s) {
    const int64_t b = g.row_offsets[s], e = g.row_offsets[s + 1];
    const int64_t tiles = (e - b + tile - 1) / tile;
    if (tile_id < before + tiles) {
      *slice = s;
      *row0 = b + (tile_id - before) * tile;
      const int64_t left = e - *row0;
      *count = (int)(left < tile ? left : tile);
      return;
    }
    before += tiles;
  }
  *slice = 0;
  *row0 = 0;
  *count = 0;
}

}  // namespace sdk
