// Deterministic key-major backward of top-k attention, bf16/fp16 with
// d = dv = 64 (the reference's B1 _backward_dq and B2 _backward_dkv,
// kernels/fused_topk_attn.py:609-977, restated without atomics).
//
// The reference (and sparse_bwd_d64 in bwd.cu) scatters dK/dV with one
// atomic add per (query row, selected key, feature).  Here every output is
// written exactly once, in a fixed summation order:
//
//   rows       one warp per query row i (lanes in four groups of eight, eight
//              lanes per 128-byte row, four gathered rows per load): over the
//              row's k selected keys j it forms s_ij = q_i·k_j,
//              g_ij = dout_i·v_j, P_ij = exp(scale·s_ij - lse_i) and the sums
//              delta_i = sum_j P_ij g_ij, A_i = sum_j P_ij g_ij k_j,
//              B_i = sum_j P_ij k_j in one pass over the gathered rows;
//              dq_i = scale·(A_i - delta_i B_i) = scale·sum_j dS_ij k_j
//              (dS = P (g - delta)).  It writes dq_i and (lse_i, delta_i).
//   transpose  a stable counting sort of each slice's (row, key) pairs by
//              key, in three launches over chunks of CH rows (one warp per
//              chunk): count (the chunk's per-key 16-bit counts, from a
//              shared-memory histogram), scan (per slice: for each key the
//              exclusive sum over the slice's chunks in order, and the key
//              offsets), place (each warp walks its chunk's entries in order
//              from its prefix cursors, equal keys inside a 32-entry batch
//              ranked by lane) — giving each key the list of rows that
//              selected it, in ascending row order.
//   keys       one warp per key j: over its rows i (four per load, eight
//              lanes per row) it recomputes s_ij, g_ij, P_ij and dS_ij from
//              the gathered q_i, dout_i and (lse_i, delta_i) and sums
//              dK_j = scale·sum_i dS_ij q_i and dV_j = sum_i P_ij dout_i in
//              registers; the four lane groups are added in a fixed order and
//              the row is written once (in the input dtype, or added to fp32
//              accumulators).
//
// The result is bit-identical from run to run and needs no zeroed
// accumulators and no conversion pass.  Keys no row selected get zeros.
#include "common.cuh"
#include "kernels.h"

namespace sdk {
namespace {

constexpr int D = 64;
constexpr int RW = 8;        // warps per block of the row and key passes
constexpr int CH = 256;      // rows per transpose chunk (one warp)
constexpr int TW = 6;        // chunk warps per block of the count and place kernels
constexpr int SCAN_NT = 1024;    // threads of a scan block (one per slice)
constexpr int kMaxKeys = 16384;  // keys per slice the 16-bit chunk histograms hold

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int h = 0; h < 8; ++h) f[h] = to_acc(e[h]);
}

__device__ __forceinline__ float dot8(const float (&a)[8], const float (&b)[8]) {
  float s = 0.f;
#pragma unroll
  for (int h = 0; h < 8; ++h) s = fmaf(a[h], b[h], s);
  return s;
}

__device__ __forceinline__ float group_sum8(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x;
}

struct KmArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* dout;
  const int32_t* top_idx;
  const float* lse;
  void* dq;
  void* dk;  // input dtype, or fp32 accumulators (out_acc)
  void* dv;
  SliceGeometry geo;
  const int32_t* row_index;
  int64_t rows, m;
  int64_t phys_rows;   // rows of q / dout (the physical row space)
  int topk;
  float scale;
  unsigned int* status;
  float2* rowstat;     // [physical row] (lse, delta)
  int32_t* key_off;    // [slices][m + 1] start of each key's row list
  int32_t* key_rows;   // [rows * topk] physical rows, grouped by key
  uint32_t* chunk_cnt; // [chunks][m / 2] 16-bit per-key counts, then prefixes
  int64_t chunks;      // chunk ids launched (grouped: surplus ids are empty)
  int out_acc;         // 1: dk/dv are fp32 accumulators
  int accumulate;      // with out_acc: add to them instead of overwriting
};

// ------------------------------------------------------------- row pass ---
template <typename T>
__global__ void __launch_bounds__(RW * kWarp, 4) km_rows(KmArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 3, l8 = lane & 7;
  const T* __restrict__ q = static_cast<const T*>(a.q);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  for (int64_t r = (int64_t)blockIdx.x * RW + warp; r < a.rows; r += (int64_t)gridDim.x * RW) {
    const int64_t slice = slice_of_row(a.geo, r);
    const int64_t pr = a.row_index ? (int64_t)a.row_index[r] : r;
    const uint4* __restrict__ kmat = reinterpret_cast<const uint4*>(static_cast<const T*>(a.k) + slice * a.m * D) + l8;
    const uint4* __restrict__ vmat = reinterpret_cast<const uint4*>(static_cast<const T*>(a.v) + slice * a.m * D) + l8;
    float qf[8], df[8];
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(q + pr * D) + l8), qf);
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(dout + pr * D) + l8), df);
    const float l = a.lse[r];
    int i0 = -1, i1 = -1;  // slots lane and lane + 32
    if (lane < a.topk) i0 = a.top_idx[r * a.topk + lane];
    if (lane + 32 < a.topk) i1 = a.top_idx[r * a.topk + lane + 32];
    const bool bad0 = lane < a.topk && (i0 < 0 || i0 >= a.m), bad1 = lane + 32 < a.topk && (i1 < 0 || i1 >= a.m);
    if (bad0 || bad1) {
      if ((bad0 && i0 >= 0) || (bad1 && i1 >= 0)) raise_device_status(a.status, kStatusIndexOutOfRange);
      if (bad0) i0 = -1;
      if (bad1) i1 = -1;
    }
    float A[8], B[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) A[h] = B[h] = 0.f;
    float part = 0.f;
    const int iters = (a.topk + 3) >> 2;
#pragma unroll 4
    for (int it = 0; it < iters; ++it) {
      const int j = 4 * it + grp;
      const int key = __shfl_sync(0xffffffffu, it < 8 ? i0 : i1, j & 31);
      float kf[8], vf[8];
      const bool ok = j < a.topk && key >= 0;
      uint4 ku = make_uint4(0u, 0u, 0u, 0u), vu = ku;
      if (ok) {
        ku = __ldg(kmat + (int64_t)key * 8);
        vu = __ldg(vmat + (int64_t)key * 8);
      }
      unpack8<T>(ku, kf);
      unpack8<T>(vu, vf);
      const float s = group_sum8(dot8(qf, kf));
      const float g = group_sum8(dot8(df, vf));
      const float p = ok ? __expf(s * a.scale - l) : 0.f;
      const float pg = p * g;
      part += pg;
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        A[h] = fmaf(pg, kf[h], A[h]);
        B[h] = fmaf(p, kf[h], B[h]);
      }
    }
    // every lane of a group holds that group's slot sums: add the four groups
    part += __shfl_xor_sync(0xffffffffu, part, 8);
    part += __shfl_xor_sync(0xffffffffu, part, 16);
    const float delta = part;
    float dq[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      dq[h] = fmaf(-delta, B[h], A[h]);
      dq[h] += __shfl_xor_sync(0xffffffffu, dq[h], 8);
      dq[h] += __shfl_xor_sync(0xffffffffu, dq[h], 16);
    }
    if (grp == 0) {
      uint4 o;
      T* e = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int h = 0; h < 8; ++h) e[h] = from_acc<T>(dq[h] * a.scale);
      reinterpret_cast<uint4*>(static_cast<T*>(a.dq) + pr * D)[l8] = o;
    }
    if (lane == 0) a.rowstat[pr] = make_float2(l, delta);
  }
}

// ------------------------------------------------------------ transpose ---
// Chunk c: rows [row0, row0 + count) of one slice (locate_tile with CH rows).
// A chunk's histogram holds m 16-bit counters, two per 32-bit word; a chunk
// has at most CH rows, so a key's count (one entry per row for distinct
// selections) stays far below 2^16, and a slice's per-key prefix stays below
// 2^16 with at most 65535 rows per slice.
__device__ __forceinline__ uint32_t half_get(uint32_t w, int key) { return (w >> ((key & 1) * 16)) & 0xffffu; }

__global__ void __launch_bounds__(TW * kWarp) km_count(KmArgs a) {
  extern __shared__ uint32_t csm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * TW + warp;
  if (c >= a.chunks) return;
  const int m = (int)a.m, hw = (m + 1) >> 1;
  uint32_t* h = csm + warp * hw;
  for (int i = lane; i < hw; i += kWarp) h[i] = 0u;
  __syncwarp();
  int64_t slice, row0;
  int count;
  locate_tile(a.geo, c, CH, &slice, &row0, &count);
  const int64_t e0 = row0 * a.topk, e1 = (row0 + count) * a.topk;
  constexpr int U = 8;  // eight 32-entry batches in flight
  for (int64_t e = e0; e < e1; e += U * kWarp) {
    int key[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t ee = e + u * kWarp + lane;
      key[u] = ee < e1 ? a.top_idx[ee] : -1;
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (key[u] >= 0 && key[u] < m) atomicAdd(&h[key[u] >> 1], 1u << ((key[u] & 1) * 16));
  }
  __syncwarp();
  uint32_t* dst = a.chunk_cnt + c * hw;
  for (int i = lane; i < hw; i += kWarp) dst[i] = h[i];
}

// One block per slice: each thread walks counter words (two keys) over the
// slice's chunks in order, replacing each count by the exclusive prefix, and
// keeps the per-key totals; a block-wide exclusive scan of the totals gives
// the key offsets.
__global__ void __launch_bounds__(SCAN_NT) km_scan(KmArgs a) {
  extern __shared__ uint32_t ssm[];  // [hw] per-key totals, two per word
  __shared__ int32_t wsum[SCAN_NT / kWarp];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t slice = blockIdx.x;
  const int m = (int)a.m, hw = (m + 1) >> 1;
  int64_t rb, re, c0;
  if (a.geo.row_offsets) {
    rb = a.geo.row_offsets[slice];
    re = a.geo.row_offsets[slice + 1];
    c0 = 0;
    for (int64_t s = 0; s < slice; ++s)
      c0 += ((int64_t)a.geo.row_offsets[s + 1] - a.geo.row_offsets[s] + CH - 1) / CH;
  } else {
    rb = slice * a.geo.n;
    re = rb + a.geo.n;
    c0 = slice * ((a.geo.n + CH - 1) / CH);
  }
  const int64_t nc = (re - rb + CH - 1) / CH;
  for (int w = t; w < hw; w += SCAN_NT) {
    uint32_t run = 0u;  // two 16-bit running sums (no carry: each stays below 2^16)
    constexpr int U = 8;  // chunk words in flight
    for (int64_t cb = c0; cb < c0 + nc; cb += U) {
      uint32_t v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = cb + u < c0 + nc ? a.chunk_cnt[(cb + u) * hw + w] : 0u;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (cb + u < c0 + nc) a.chunk_cnt[(cb + u) * hw + w] = run;
        run += v[u];
      }
    }
    ssm[w] = run;
  }
  __syncthreads();
  // keys [k0, k1) of thread t, contiguous
  const int per = (m + SCAN_NT - 1) / SCAN_NT;
  const int k0 = t * per < m ? t * per : m, k1 = k0 + per < m ? k0 + per : m;
  int32_t local = 0;
  for (int key = k0; key < k1; ++key) local += (int32_t)half_get(ssm[key >> 1], key);
  int32_t incl = local;
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == kWarp - 1) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int32_t x = lane < SCAN_NT / kWarp ? wsum[lane] : 0;
    int32_t xi = x;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += y;
    }
    if (lane < SCAN_NT / kWarp) wsum[lane] = xi - x;
  }
  __syncthreads();
  int32_t base = (int32_t)(rb * a.topk) + wsum[warp] + (incl - local);
  int32_t* koff = a.key_off + slice * (a.m + 1);
  for (int key = k0; key < k1; ++key) {
    koff[key] = base;
    base += (int32_t)half_get(ssm[key >> 1], key);
  }
  // the end of the last key's list: the slice start plus every counted entry
  // (entries with keys outside [0, m) are not listed)
  if (t == SCAN_NT - 1) koff[m] = base;
}

__global__ void __launch_bounds__(TW * kWarp) km_place(KmArgs a) {
  extern __shared__ uint32_t psm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * TW + warp;
  if (c >= a.chunks) return;
  const int m = (int)a.m, hw = (m + 1) >> 1;
  int64_t slice, row0;
  int count;
  locate_tile(a.geo, c, CH, &slice, &row0, &count);
  if (count <= 0) return;
  uint32_t* cur = psm + warp * hw;
  const uint32_t* src = a.chunk_cnt + c * hw;
  for (int i = lane; i < hw; i += kWarp) cur[i] = src[i];
  __syncwarp();
  const int32_t* koff = a.key_off + slice * (a.m + 1);
  const int64_t rb = slice_row_begin(a.geo, slice);
  const int64_t lo = rb * a.topk, hi = (int64_t)koff[m];  // the slice's list range
  const int64_t e0 = row0 * a.topk, e1 = (row0 + count) * a.topk;
  const unsigned lt = (1u << lane) - 1u;
  // row of an entry: floor((x + 0.5) / topk) for the chunk-local entry x < CH * 64;
  // the float quotient's error (< 2^-13) stays below the 1/(2 topk) margin
  const float inv_topk = 1.f / (float)a.topk;
  constexpr int U = 8;
  for (int64_t e = e0; e < e1; e += U * kWarp) {
    int keys[U];
    int32_t kb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t ee = e + u * kWarp + lane;
      keys[u] = ee < e1 ? a.top_idx[ee] : -1;
      if (keys[u] >= m) keys[u] = -1;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) kb[u] = keys[u] >= 0 ? koff[keys[u]] : 0;
    // the batches in order (ranks stay in row order across batches)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int key = keys[u];
      const int64_t ee = e + u * kWarp + lane;
      const unsigned same = __match_any_sync(0xffffffffu, key);
      const int rank = __popc(same & lt);
      int64_t pos = 0;
      if (key >= 0) pos = (int64_t)kb[u] + half_get(cur[key >> 1], key) + rank;
      __syncwarp();
      if (key >= 0 && rank == 0) atomicAdd(&cur[key >> 1], (uint32_t)__popc(same) << ((key & 1) * 16));
      __syncwarp();
      if (key >= 0) {
        if (pos >= lo && pos < hi) {
          const int64_t r = row0 + (int64_t)(((float)(int)(ee - e0) + 0.5f) * inv_topk);
          a.key_rows[pos] = a.row_index ? a.row_index[r] : (int32_t)r;
        } else {
          raise_device_status(a.status, kStatusIndexOutOfRange);  // inconsistent counts: duplicate keys in a row
        }
      }
    }
  }
}

// ------------------------------------------------------------- key pass ---
template <typename T>
__global__ void __launch_bounds__(RW * kWarp, 4) km_keys(KmArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 3, l8 = lane & 7;
  const int64_t total = a.geo.slices * a.m;
  const T* __restrict__ q = static_cast<const T*>(a.q);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  for (int64_t kk = (int64_t)blockIdx.x * RW + warp; kk < total; kk += (int64_t)gridDim.x * RW) {
    const int64_t slice = kk / a.m, key = kk - slice * a.m;
    float kf[8], vf[8];
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(a.k) + kk * D) + l8), kf);
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(a.v) + kk * D) + l8), vf);
    const int32_t b0 = a.key_off[slice * (a.m + 1) + key], b1 = a.key_off[slice * (a.m + 1) + key + 1];
    float dk[8], dv[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) dk[h] = dv[h] = 0.f;
    for (int32_t c0 = b0; c0 < b1; c0 += kWarp) {
      const int32_t my = c0 + lane < b1 ? a.key_rows[c0 + lane] : -1;
      const int cnt = b1 - c0 < kWarp ? b1 - c0 : kWarp;
#pragma unroll 2
      for (int t = 0; t < cnt; t += 4) {
        const int src = t + grp;
        const int32_t row = __shfl_sync(0xffffffffu, my, src & 31);
        const bool ok = src < cnt && row >= 0 && row < a.phys_rows;
        uint4 qu = make_uint4(0u, 0u, 0u, 0u), du = qu;
        float2 st = make_float2(0.f, 0.f);
        if (ok) {
          qu = __ldg(reinterpret_cast<const uint4*>(q + (int64_t)row * D) + l8);
          du = __ldg(reinterpret_cast<const uint4*>(dout + (int64_t)row * D) + l8);
          st = a.rowstat[row];
        }
        float qf[8], df[8];
        unpack8<T>(qu, qf);
        unpack8<T>(du, df);
        const float s = group_sum8(dot8(qf, kf));
        const float g = group_sum8(dot8(df, vf));
        const float p = ok ? __expf(s * a.scale - st.x) : 0.f;
        const float ds = p * (g - st.y);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          dk[h] = fmaf(ds, qf[h], dk[h]);
          dv[h] = fmaf(p, df[h], dv[h]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      dk[h] += __shfl_xor_sync(0xffffffffu, dk[h], 8);
      dk[h] += __shfl_xor_sync(0xffffffffu, dk[h], 16);
      dv[h] += __shfl_xor_sync(0xffffffffu, dv[h], 8);
      dv[h] += __shfl_xor_sync(0xffffffffu, dv[h], 16);
    }
    if (a.dk == a.dv) {
      // keys and values are one dictionary: its gradient is dK + dV
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        dv[h] = fmaf(dk[h], a.scale, dv[h]);
        dk[h] = 0.f;
      }
    }
    if (grp == 0) {
      if (a.out_acc) {
        float4* pk = reinterpret_cast<float4*>(static_cast<float*>(a.dk) + kk * D) + 2 * l8;
        float4* pv = reinterpret_cast<float4*>(static_cast<float*>(a.dv) + kk * D) + 2 * l8;
        float4 k0 = make_float4(dk[0] * a.scale, dk[1] * a.scale, dk[2] * a.scale, dk[3] * a.scale);
        float4 k1 = make_float4(dk[4] * a.scale, dk[5] * a.scale, dk[6] * a.scale, dk[7] * a.scale);
        float4 v0 = make_float4(dv[0], dv[1], dv[2], dv[3]), v1 = make_float4(dv[4], dv[5], dv[6], dv[7]);
        if (a.accumulate) {
          const float4 ov0 = pv[0], ov1 = pv[1];
          if (a.dk != a.dv) {
            const float4 ok0 = pk[0], ok1 = pk[1];
            k0.x += ok0.x; k0.y += ok0.y; k0.z += ok0.z; k0.w += ok0.w;
            k1.x += ok1.x; k1.y += ok1.y; k1.z += ok1.z; k1.w += ok1.w;
          }
          v0.x += ov0.x; v0.y += ov0.y; v0.z += ov0.z; v0.w += ov0.w;
          v1.x += ov1.x; v1.y += ov1.y; v1.z += ov1.z; v1.w += ov1.w;
        }
        if (a.dk != a.dv) {
          pk[0] = k0;
          pk[1] = k1;
        }
        pv[0] = v0;
        pv[1] = v1;
      } else {
        uint4 ok_, ov_;
        T* ek = reinterpret_cast<T*>(&ok_);
        T* ev = reinterpret_cast<T*>(&ov_);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          ek[h] = from_acc<T>(dk[h] * a.scale);
          ev[h] = from_acc<T>(dv[h]);
        }
        if (a.dk != a.dv) reinterpret_cast<uint4*>(static_cast<T*>(a.dk) + kk * D)[l8] = ok_;
        reinterpret_cast<uint4*>(static_cast<T*>(a.dv) + kk * D)[l8] = ov_;
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Transpose chunks: enough for uniform slices (slices * ceil(n / CH)) and
// for grouped ones (ceil(rows / CH) + slices) alike.
int64_t km_chunk_bound(int64_t rows, int64_t slices) { return (rows + CH - 1) / CH + slices; }

// Workspace layout (256-byte aligned parts): rowstat [phys rows] float2,
// key_off [slices][m + 1] int32, key_rows [rows * topk] int32, chunk
// counters [chunks][(m + 1) / 2] uint32.
struct KmLayout {
  size_t rowstat, key_off, key_rows, chunk_cnt, total;
};

KmLayout km_layout(int64_t rows, int64_t phys_rows, int64_t slices, int64_t m, int topk) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  KmLayout L;
  L.rowstat = 0;
  L.key_off = up((size_t)phys_rows * sizeof(float2));
  L.key_rows = L.key_off + up((size_t)slices * (size_t)(m + 1) * 4);
  L.chunk_cnt = L.key_rows + up((size_t)rows * (size_t)topk * 4);
  L.total = L.chunk_cnt + up((size_t)km_chunk_bound(rows, slices) * (size_t)((m + 1) / 2) * 4);
  return L;
}

template <typename T>
int launch_km(const BwdLaunch& L, void* dk, void* dv, int out_acc, int accumulate, void* ws) {
  const int64_t rows = L.row_offsets ? L.n : L.slices * L.n;
  KmArgs a;
  a.q = L.q; a.k = L.k; a.v = L.v; a.dout = L.dout; a.top_idx = L.top_idx;
  a.lse = static_cast<const float*>(L.lse);
  a.dq = L.dq;
  a.dk = dk;
  a.dv = dv;
  a.geo = SliceGeometry{L.row_offsets, L.slices, L.n};
  a.row_index = L.row_index;
  a.rows = rows;
  a.m = L.m;
  a.topk = L.topk;
  a.scale = (float)L.scale;
  a.status = L.status;
  const KmLayout lay = km_layout(rows, rows, L.slices, L.m, L.topk);
  uint8_t* w = static_cast<uint8_t*>(ws);
  a.rowstat = reinterpret_cast<float2*>(w + lay.rowstat);
  a.key_off = reinterpret_cast<int32_t*>(w + lay.key_off);
  a.key_rows = reinterpret_cast<int32_t*>(w + lay.key_rows);
  a.chunk_cnt = reinterpret_cast<uint32_t*>(w + lay.chunk_cnt);
  a.chunks = L.row_offsets ? km_chunk_bound(rows, L.slices) : L.slices * ((L.n + CH - 1) / CH);
  a.phys_rows = rows;
  a.out_acc = out_acc;
  a.accumulate = accumulate;
  if (rows > 0) {
    km_rows<T><<<(unsigned)((rows + RW - 1) / RW), RW * kWarp, 0, L.stream>>>(a);
    if (cudaPeekAtLastError() != cudaSuccess) return SDK_ERR_CUDA;
  }
  const size_t hsm = (size_t)TW * (size_t)((L.m + 1) / 2) * 4;  // one histogram per warp
  const size_t ssm = (size_t)((L.m + 1) / 2) * 4;
  if (cudaFuncSetAttribute(km_count, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hsm) != cudaSuccess ||
      cudaFuncSetAttribute(km_place, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hsm) != cudaSuccess ||
      cudaFuncSetAttribute(km_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm) != cudaSuccess)
    return SDK_ERR_CUDA;
  const unsigned cblocks = (unsigned)((a.chunks + TW - 1) / TW);
  if (a.chunks > 0) {
    km_count<<<cblocks, TW * kWarp, hsm, L.stream>>>(a);
    km_scan<<<(unsigned)L.slices, SCAN_NT, ssm, L.stream>>>(a);
    km_place<<<cblocks, TW * kWarp, hsm, L.stream>>>(a);
  } else {
    km_scan<<<(unsigned)L.slices, SCAN_NT, ssm, L.stream>>>(a);
  }
  if (cudaPeekAtLastError() != cudaSuccess) return SDK_ERR_CUDA;
  const int64_t keys = L.slices * L.m;
  km_keys<T><<<(unsigned)((keys + RW - 1) / RW), RW * kWarp, 0, L.stream>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

}  // namespace

bool bwd_keymajor_supports(const BwdLaunch& L) {
  if (L.dtype != SDK_DTYPE_BF16 && L.dtype != SDK_DTYPE_F16) return false;
  if (L.d != D || L.dv != D || L.topk < 1 || L.topk > 64 || L.score_grid != 0) return false;
  if (L.seg_bias || L.dseg_bias) return false;
  if (L.m < 1 || L.m > kMaxKeys) return false;
  const int64_t rows = L.row_offsets ? L.n : L.slices * L.n;
  // 16-bit per-key cursors: at most 65535 rows per slice (grouped: in all);
  // int32 list positions
  if (L.n > 65535) return false;
  if (rows * (int64_t)L.topk > 0x7fffffff || L.slices * L.m > 0x7fffffff || L.slices > 0x7fffffff) return false;
  return aligned16(L.q) && aligned16(L.k) && aligned16(L.v) && aligned16(L.dout) && aligned16(L.dq);
}

size_t bwd_keymajor_workspace(int64_t rows, int64_t slices, int64_t m, int topk) {
  if (rows < 0 || slices < 1 || m < 1 || topk < 1) return 0;
  return km_layout(rows, rows, slices, m, topk).total;
}

int bwd_keymajor(const BwdLaunch& L, void* dk, void* dv, int out_acc, int accumulate, void* ws) {
  if (L.dtype == SDK_DTYPE_BF16) return launch_km<__nv_bfloat16>(L, dk, dv, out_acc, accumulate, ws);
  return launch_km<__half>(L, dk, dv, out_acc, accumulate, ws);
}

}  // namespace sdk
