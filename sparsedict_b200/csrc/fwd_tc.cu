// Fused top-k attention forward on the 5th-generation tensor cores (sm_100a).
//
// One CTA owns 128 query rows of one (b, h) slice (d = dv = 64, bf16 or fp16)
// and streams the slice's keys in tiles of 128:
//
//   warp 0      TMA producer: the Q tile once, then K tiles into a 3-stage
//               ring of 128-byte-swizzled shared-memory buffers;
//   warp 1      allocates 256 TMEM columns and issues tcgen05.mma
//               (M=128, N=128, K=16 x 4) of S = Q·Kᵀ into one of two TMEM
//               accumulators, committing to the "S full" and "stage free"
//               mbarriers;
//   warps 4..7  selection: thread i owns query row i (TMEM lane i), reads
//               its 128 scores of the tile with tcgen05.ld 32 columns at a
//               time, keeps every key that beats the row's running
//               threshold in a shared-memory candidate list and, when the
//               list could overflow, raises the threshold with a sampled
//               pivot and compacts the list.  The score row never reaches
//               global memory.
//
// After the last tile each selection thread trims its list to exactly k
// keys (lowest-rank-first removal; ties at the k-th score keep the lower
// key index), writes the indices, the row LSE, and the softmax-weighted
// sum of the gathered value rows.  The k indices of a row are written in no
// particular order; the set is the reference's top-k set.
//
// Selection runs on the raw dot products; scale = 1/(T·sqrt(d)) > 0 is
// applied in the epilogue (for d = 64 the scale is a power of two, so the
// order is exactly that of the scaled scores).
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sdk {
namespace {

using namespace sm100;

constexpr int TQ = 128;  // query rows per CTA (TMEM lanes)
constexpr int TK = 128;  // keys per score tile (MMA N)
constexpr int D = 64;    // feature width (one 128-byte swizzle row)
constexpr int KSTAGES = 3;
constexpr int CAP = 192;  // candidate slots per row
constexpr int NT = 256;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TILE_BYTES = TK * D * 2;

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TQ * D * 2;
constexpr int OFF_CV = OFF_K + KSTAGES * (int)TILE_BYTES;
constexpr int OFF_CI = OFF_CV + CAP * TQ * 4;
constexpr int OFF_BAR = OFF_CI + CAP * TQ * 2;
constexpr int NBARS = 1 + 2 * KSTAGES + 4;
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack

struct TcArgs {
  const void* v;
  void* out;
  int32_t* top_idx;
  float* lse;
  float* top_scores;
  int64_t n, m;
  int tiles_per_slice, topk;
  float scale;
  unsigned int* status;
};

// ----------------------------------------------------------- selection ---
// Candidate list of row r: slots s = 0..cnt-1 at cv[s*TQ + r] / ci[s*TQ + r]
// (row-fastest, so the 32 lanes of a warp hit 32 distinct banks).

// Order-preserving 64-bit rank key: larger key = ranks higher.  The high
// word maps the float onto an unsigned order (NaN highest, -0 == +0); the
// low word is the complemented key index, so equal scores rank the lower
// index higher.
__device__ __forceinline__ uint64_t rank_key(float x, uint32_t idx) {
  uint32_t u;
  if (x != x) {
    u = 0xffffffffu;
  } else {
    u = __float_as_uint(x + 0.0f);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  return ((uint64_t)u << 32) | (uint64_t)(0xffffffffu - idx);
}

__device__ __forceinline__ void sort16_desc(float (&x)[16]) {
#pragma unroll
  for (int size = 2; size <= 16; size <<= 1)
#pragma unroll
    for (int st = size >> 1; st > 0; st >>= 1)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = i ^ st;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float hi = fmaxf(x[i], x[j]), lo = fminf(x[i], x[j]);
          x[i] = desc ? hi : lo;
          x[j] = desc ? lo : hi;
        }
      }
}

// Counts of listed values >= each of four pivots, in one pass.
__device__ __forceinline__ void count4(const float* cv, int r, int cnt, const float (&p)[4], int (&c)[4]) {
  c[0] = c[1] = c[2] = c[3] = 0;
#pragma unroll 4
  for (int s = 0; s < cnt; ++s) {
    const float x = cv[s * TQ + r];
#pragma unroll
    for (int q = 0; q < 4; ++q) c[q] += !(x < p[q]);
  }
}

// Raise the row's threshold to the highest of 16 sampled list values that at
// least `topk` listed keys meet (keys seen later rank below these on equal
// scores, so `!(s <= tau)` stays exact) and drop the keys below it.  The
// search starts near the sample rank expected to keep about
// topk + slack*cnt/16 keys and tests four candidate pivots per pass.
__device__ void compact_list(float* cv, uint16_t* ci, int r, int& cnt, float& tau, int topk, int slack) {
  float smp[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float x = cv[((j * cnt) >> 4) * TQ + r];
    smp[j] = (x != x) ? __int_as_float(0x7f800000) : x;
  }
  sort16_desc(smp);
  int t = (16 * topk) / (cnt > 0 ? cnt : 1) + slack - 1;
  t = t < 0 ? 0 : (t > 12 ? 12 : t);
  float pivot = __int_as_float(0xff800000);
  bool found = false;
  for (int pass = 0; pass < 4 && !found; ++pass) {
    float p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int want = t + q;
      float v = smp[15];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j == want) v = smp[j];
      p[q] = v;
    }
    int c[4];
    count4(cv, r, cnt, p, c);
#pragma unroll
    for (int q = 3; q >= 0; --q)
      if (c[q] >= topk) {
        pivot = p[q];
        found = true;
      }
    t = t + 4 > 12 ? 12 : t + 4;
  }
  uint32_t w = 0;
  const uint32_t cvb = smem_addr(cv) + 4u * r, cib = smem_addr(ci) + 2u * r;
  for (int s = 0; s < cnt; ++s) {
    const float x = cv[s * TQ + r];
    const uint32_t i = ci[s * TQ + r];
    const uint32_t keep = (uint32_t)!(x < pivot);
    st_shared_f32_if(cvb + w * (4u * TQ), x, keep);
    st_shared_u16_if(cib + w * (2u * TQ), i, keep);
    w += keep;
  }
  cnt = (int)w;
  tau = pivot;
}

// Remove lowest-ranked keys until exactly `topk` remain; the survivors are
// the list's top-k by (score descending, index ascending).
__device__ void trim_to_topk(float* cv, uint16_t* ci, int r, int& cnt, float& tau, int topk) {
  while (cnt > topk) {
    uint64_t worst = ~0ull;
    int pos = 0;
#pragma unroll 4
    for (int s = 0; s < cnt; ++s) {
      const uint64_t key = rank_key(cv[s * TQ + r], ci[s * TQ + r]);
      const bool lower = key < worst;
      worst = lower ? key : worst;
      pos = lower ? s : pos;
    }
    tau = cv[pos * TQ + r];
    const int last = cnt - 1;
    cv[pos * TQ + r] = cv[last * TQ + r];
    ci[pos * TQ + r] = ci[last * TQ + r];
    cnt = last;
  }
}

// Append every key of a 32-key chunk whose score passes !(x <= tau) to the
// row's list.  Branch-free: each key's slot is the running count and the
// stores are predicated instructions, so lanes never diverge per key.
__device__ __forceinline__ void append_chunk(const uint32_t* v, int valid, float tau, int key0, float* cv,
                                             uint16_t* ci, int r, int& cnt) {
  uint32_t slot = (uint32_t)cnt;
  const uint32_t cvb = smem_addr(cv) + 4u * r, cib = smem_addr(ci) + 2u * r;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float x = __uint_as_float(v[i]);
    const uint32_t take = (uint32_t)(i < valid && !(x <= tau));
    st_shared_f32_if(cvb + slot * (4u * TQ), x, take);
    st_shared_u16_if(cib + slot * (2u * TQ), (uint32_t)(key0 + i), take);
    slot += take;
  }
  cnt = (int)slot;
}

__device__ __forceinline__ float chunk_max(const uint32_t (&v)[32]) {
  float a[11];
#pragma unroll
  for (int g = 0; g < 10; ++g)
    a[g] = max3_nan(__uint_as_float(v[3 * g]), __uint_as_float(v[3 * g + 1]), __uint_as_float(v[3 * g + 2]));
  a[10] = max_nan(__uint_as_float(v[30]), __uint_as_float(v[31]));
  const float b0 = max3_nan(a[0], a[1], a[2]), b1 = max3_nan(a[3], a[4], a[5]),
              b2 = max3_nan(a[6], a[7], a[8]);
  const float b3 = max_nan(a[9], a[10]);
  return max_nan(max3_nan(b0, b1, b2), b3);
}

template <typename T>
__global__ void __launch_bounds__(NT, 1)
    fused_fwd_tc(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                 TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* qs = sm + OFF_Q;
  uint8_t* ks = sm + OFF_K;
  float* cv = reinterpret_cast<float*>(sm + OFF_CV);
  uint16_t* ci = reinterpret_cast<uint16_t*>(sm + OFF_CI);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 1 + KSTAGES;
  uint64_t* s_full = bars + 1 + 2 * KSTAGES;
  uint64_t* s_empty = s_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t slice = blockIdx.x / a.tiles_per_slice;
  const int64_t local0 = (int64_t)(blockIdx.x % a.tiles_per_slice) * TQ;
  const int rows = (int)((a.n - local0) < TQ ? (a.n - local0) : TQ);
  const int64_t row0 = slice * a.n + local0;
  const int ntiles = (int)((a.m + TK - 1) / TK);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4 * kWarp);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      mbar_arrive_expect_tx(q_full, TQ * D * 2);
      tma_load_2d(qs, &tmap_q, 0, (int)row0, q_full);
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % KSTAGES;
        const uint32_t ph = (uint32_t)(t / KSTAGES) & 1u;
        if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[s], TILE_BYTES);
        tma_load_2d(ks + s * TILE_BYTES, &tmap_k, 0, (int)(slice * a.m + (int64_t)t * TK), &k_full[s]);
        ++issued;
      }
      if (*abort_flag) {
        // let the copies already in flight land before the CTA exits
        for (int t = (issued > KSTAGES ? issued - KSTAGES : 0); t < issued; ++t) {
          const uint64_t t0 = global_timer();
          while (!mbar_try_wait(&k_full[t % KSTAGES], (uint32_t)(t / KSTAGES) & 1u) &&
                 global_timer() - t0 < kWaitLimitNs) {
          }
        }
        const uint64_t t0 = global_timer();
        while (!mbar_try_wait(q_full, 0) && global_timer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc_f16(sizeof(T) == 2 && !std::is_same<T, __half>::value, TQ, TK);
      const uint32_t q_addr = smem_addr(qs);
      int committed = -1;
      if (mbar_wait(q_full, 0, abort_flag)) {
        for (int t = 0; t < ntiles; ++t) {
          const int s = t % KSTAGES, b = t & 1;
          if (!mbar_wait(&k_full[s], (uint32_t)(t / KSTAGES) & 1u, abort_flag)) break;
          if (!mbar_wait(&s_empty[b], ((uint32_t)(t >> 1) & 1u) ^ 1u, abort_flag)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_addr(ks + s * TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_f16(tmem + b * TK, smem_desc_k128(q_addr + kk * 32), smem_desc_k128(k_addr + kk * 32), idesc,
                    kk > 0);
          mma_commit(&k_empty[s]);
          mma_commit(&s_full[b]);
          committed = t;
        }
      }
      if (*abort_flag && committed >= 0) {
        // wait for the last MMAs before TMEM is released
        const int b = committed & 1;
        const uint64_t t0 = global_timer();
        while (!mbar_try_wait(&s_full[b], (uint32_t)(committed >> 1) & 1u) && global_timer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp >= 4) {
    const int r = threadIdx.x - 4 * kWarp;  // row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)((warp - 4) * kWarp) << 16;
    float tau = __int_as_float(0x7fc00000);  // "no threshold yet"
    int cnt = 0;
    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int b = t & 1;
      if (!mbar_wait(&s_full[b], (uint32_t)(t >> 1) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t key_tile = (int64_t)t * TK;
      const int tile_valid = (int)((a.m - key_tile) < TK ? (a.m - key_tile) : TK);
      // All four 32-column chunks of this tile go to registers at once; the
      // TMEM buffer is released before any selection work so the next MMA
      // into it can start.
      uint32_t v[TK];
#pragma unroll
      for (int c = 0; c < TK / 32; ++c)
        tmem_load_32cols(tmem + lane_base + b * TK + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tmem_wait_load();
      tc_fence_before();
      mbar_arrive(&s_empty[b]);
      float mx[TK / 32];
#pragma unroll
      for (int c = 0; c < TK / 32; ++c) {
        if (tile_valid >= TK) {
          mx[c] = chunk_max(*reinterpret_cast<const uint32_t(*)[32]>(&v[c * 32]));
        } else {
          float m = __int_as_float(0xff800000);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i < tile_valid) m = max_nan(m, __uint_as_float(v[c * 32 + i]));
          mx[c] = m;
        }
      }
#pragma unroll
      for (int c = 0; c < TK / 32; ++c) {
        if (!__any_sync(0xffffffffu, !(mx[c] <= tau))) continue;
        append_chunk(&v[c * 32], tile_valid - c * 32, tau, (int)(key_tile + c * 32), cv, ci, r, cnt);
        // When one lane's list could overflow, every lane holding well over
        // k keys compacts in the same pass: under SIMT the warp pays for the
        // longest list either way.
        if (__any_sync(0xffffffffu, cnt > CAP - 32)) {
          if (cnt > a.topk + 32) {
            compact_list(cv, ci, r, cnt, tau, a.topk, 2);
            if (cnt > CAP - 32) trim_to_topk(cv, ci, r, cnt, tau, a.topk);
          }
        }
      }
    }
    if (ok && !*abort_flag) {
      if (cnt > a.topk + 16) compact_list(cv, ci, r, cnt, tau, a.topk, 1);
      trim_to_topk(cv, ci, r, cnt, tau, a.topk);
      if (r < rows) {
        const int64_t gr = row0 + r;
        float mx = cv[r];
        for (int j = 1; j < a.topk; ++j) mx = fmaxf(mx, cv[j * TQ + r]);
        const float mxs = mx * a.scale;
        float total = 0.f;
        for (int j = 0; j < a.topk; ++j) total += expf(cv[j * TQ + r] * a.scale - mxs);
        const float lse = mxs + logf(total);
        a.lse[gr] = lse;
        int32_t* idx_row = a.top_idx + gr * a.topk;
        for (int j = 0; j < a.topk; ++j) {
          idx_row[j] = ci[j * TQ + r];
          if (a.top_scores) a.top_scores[gr * a.topk + j] = cv[j * TQ + r] * a.scale;
        }
        float acc[D];
#pragma unroll
        for (int f = 0; f < D; ++f) acc[f] = 0.f;
        const T* vbase = static_cast<const T*>(a.v) + slice * a.m * D;
#pragma unroll 2
        for (int j = 0; j < a.topk; ++j) {
          const float p = expf(cv[j * TQ + r] * a.scale - lse);
          const uint4* vrow = reinterpret_cast<const uint4*>(vbase + (int64_t)ci[j * TQ + r] * D);
#pragma unroll
          for (int q4 = 0; q4 < D / 8; ++q4) {
            const uint4 u = __ldg(vrow + q4);
            const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int h = 0; h < 8; ++h) acc[q4 * 8 + h] = fmaf(p, to_acc(e[h]), acc[q4 * 8 + h]);
          }
        }
        uint4* orow = reinterpret_cast<uint4*>(static_cast<T*>(a.out) + gr * D);
#pragma unroll
        for (int q4 = 0; q4 < D / 8; ++q4) {
          uint4 u;
          T* e = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int h = 0; h < 8; ++h) e[h] = from_acc<T>(acc[q4 * 8 + h]);
          orow[q4] = u;
        }
      }
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) raise_device_status(a.status, kStatusWaitTimeout);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host ---
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

// Row-major [rows, 64] 16-bit matrix, 128-row boxes, 128-byte swizzle.
bool make_rows_map(CUtensorMap* map, const void* base, int64_t rows, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {(cuuint32_t)D, (cuuint32_t)TQ};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
int launch(const FwdLaunch& L) {
  CUtensorMap tq, tk;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (!make_rows_map(&tq, L.q, L.slices * L.n, bf16)) return SDK_ERR_CUDA;
  if (!make_rows_map(&tk, L.k, L.slices * L.m, bf16)) return SDK_ERR_CUDA;
  TcArgs a;
  a.v = L.v;
  a.out = L.out;
  a.top_idx = L.top_idx;
  a.lse = static_cast<float*>(L.lse);
  a.top_scores = static_cast<float*>(L.top_scores);
  a.n = L.n;
  a.m = L.m;
  a.tiles_per_slice = (int)((L.n + TQ - 1) / TQ);
  a.topk = L.topk;
  a.scale = (float)L.scale;
  a.status = L.status;
  const int64_t grid = L.slices * a.tiles_per_slice;
  if (grid <= 0) return SDK_OK;
  auto kern = fused_fwd_tc<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
    return SDK_ERR_CUDA;
  kern<<<(unsigned)grid, NT, SMEM_BYTES, L.stream>>>(tq, tk, a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool fwd_tensorcore_supports(const FwdLaunch& L) {
  if (L.dtype != SDK_DTYPE_BF16 && L.dtype != SDK_DTYPE_F16) return false;
  if (L.d != D || L.dv != D || L.score_grid != 0) return false;
  if (L.row_offsets || L.row_index) return false;
  if (L.m > 65536 || L.topk > 64 || L.n < 1) return false;
  if (L.slices * L.n > 0x7fffffff || L.slices * L.m > 0x7fffffff) return false;
  if (!aligned16(L.q) || !aligned16(L.k) || !aligned16(L.v) || !aligned16(L.out)) return false;
  return encode_fn() != nullptr;
}

int fwd_tensorcore(const FwdLaunch& L) {
  if (L.dtype == SDK_DTYPE_BF16) return launch<__nv_bfloat16>(L);
  if (L.dtype == SDK_DTYPE_F16) return launch<__half>(L);
  return SDK_ERR_UNSUPPORTED;
}

}  // namespace sdk
