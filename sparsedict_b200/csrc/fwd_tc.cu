// Fused top-k attention forward on the 5th-generation tensor cores (sm_100a).
//
// One CTA owns 256 query rows of one (b, h) slice (d = dv = 64, bf16 or fp16)
// as two 128-row tiles, A and B, and streams the slice's keys in tiles of 128:
//
//   warp 0       TMA producer: both Q tiles once, then each K tile into one
//                128-byte-swizzled shared-memory buffer (the MMAs of a tile
//                take a fraction of a microsecond, a tile's selection several,
//                so one buffer never starves the pipeline);
//   warp 1       allocates 512 TMEM columns and issues tcgen05.mma
//                (M=128, N=128, K=16 x 4) of S_A = Q_A·Kᵀ and S_B = Q_B·Kᵀ
//                for every K tile, each into one of two TMEM accumulators of
//                its query tile, committing to "S full" / "stage free"
//                mbarriers;
//   warps 4..7   selection for tile A, warps 8..11 for tile B (two selection
//                warps per SM sub-partition): thread i of a group owns query
//                row i of its tile (TMEM lane i), reads its 128 scores of the
//                K tile with tcgen05.ld, and appends every key that beats the
//                row's running threshold to a slot-major shared-memory list.
//
// A list entry is 4 bytes: the upper 16 bits of the fp32 score's bit pattern
// (its bf16 truncation, which names the score's bf16 "bucket") and the 16-bit
// key index.  When a list could overflow it is compacted with a bucket pivot:
// the highest of 16 sampled buckets that at least k listed keys reach.  Keys
// below that bucket are dropped and the row's threshold becomes the lowest
// score of the bucket; both steps are exact (no top-k key is ever dropped).
// A row whose list cannot be shrunk that way (more than ~100 listed keys
// share the cut bucket, which needs heavily tied scores) is marked and
// re-selected exactly at the end, see below.
//
// After the last tile the survivors of each row (at most 96) are re-scored
// exactly: the row's Q values go to registers, the candidates' key indices
// move to the row's own unused list slots, and each candidate's fp32 score
// is recomputed from the gathered key row by one fixed FMA order, replacing
// its bucketed entry.  The exact cut to k keys uses order-preserving 64-bit
// keys (score, complemented index), so ties keep the lower key index.  Then
// the row LSE, the k indices (in no particular order; the set is the
// reference's top-k set) and the softmax-weighted sum of the gathered value
// rows are written.
//
// Marked rows are re-selected by their warp: lanes score 32 keys at a time
// with the same FMA order and keep an exact candidate list sorted by a warp
// bitonic network, as the CUDA-core kernel does.
//
// Selection runs on the raw dot products; scale = 1/(T·sqrt(d)) > 0 is
// applied in the epilogue (for d = 64 and T a power of two the scale is a
// power of two, so the order is exactly that of the scaled scores).
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sdk {
namespace {

using namespace sm100;

constexpr int TQ = 128;         // query rows per tile (TMEM lanes, MMA M)
constexpr int NTILE = 2;        // query tiles per CTA
constexpr int RS = TQ * NTILE;  // rows per CTA; row stride of the slot-major lists
constexpr int TK = 128;         // keys per score tile (MMA N)
constexpr int D = 64;           // feature width (one 128-byte swizzle row)
constexpr int KSTAGES = 1;
constexpr int CAP = 176;        // list slots per row
constexpr int FINAL_CAP = 96;   // most candidates a row may carry into exact re-scoring
constexpr int FIX_CAP = 128;    // exact list of a row re-selected by one warp
constexpr int NT = 384;
constexpr int NSEL = 8 * kWarp;  // selection threads
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TILE_BYTES = TK * D * 2;  // a K tile, also a Q tile

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + NTILE * (int)TILE_BYTES;
constexpr int OFF_LIST = OFF_K + KSTAGES * (int)TILE_BYTES;
constexpr int OFF_BAR = OFF_LIST + CAP * RS * 4;
constexpr int NBARS = 1 + 2 * KSTAGES + 4 * NTILE;
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
// After the stream: the key indices of a row's re-scored candidates go to
// the row's own list column above FINAL_CAP (two 16-bit indices per word),
// and the Q/K region holds one exact re-selection buffer per selection warp.
constexpr int OFF_FIX = 0;
constexpr int FIX_BYTES = FIX_CAP * 8 + 16;
static_assert(OFF_FIX + 8 * FIX_BYTES <= OFF_LIST, "post-stream buffers exceed the Q/K region");
static_assert(FINAL_CAP + (FINAL_CAP + 1) / 2 <= CAP, "re-scoring indices exceed the list column");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");

struct TcArgs {
  const void* q;
  const void* k;
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

// ---------------------------------------------------- bucketed list entries ---
// Order-preserving form of an entry: the high 16 bits order the buckets like
// their scores (negative scores complemented); the low 16 bits are not used.
__device__ __forceinline__ uint32_t ord_entry(uint32_t e) {
  return e ^ ((uint32_t)((int32_t)e >> 31) | 0x80000000u);
}

// Threshold after a compaction that kept every key of bucket >= p (p is an
// ordered bucket << 16): a later key x is dropped iff !(x > tau), i.e. iff its
// ordered score is <= p.  At least k kept keys rank at or above p, and a later
// key equal to them loses the index tie, so the drop is exact.
__device__ __forceinline__ float tau_of_bucket(uint32_t p) {
  if (p >= 0xff800000u) return __int_as_float(0x7f800000);  // only NaN ranks higher
  if (p < 0x00800000u) return __int_as_float(0x7fc00000);   // at or below -inf: admit all
  return __uint_as_float((p & 0x80000000u) ? (p & 0x7fffffffu) : ~p);
}

__device__ __forceinline__ void sort16_desc(uint32_t (&x)[16]) {
#pragma unroll
  for (int size = 2; size <= 16; size <<= 1)
#pragma unroll
    for (int st = size >> 1; st > 0; st >>= 1)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = i ^ st;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const uint32_t hi = max(x[i], x[j]), lo = min(x[i], x[j]);
          x[i] = desc ? hi : lo;
          x[j] = desc ? lo : hi;
        }
      }
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

template <typename V>
__device__ __forceinline__ V pick16(const V (&x)[16], int want) {
  V v = x[15];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (j == want) v = x[j];
  return v;
}

// Counts of row R's listed entries whose ordered form reaches each of four
// pivots.  Eight entries per step and two sets of counters keep several
// loads and adds in flight (the counters are the only dependency chains).
__device__ __forceinline__ void count4(const uint32_t* list, int R, int cnt, const uint32_t (&p)[4], int (&c)[4]) {
  int a[4] = {0, 0, 0, 0}, b[4] = {0, 0, 0, 0};
  int s = 0;
  for (; s + 8 <= cnt; s += 8) {
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = ord_entry(list[(s + i) * RS + R]);
#pragma unroll
    for (int i = 0; i < 8; i += 2)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        a[q] += (int)(o[i] >= p[q]);
        b[q] += (int)(o[i + 1] >= p[q]);
      }
  }
  for (; s < cnt; ++s) {
    const uint32_t o = ord_entry(list[s * RS + R]);
#pragma unroll
    for (int q = 0; q < 4; ++q) a[q] += (int)(o >= p[q]);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) c[q] = a[q] + b[q];
}

// Keep the entries whose ordered score reaches `pivot`, in place and in
// order.  Entries are read eight at a time ahead of the predicated stores:
// a store goes to a slot at or below the slot being read, so the batch
// already holds anything a store could overwrite, and the loads no longer
// wait on the stores one by one.
__device__ __forceinline__ int keep_pass(uint32_t* list, int R, int cnt, uint32_t pivot) {
  uint32_t w = 0;
  const uint32_t base = smem_addr(list) + 4u * R;
  int s = 0;
  for (; s + 8 <= cnt; s += 8) {
    uint32_t e[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = list[(s + i) * RS + R];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t keep = (uint32_t)(ord_entry(e[i]) >= pivot);
      st_shared_u32_if(base + w * (4u * RS), e[i], keep);
      w += keep;
    }
  }
  for (; s < cnt; ++s) {
    const uint32_t e = list[s * RS + R];
    const uint32_t keep = (uint32_t)(ord_entry(e) >= pivot);
    st_shared_u32_if(base + w * (4u * RS), e, keep);
    w += keep;
  }
  return (int)w;
}

// Shrink row R's list to the keys whose bucket reaches the highest of 16
// sampled buckets that at least `topk` listed keys reach (four candidate
// pivots per counting pass, starting near the sample rank expected to keep
// topk + slack*cnt/16 keys).  Returns false when no sampled pivot qualifies
// or nothing would be dropped.  Kept out of line: it runs rarely, and one
// copy keeps the streaming loop small enough for the instruction cache.
struct Compacted {
  int cnt;
  float tau;
  bool shrank;
};

__device__ __noinline__ Compacted compact_bucket(const uint32_t* list_c, int R, int cnt, float tau, int topk,
                                                 int slack) {
  uint32_t* list = const_cast<uint32_t*>(list_c);
  uint32_t smp[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) smp[j] = ord_entry(list[((j * cnt) >> 4) * RS + R]) & 0xffff0000u;
  sort16_desc(smp);
  int t = (16 * topk) / (cnt > 0 ? cnt : 1) + slack - 1;
  t = t < 0 ? 0 : (t > 12 ? 12 : t);
  uint32_t pivot = 0;
  bool found = false;
  for (int pass = 0; pass < 4 && !found; ++pass) {
    uint32_t p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = pick16(smp, t + q);
    int c[4];
    count4(list, R, cnt, p, c);
#pragma unroll
    for (int q = 3; q >= 0; --q)
      if (c[q] >= topk) {
        pivot = p[q];
        found = true;
      }
    t = t + 4 > 12 ? 12 : t + 4;
  }
  if (!found) return Compacted{cnt, tau, false};
  const int w = keep_pass(list, R, cnt, pivot);
  // both thresholds are exact; keep the higher
  return Compacted{w, fmaxf(tau, tau_of_bucket(pivot)), w < cnt};
}

// Exact bucket cut, for lists the sampled pivots cannot shrink: the highest
// bucket P that at least `topk` listed keys reach, found by narrowing
// [lowest bucket, highest bucket + 1) with four pivots per counting pass
// (the range shrinks five-fold per pass), then keep the keys of bucket >= P.
// What remains is k keys plus the other keys of bucket P; needs cnt >= topk.
__device__ __noinline__ Compacted compact_bucket_exact(const uint32_t* list_c, int R, int cnt, float tau, int topk) {
  uint32_t* list = const_cast<uint32_t*>(list_c);
  uint32_t lo = 0xffffu, hi = 0u;
  for (int s = 0; s < cnt; ++s) {
    const uint32_t b = ord_entry(list[s * RS + R]) >> 16;
    lo = min(lo, b);
    hi = max(hi, b);
  }
  hi += 1u;  // count(>= lo) = cnt >= topk, count(>= hi) = 0 < topk
  while (hi - lo > 1u) {
    const uint32_t span = hi - lo;
    uint32_t p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = (lo + (span * (uint32_t)(q + 1)) / 5u) << 16;
    int c[4];
    count4(list, R, cnt, p, c);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (c[q] >= topk)
        lo = max(lo, p[q] >> 16);
      else
        hi = min(hi, p[q] >> 16);
    }
  }
  const uint32_t pivot = lo << 16;
  const int w = keep_pass(list, R, cnt, pivot);
  return Compacted{w, fmaxf(tau, tau_of_bucket(pivot)), w < cnt};
}

// Append every key of a 32-key chunk whose score passes !(x <= tau) to the
// row's list.  Branch-free: each key's slot is the running count and the
// store is a predicated instruction, so lanes never diverge per key.
__device__ __forceinline__ void append_chunk(const uint32_t* v, int valid, float tau, uint32_t key0,
                                             uint32_t base, int& cnt) {
  uint32_t slot = (uint32_t)cnt;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t take = (uint32_t)(i < valid && !(__uint_as_float(v[i]) <= tau));
    st_shared_u32_if(base + slot * (4u * RS), __byte_perm(key0 + (uint32_t)i, v[i], 0x7610), take);
    slot += take;
  }
  cnt = (int)slot;
}

__device__ __forceinline__ float chunk_max(const uint32_t* v) {
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

// ------------------------------------------------------- exact re-scoring ---
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int h = 0; h < 8; ++h) f[h] = to_acc(e[h]);
}

// Exact fp32 score of the re-scoring stage: four FMA chains (feature f feeds
// chain f mod 4) summed pairwise.
__device__ __forceinline__ float dot64_regs(const float (&q)[D], const uint4 (&u)[8], bool bf16) {
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float f[8];
    if (bf16)
      unpack8<__nv_bfloat16>(u[c], f);
    else
      unpack8<__half>(u[c], f);
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h & 3] = fmaf(q[c * 8 + h], f[h], acc[h & 3]);
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

template <typename T>
__device__ __forceinline__ void load_row(const T* row, uint4 (&u)[8]) {
  const uint4* p = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int c = 0; c < 8; ++c) u[c] = __ldg(p + c);
}

// Warp re-selection works on one query row with the whole warp: lane
// 8*grp + g handles features 8g..8g+7 (16 bytes) of key grp of a group of
// four, so one 16-byte load instruction reads four whole 128-byte key or
// value rows.
template <typename T>
__device__ __forceinline__ void load_chunk8(const T* p, float (&f)[8]) {
  unpack8<T>(__ldg(reinterpret_cast<const uint4*>(p)), f);
}

// Exact fp32 score of the warp re-selection: each lane runs one FMA chain
// over its 8 features in order, then the 8 lanes of a group add their
// partial sums by xor-shuffles over 1, 2 and 4, so all 8 lanes hold the same
// sum.  (A row's scores all come from one of the two exact stages, so each
// row ranks its keys by one rounding of the dot product.)
template <typename T>
__device__ __forceinline__ float group_dot(const float (&qg)[8], const uint4& kc) {
  float f[8];
  unpack8<T>(kc, f);
  float acc = 0.f;
#pragma unroll
  for (int h = 0; h < 8; ++h) acc = fmaf(qg[h], f[h], acc);
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  return acc;
}

// Softmax-weighted sum of one query row's selected value rows, by the whole
// warp.  score_of(j) / index_of(j) give the raw score and key of selection j.
// Lane 8*grp + g accumulates features 8g..8g+7 of selections grp, grp+4, ...
// in that order; the four groups are added by xor-shuffles over 8 and 16 and
// lanes 0..7 store the 128-byte output row.  Also writes the row's indices
// (and scaled scores when asked) with consecutive lanes on consecutive
// entries.
template <typename T, typename ScoreOf, typename IndexOf>
__device__ __forceinline__ void write_row(const T* vbase, ScoreOf score_of, IndexOf index_of, int topk, float scale,
                                          float lse, T* orow, int32_t* idx_row, float* score_row, int lane) {
  for (int j = lane; j < topk; j += kWarp) {
    idx_row[j] = (int32_t)index_of(j);
    if (score_row) score_row[j] = score_of(j) * scale;
  }
  const int g = lane & 7, grp = lane >> 3;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int b0 = 0; b0 < topk; b0 += 8) {
    const int j0 = b0 + grp, j1 = b0 + 4 + grp;
    const bool v0 = j0 < topk, v1 = j1 < topk;
    float p0 = 0.f, p1 = 0.f;
    uint4 c0 = make_uint4(0u, 0u, 0u, 0u), c1 = c0;
    if (v0) {
      p0 = expf(score_of(j0) * scale - lse);
      c0 = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)index_of(j0) * D) + g);
    }
    if (v1) {
      p1 = expf(score_of(j1) * scale - lse);
      c1 = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)index_of(j1) * D) + g);
    }
    float f[8];
    unpack8<T>(c0, f);
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h] = fmaf(p0, f[h], acc[h]);
    unpack8<T>(c1, f);
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h] = fmaf(p1, f[h], acc[h]);
  }
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 8);
    acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 16);
  }
  if (lane < 8) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int h = 0; h < 8; ++h) e[h] = from_acc<T>(acc[h]);
    reinterpret_cast<uint4*>(orow)[g] = u;
  }
}

// Key index of re-scored candidate s of a row: `srow` points at the row's
// list column at slot FINAL_CAP; candidate s sits in slot FINAL_CAP + s/2,
// half s%2 of the word.
__device__ __forceinline__ uint32_t stage_byte(int s) { return (uint32_t)((s >> 1) * (4 * RS) + 2 * (s & 1)); }
__device__ __forceinline__ uint16_t& stage_at(uint16_t* srow, int s) {
  return *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(srow) + stage_byte(s));
}

// Exact cut on re-scored candidates (fp32 scores in cv, key indices in ci,
// both slot-major with stride RS).  Raise a pivot as compact_bucket does,
// with exact scores: keep the keys scoring at least the highest of 16
// sampled scores that >= topk candidates meet.
__device__ __noinline__ int compact_exact(float* cv, uint16_t* srow, int R, int cnt, int topk) {
  float smp[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float x = cv[((j * cnt) >> 4) * RS + R];
    smp[j] = (x != x) ? __int_as_float(0x7f800000) : x;
  }
  sort16_desc(smp);
  int t = (16 * topk) / (cnt > 0 ? cnt : 1);
  t = t > 12 ? 12 : t;
  float pivot = __int_as_float(0xff800000);
  bool found = false;
  for (int pass = 0; pass < 4 && !found; ++pass) {
    float p[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = pick16(smp, t + q);
    int c[4] = {0, 0, 0, 0};
#pragma unroll 4
    for (int s = 0; s < cnt; ++s) {
      const float x = cv[s * RS + R];
#pragma unroll
      for (int q = 0; q < 4; ++q) c[q] += !(x < p[q]);
    }
#pragma unroll
    for (int q = 3; q >= 0; --q)
      if (c[q] >= topk) {
        pivot = p[q];
        found = true;
      }
    t = t + 4 > 12 ? 12 : t + 4;
  }
  if (!found) return cnt;
  uint32_t w = 0;
  const uint32_t cvb = smem_addr(cv) + 4u * R, cib = smem_addr(srow);
  int s = 0;
  for (; s + 8 <= cnt; s += 8) {  // loads ahead of stores, as in keep_pass
    float x[8];
    uint32_t i[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = cv[(s + j) * RS + R];
      i[j] = stage_at(srow, s + j);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t keep = (uint32_t)!(x[j] < pivot);
      st_shared_f32_if(cvb + w * (4u * RS), x[j], keep);
      st_shared_u16_if(cib + stage_byte((int)w), i[j], keep);
      w += keep;
    }
  }
  for (; s < cnt; ++s) {
    const float x = cv[s * RS + R];
    const uint32_t i = stage_at(srow, s);
    const uint32_t keep = (uint32_t)!(x < pivot);
    st_shared_f32_if(cvb + w * (4u * RS), x, keep);
    st_shared_u16_if(cib + stage_byte((int)w), i, keep);
    w += keep;
  }
  return (int)w;
}

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

// Remove lowest-ranked keys until exactly `topk` remain.
__device__ __noinline__ int trim_exact(float* cv, uint16_t* srow, int R, int cnt, int topk) {
  while (cnt > topk) {
    uint64_t worst = ~0ull;
    int pos = 0;
#pragma unroll 4
    for (int s = 0; s < cnt; ++s) {
      const uint64_t key = rank_key(cv[s * RS + R], stage_at(srow, s));
      const bool lower = key < worst;
      worst = lower ? key : worst;
      pos = lower ? s : pos;
    }
    const int last = cnt - 1;
    cv[pos * RS + R] = cv[last * RS + R];
    stage_at(srow, pos) = stage_at(srow, last);
    cnt = last;
  }
  return cnt;
}

template <typename T>
__device__ __forceinline__ void store_out_row(const float (&acc)[D], T* orow_t) {
  uint4* orow = reinterpret_cast<uint4*>(orow_t);
#pragma unroll
  for (int q4 = 0; q4 < D / 8; ++q4) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int h = 0; h < 8; ++h) e[h] = from_acc<T>(acc[q4 * 8 + h]);
    orow[q4] = u;
  }
}

// Exact re-selection of one row by a whole warp (rows whose bucketed list
// could not be shrunk).  32 keys per step: eight group dots of four keys,
// then lane L takes the score of key k0 + L; a lane keeps each key beating
// the row's threshold in an exact list (fv/fi, FIX_CAP entries) that a warp
// bitonic sort cuts back to k when it could overflow.  ftau is one float.
struct RowOut {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int32_t* top_idx;
  float* lse;
  float* top_scores;
};

template <typename T>
__device__ __noinline__ void reselect_row(RowOut a, int64_t m, int topk, float scale, int64_t slice, int64_t gr,
                                          float* fv, int* fi, float* ftau, int lane) {
  const int g = lane & 7, grp = lane >> 3;
  float qg[8];
  load_chunk8<T>(static_cast<const T*>(a.q) + gr * D + 8 * g, qg);
  const T* kbase = static_cast<const T*>(a.k) + slice * m * D;
  if (lane == 0) *ftau = __int_as_float(0x7fc00000);
  __syncwarp();
  float tau = __int_as_float(0x7fc00000);
  int c0 = 0;
  for (int64_t k0 = 0; k0 < m; k0 += kWarp) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t kk = k0 + 4 * i + grp;
      uint4 kc = make_uint4(0u, 0u, 0u, 0u);
      if (kk < m) kc = __ldg(reinterpret_cast<const uint4*>(kbase + kk * D) + g);
      const float d = group_dot<T>(qg, kc);  // score of key k0 + 4i + grp
      const float x = __shfl_sync(0xffffffffu, d, 8 * (lane & 3));
      if ((lane >> 2) == i) s = x;
    }
    const int64_t key = k0 + lane;
    const bool valid = key < m;
    const bool pass = valid && !(s <= tau);
    const unsigned bal = __ballot_sync(0xffffffffu, pass);
    if (pass) {
      const int pos = c0 + __popc(bal & ((1u << lane) - 1u));
      fv[pos] = s;
      fi[pos] = (int)key;
    }
    c0 += __popc(bal);
    if (c0 > FIX_CAP - kWarp) {
      __syncwarp();
      c0 = compact_row(fv, fi, c0, topk, ftau, lane);
      tau = *ftau;
    }
  }
  __syncwarp();
  c0 = compact_row(fv, fi, c0, topk, ftau, lane);  // sorted, c0 == topk (topk <= m)
  const float mxs = fv[0] * scale;
  float part = 0.f;
  for (int j = lane; j < c0; j += kWarp) part += expf(fv[j] * scale - mxs);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  const float lse = mxs + logf(part);
  if (lane == 0) a.lse[gr] = lse;
  write_row<T>(static_cast<const T*>(a.v) + slice * m * D, [&](int j) { return fv[j]; }, [&](int j) { return fi[j]; },
               c0, scale, lse, static_cast<T*>(a.out) + gr * D, a.top_idx + gr * topk,
               a.top_scores ? a.top_scores + gr * topk : nullptr, lane);
  __syncwarp();
}

template <typename T>
__global__ void __launch_bounds__(NT, 1)
    fused_fwd_tc(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                 TcArgs a) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* qs = sm + OFF_Q;
  uint8_t* ks = sm + OFF_K;
  uint32_t* list = reinterpret_cast<uint32_t*>(sm + OFF_LIST);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 1 + KSTAGES;
  uint64_t* s_full = bars + 1 + 2 * KSTAGES;  // [tile][buffer]
  uint64_t* s_empty = s_full + 2 * NTILE;     // [tile][buffer]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t slice = blockIdx.x / a.tiles_per_slice;
  const int64_t local0 = (int64_t)(blockIdx.x % a.tiles_per_slice) * RS;
  const int64_t row0 = slice * a.n + local0;
  const int ntiles = (int)((a.m + TK - 1) / TK);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int b = 0; b < 2 * NTILE; ++b) {
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
      mbar_arrive_expect_tx(q_full, NTILE * TILE_BYTES);
      for (int g = 0; g < NTILE; ++g) tma_load_2d(qs + g * TILE_BYTES, &tmap_q, 0, (int)(row0 + g * TQ), q_full);
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
      const uint32_t idesc = instr_desc_f16(kBf16, TQ, TK);
      const uint32_t q_addr = smem_addr(qs);
      uint64_t* last_bar = nullptr;  // barrier of the last commit, for the abort path
      uint32_t last_ph = 0;
      if (mbar_wait(q_full, 0, abort_flag)) {
        for (int t = 0; t < ntiles; ++t) {
          const int s = t % KSTAGES, b = t & 1;
          const uint32_t ph_s = ((uint32_t)(t >> 1) & 1u);
          if (!mbar_wait(&k_full[s], (uint32_t)(t / KSTAGES) & 1u, abort_flag)) break;
          const uint32_t k_addr = smem_addr(ks + s * TILE_BYTES);
          bool stop = false;
#pragma unroll
          for (int g = 0; g < NTILE; ++g) {
            if (!mbar_wait(&s_empty[2 * g + b], ph_s ^ 1u, abort_flag)) {
              stop = true;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma_f16(tmem + (uint32_t)((2 * g + b) * TK), smem_desc_k128(q_addr + g * TILE_BYTES + kk * 32),
                      smem_desc_k128(k_addr + kk * 32), idesc, kk > 0);
            mma_commit(&s_full[2 * g + b]);
            last_bar = &s_full[2 * g + b];
            last_ph = ph_s;
          }
          if (stop) break;
          mma_commit(&k_empty[s]);
        }
      }
      if (*abort_flag && last_bar) {
        // wait for the last MMAs before TMEM is released
        const uint64_t t0 = global_timer();
        while (!mbar_try_wait(last_bar, last_ph) && global_timer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp >= 4) {
    const int wg = (warp - 4) >> 2, quarter = warp & 3;
    const int rl = quarter * kWarp + lane;  // row within the query tile == TMEM lane
    const int R = wg * TQ + rl;              // list column
    const int64_t tile_left = a.n - local0 - (int64_t)wg * TQ;
    const int rows = (int)(tile_left < 0 ? 0 : (tile_left < TQ ? tile_left : TQ));
    const uint32_t tm = tmem + ((uint32_t)(quarter * kWarp) << 16) + (uint32_t)(2 * wg * TK);
    uint64_t* my_full = s_full + 2 * wg;
    uint64_t* my_empty = s_empty + 2 * wg;
    const uint32_t lbase = smem_addr(list) + 4u * R;
    float tau = __int_as_float(0x7fc00000);  // "no threshold yet"
    int cnt = 0;
    bool dead = false;  // list could not be shrunk: exact re-selection at the end
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&my_full[b], (uint32_t)(t >> 1) & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int64_t key_tile = (int64_t)t * TK;
      const int tile_valid = (int)((a.m - key_tile) < TK ? (a.m - key_tile) : TK);
      // One 32-column chunk at a time; the TMEM load of the next chunk is in
      // flight while the current one is filtered.  The loop body holds two
      // chunk steps (two register buffers) so that the hot path stays small
      // enough for the instruction cache.  The TMEM buffer is released once
      // its last chunk is in registers.
      auto chunk_step = [&](uint32_t(&v)[32], int c) {
        const int valid = tile_valid - c * 32;
        float mx;
        if (valid >= 32) {
          mx = chunk_max(v);
        } else {
          mx = __int_as_float(0xff800000);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < valid) mx = max_nan(mx, __uint_as_float(v[i]));
        }
        if (!__any_sync(0xffffffffu, !(mx <= tau))) return;
        if (__any_sync(0xffffffffu, mx != mx)) {
          // one NaN pattern, ranked above every number
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = ((v[i] & 0x7fffffffu) > 0x7f800000u) ? 0x7fffffffu : v[i];
        }
        append_chunk(v, dead ? 0 : valid, tau, (uint32_t)(key_tile + c * 32), lbase, cnt);
        // When one lane's list could overflow, every lane holding well over
        // k keys compacts in the same pass: under SIMT the warp pays for the
        // longest list either way.
        if (__any_sync(0xffffffffu, !dead && cnt > CAP - 32)) {
          // The next chunk's TMEM load may still be writing its registers:
          // complete it before calling out of line.
          tmem_wait_load();
          if (!dead && cnt > a.topk + 16) {
            Compacted r = compact_bucket(list, R, cnt, tau, a.topk, 2);
            if (r.cnt > CAP - 32) r = compact_bucket_exact(list, R, r.cnt, r.tau, a.topk);
            cnt = r.cnt;
            tau = r.tau;
            dead = cnt > CAP - 32;
          }
        }
      };
      uint32_t va[32], vb[32];
      tmem_load_32cols(tm + b * TK, va);
      tmem_wait_load(va);
#pragma unroll 1
      for (int cp = 0; cp < TK / 64; ++cp) {
        const int c0 = 2 * cp;
        tmem_load_32cols(tm + b * TK + (c0 + 1) * 32, vb);
        chunk_step(va, c0);
        tmem_wait_load(vb);
        const bool last = cp == TK / 64 - 1;
        if (!last) {
          tmem_load_32cols(tm + b * TK + (c0 + 2) * 32, va);
        } else {
          tc_fence_before();
          mbar_arrive(&my_empty[b]);
        }
        chunk_step(vb, c0 + 1);
        if (!last) tmem_wait_load(va);
      }
    }
    // Shrink to the candidates that go to exact re-scoring.
    if (ok && !dead) {
      while (cnt > a.topk + 16) {
        const Compacted r = compact_bucket(list, R, cnt, tau, a.topk, 1);
        cnt = r.cnt;
        tau = r.tau;
        if (!r.shrank) break;
      }
      if (cnt > a.topk + 16) {
        const Compacted r = compact_bucket_exact(list, R, cnt, tau, a.topk);
        cnt = r.cnt;
        tau = r.tau;
      }
      dead = cnt > FINAL_CAP;
    }
    float q[D];
    if (ok) {
      const uint8_t* qrow = qs + wg * TILE_BYTES + rl * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 u = *reinterpret_cast<const uint4*>(qrow + ((c ^ (rl & 7)) << 4));
        unpack8<T>(u, &q[c * 8]);
      }
    }
    // Every MMA has completed (each selection warp saw its last tile) and no
    // copy is in flight: the Q/K buffers are free after this barrier.
    __syncwarp();
    named_bar_sync(1, NSEL);
    const bool live = __all_sync(0xffffffffu, ok && !*abort_flag);
    if (live) {
      uint16_t* srow = reinterpret_cast<uint16_t*>(list + FINAL_CAP * RS + R);
      float* lf = reinterpret_cast<float*>(list);
      const T* kbase = static_cast<const T*>(a.k) + slice * a.m * D;
      const int64_t gr = row0 + (int64_t)wg * TQ + rl;
      if (!dead) {
        int s = 0;
        for (; s + 1 < cnt; s += 2) {
          const uint32_t e0 = list[s * RS + R], e1 = list[(s + 1) * RS + R];
          uint4 u0[8], u1[8];
          load_row(kbase + (int64_t)(e0 & 0xffffu) * D, u0);
          load_row(kbase + (int64_t)(e1 & 0xffffu) * D, u1);
          stage_at(srow, s) = (uint16_t)(e0 & 0xffffu);
          stage_at(srow, s + 1) = (uint16_t)(e1 & 0xffffu);
          lf[s * RS + R] = dot64_regs(q, u0, kBf16);
          lf[(s + 1) * RS + R] = dot64_regs(q, u1, kBf16);
        }
        if (s < cnt) {
          const uint32_t e0 = list[s * RS + R];
          uint4 u0[8];
          load_row(kbase + (int64_t)(e0 & 0xffffu) * D, u0);
          stage_at(srow, s) = (uint16_t)(e0 & 0xffffu);
          lf[s * RS + R] = dot64_regs(q, u0, kBf16);
        }
        if (cnt > a.topk + 4) cnt = compact_exact(lf, srow, R, cnt, a.topk);
        cnt = trim_exact(lf, srow, R, cnt, a.topk);
        if (rl < rows) {
          float mx = lf[R];
          for (int j = 1; j < a.topk; ++j) mx = fmaxf(mx, lf[j * RS + R]);
          const float mxs = mx * a.scale;
          float total = 0.f;
          for (int j = 0; j < a.topk; ++j) total += expf(lf[j * RS + R] * a.scale - mxs);
          const float lse = mxs + logf(total);
          a.lse[gr] = lse;
          int32_t* idx_row = a.top_idx + gr * a.topk;
          for (int j = 0; j < a.topk; ++j) {
            idx_row[j] = stage_at(srow, j);
            if (a.top_scores) a.top_scores[gr * a.topk + j] = lf[j * RS + R] * a.scale;
          }
          float acc[D];
#pragma unroll
          for (int f = 0; f < D; ++f) acc[f] = 0.f;
          const T* vbase = static_cast<const T*>(a.v) + slice * a.m * D;
#pragma unroll 2
          for (int j = 0; j < a.topk; ++j) {
            const float p = expf(lf[j * RS + R] * a.scale - lse);
            const uint4* vrow = reinterpret_cast<const uint4*>(vbase + (int64_t)stage_at(srow, j) * D);
#pragma unroll
            for (int q4 = 0; q4 < D / 8; ++q4) {
              float f[8];
              unpack8<T>(__ldg(vrow + q4), f);
#pragma unroll
              for (int h = 0; h < 8; ++h) acc[q4 * 8 + h] = fmaf(p, f[h], acc[q4 * 8 + h]);
            }
          }
          store_out_row<T>(acc, static_cast<T*>(a.out) + gr * D);
        }
      }
      uint8_t* fix = sm + OFF_FIX + (warp - 4) * FIX_BYTES;
      unsigned pending = __ballot_sync(0xffffffffu, dead && rl < rows);
      while (pending) {
        const int l = __ffs(pending) - 1;
        pending &= pending - 1;
        reselect_row<T>(RowOut{a.q, a.k, a.v, a.out, a.top_idx, a.lse, a.top_scores}, a.m, a.topk, a.scale, slice,
                        row0 + (int64_t)wg * TQ + quarter * kWarp + l, reinterpret_cast<float*>(fix),
                        reinterpret_cast<int*>(fix + FIX_CAP * 4), reinterpret_cast<float*>(fix + FIX_CAP * 8),
                        lane);
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
  a.q = L.q;
  a.k = L.k;
  a.v = L.v;
  a.out = L.out;
  a.top_idx = L.top_idx;
  a.lse = static_cast<float*>(L.lse);
  a.top_scores = static_cast<float*>(L.top_scores);
  a.n = L.n;
  a.m = L.m;
  a.tiles_per_slice = (int)((L.n + RS - 1) / RS);
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
  if (L.row_offsets || L.row_index || L.seg_bias) return false;
  if (L.m > 65536 || L.topk > 64 || L.n < 1) return false;
  if (L.slices * L.n > 0x7fffff00 || L.slices * L.m > 0x7fffffff) return false;
  if (!aligned16(L.q) || !aligned16(L.k) || !aligned16(L.v) || !aligned16(L.out)) return false;
  return encode_fn() != nullptr;
}

int fwd_tensorcore(const FwdLaunch& L) {
  if (L.dtype == SDK_DTYPE_BF16) return launch<__nv_bfloat16>(L);
  if (L.dtype == SDK_DTYPE_F16) return launch<__half>(L);
  return SDK_ERR_UNSUPPORTED;
}

}  // namespace sdk
