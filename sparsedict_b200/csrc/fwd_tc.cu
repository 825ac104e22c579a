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
//   warps 2, 3   in the first CTA of each slice: the input magnitude check
//                of the slice's keys (below); idle elsewhere;
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
// After the last tile each selection thread writes its row's list (at most
// 176 entries, four per 16-byte store) and count to a candidate buffer in
// HBM, and the CTA ends: the SM is free for the next CTA's stream while the
// exact work runs elsewhere.  A second kernel, one warp per query row at high
// occupancy, finishes every row:
//
//   bucket cut   the k-th largest bucket of the row's entries, by 8-bit radix
//                digits over a shared histogram (from the highest bit in
//                which the row's buckets differ); entries of lower buckets
//                cannot be in the top k and are dropped;
//   re-score     each survivor's fp32 score is recomputed from the gathered
//                key row (eight lanes per 128-byte row, one fixed summation
//                order);
//   exact cut    the k best by order-preserving keys (score, then lower key
//                index on ties), by the same radix select;
//   epilogue     row LSE, the k indices (in list order; the set is the
//                reference's top-k set) and the softmax-weighted sum of the
//                gathered value rows.
//
// Marked rows are re-selected by their warp: lanes score 32 keys at a time
// with the same summation order and keep an exact candidate list sorted by a
// warp bitonic network, as the CUDA-core kernel does.
//
// Selection runs on the raw dot products; scale = 1/(T·sqrt(d)) > 0 is
// applied in the epilogue (for d = 64 and T a power of two the scale is a
// power of two, so the order is exactly that of the scaled scores).
#include <cuda.h>

#include <mutex>
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
constexpr int CAP = 160;        // list slots per row (and candidate buffer entries per row)
constexpr int FIX_CAP = 128;    // exact list of a row re-selected by one warp
constexpr int kDenseHits = 8;   // a chunk row with more hits makes the warp append branch-free
constexpr int NT = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TILE_BYTES = TK * D * 2;  // a K tile, also a Q tile

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + NTILE * (int)TILE_BYTES;
constexpr int OFF_LIST = OFF_K + KSTAGES * (int)TILE_BYTES;
constexpr int OFF_STAGE = OFF_LIST + CAP * RS * 4;  // per row: the current chunk's 32 buckets
constexpr int OFF_BAR = OFF_STAGE + RS * 64;
constexpr int NBARS = 1 + 2 * KSTAGES + 4 * NTILE;
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
static_assert(CAP % 4 == 0, "lists are written four entries per store");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");

// Count word of a row in the candidate buffer: the number of entries, or
constexpr int32_t kCandDead = -1;     // list could not be shrunk: re-select exactly
constexpr int32_t kCandAborted = -2;  // a pipeline wait timed out: nothing to finish

struct TcArgs {
  const void* q;     // query rows, gathered through row_index when that is set
  const void* k;     // key rows, for the magnitude check
  const int32_t* row_index;  // nullable: logical row -> query row (grouped slices)
  uint32_t* cand;    // [rows][CAP] list entries of each query row
  int32_t* cand_n;   // [rows] entry count, kCandDead or kCandAborted
  uint32_t* unsafe;  // [rows], at each slice's first row: 1 when a key of the slice fails the magnitude check
  SliceGeometry geo;
  int64_t m;
  int topk;
  uint32_t big16;    // 16-bit magnitude field at which an element counts as unsafe
  unsigned int* status;
  uint64_t wait_limit_ns;  // bound of each pipeline wait (sdk_set_wait_limit)
  // kBias: score(r, j) = dot * scale + seg_bias[r * segs + j / seg_len], with
  // seg_len a multiple of TK so that each key tile lies in one segment
  const float* seg_bias;
  int64_t seg_len;
  int segs;
  float scale;
};

// Input magnitude check.  With every |q|, |k| < 2^60 and finite, each of the
// 64 products is below 2^120 and their fp32 sum below 2^126, so no score can
// overflow to inf or become NaN; the stream filter then needs no NaN
// handling.  Rows whose inputs fail the check (a non-finite or huge element
// in the query row or anywhere in the slice's keys) are re-selected exactly
// by the finish kernel.  `big16` is the lowest 15-bit magnitude pattern that
// fails: 2^60 for bf16 (0x5d80), inf/NaN for fp16 (0x7c00, fp16 has no
// finite value that large).
__device__ __forceinline__ uint32_t big_halves(uint32_t w, uint32_t add) {
  // bit 15 / 31 set when that half's magnitude reaches big16 (add = 0x8000 -
  // big16 in both halves; the sum of a half stays below 0x10000)
  return ((w & 0x7fff7fffu) + add) & 0x80008000u;
}


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

// Threshold of the stream filter in bucket form, both halves of a bf16x2:
// the bucket of tau (the lowest score of the compaction pivot's bucket), or
// -inf before the first compaction.  A key passes when its bucket, compared
// as a bf16 number, reaches this one: every key with score > tau passes
// (truncation is monotonic), plus the other keys of tau's own bucket.
__device__ __forceinline__ uint32_t packed_threshold(float tau) {
  const uint32_t b = (tau != tau) ? 0xff80u : (__float_as_uint(tau) >> 16);
  return b * 0x00010001u;
}

// Hit mask of a 32-key chunk: bit i is set when key i's bucket reaches the
// packed threshold.  Word j of `p` receives the buckets of keys j (low half)
// and j + 16 (high half); one byte permute, one packed bf16 compare and one
// logic op cover two keys.
__device__ __forceinline__ uint32_t hit_mask(const uint32_t (&v)[32], uint32_t tb2, uint32_t (&p)[16]) {
  uint32_t m[4] = {0u, 0u, 0u, 0u};  // four independent chains, joined at the end
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    p[j] = __byte_perm(v[j], v[j + 16], 0x7632);
    uint32_t w;
    asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(w) : "r"(p[j]), "r"(tb2));
    m[j & 3] |= w & (0x00010001u << j);
  }
  return (m[0] | m[1]) | (m[2] | m[3]);
}

// Append the keys of mask `m` of a chunk to the row's list, branch-free: each
// key's slot is the running count and the store is a predicated instruction.
// Used when some row of the warp has many hits in the chunk (early in the
// stream, before the threshold has risen).
__device__ __forceinline__ void append_dense(const uint32_t (&v)[32], uint32_t m, uint32_t key0, uint32_t base,
                                             int& cnt) {
  uint32_t slot = (uint32_t)cnt;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t take = (m >> i) & 1u;
    st_shared_u32_if(base + slot * (4u * RS), __byte_perm(key0 + (uint32_t)i, v[i], 0x7610), take);
    slot += take;
  }
  cnt = (int)slot;
}

// Append the keys of mask `m` one hit at a time.  The chunk's packed buckets
// are first stored to the row's 64-byte stage (four 16-byte stores, chunk c
// at position c ^ sw so that eight lanes' stores cover all 32 banks); each
// hit then reads its bucket back by its bit position.  A lane loops only over
// its own hits, so a warp pays for its row with the most hits, usually two
// or three per chunk.
__device__ __forceinline__ void append_sparse(const uint32_t (&p)[16], uint32_t m, uint32_t key0, uint32_t stage,
                                              uint32_t sw, uint32_t base, int& cnt) {
  if (m == 0u) return;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(stage + ((16u * c) ^ sw)), "r"(p[4 * c]),
                 "r"(p[4 * c + 1]), "r"(p[4 * c + 2]), "r"(p[4 * c + 3])
                 : "memory");
  // two hits per iteration (most lanes have at most two): both bucket reads
  // are in flight together
  uint32_t slot = (uint32_t)cnt;
  do {
    const uint32_t b0 = 31u - __clz(m);
    m ^= 1u << b0;
    const uint32_t two = m != 0u;
    const uint32_t b1 = two ? 31u - __clz(m) : b0;
    m &= ~(two << b1);
    uint32_t k0b, k1b;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(k0b) : "r"(stage + ((((b0 << 2) & 60u) ^ sw) | ((b0 >> 3) & 2u))) : "memory");
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(k1b) : "r"(stage + ((((b1 << 2) & 60u) ^ sw) | ((b1 >> 3) & 2u))) : "memory");
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(base + slot * (4u * RS)), "r"(__byte_perm(key0 + b0, k0b, 0x5410))
                 : "memory");
    st_shared_u32_if(base + (slot + 1u) * (4u * RS), __byte_perm(key0 + b1, k1b, 0x5410), two);
    slot += 1u + two;
  } while (m != 0u);
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

// Exact-score stages work on one query row with the whole warp: lane
// 8*grp + g handles features 8g..8g+7 (16 bytes) of key grp of a group of
// four, so one 16-byte load instruction reads four whole 128-byte key or
// value rows.
//
// dot8: one fp32 FMA chain over 8 features in order, both operands 16-bit.
// The mixed-precision FMA widens them exactly and the product of two 16-bit
// floats is exact in fp32, so each step equals fmaf of the widened values.
template <typename T>
__device__ __forceinline__ float dot8(const uint4& a, const uint4& b) {
  float acc = 0.f;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("{\n .reg .b16 a0, a1, a2, a3, a4, a5, a6, a7, b0, b1, b2, b3, b4, b5, b6, b7;\n"
        " mov.b32 {a0, a1}, %1;\n mov.b32 {a2, a3}, %2;\n mov.b32 {a4, a5}, %3;\n mov.b32 {a6, a7}, %4;\n"
        " mov.b32 {b0, b1}, %5;\n mov.b32 {b2, b3}, %6;\n mov.b32 {b4, b5}, %7;\n mov.b32 {b6, b7}, %8;\n"
        " fma.rn.f32.bf16 %0, a0, b0, %0;\n fma.rn.f32.bf16 %0, a1, b1, %0;\n"
        " fma.rn.f32.bf16 %0, a2, b2, %0;\n fma.rn.f32.bf16 %0, a3, b3, %0;\n"
        " fma.rn.f32.bf16 %0, a4, b4, %0;\n fma.rn.f32.bf16 %0, a5, b5, %0;\n"
        " fma.rn.f32.bf16 %0, a6, b6, %0;\n fma.rn.f32.bf16 %0, a7, b7, %0;\n}"
        : "+f"(acc)
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w));
  } else {
    asm("{\n .reg .b16 a0, a1, a2, a3, a4, a5, a6, a7, b0, b1, b2, b3, b4, b5, b6, b7;\n"
        " mov.b32 {a0, a1}, %1;\n mov.b32 {a2, a3}, %2;\n mov.b32 {a4, a5}, %3;\n mov.b32 {a6, a7}, %4;\n"
        " mov.b32 {b0, b1}, %5;\n mov.b32 {b2, b3}, %6;\n mov.b32 {b4, b5}, %7;\n mov.b32 {b6, b7}, %8;\n"
        " fma.rn.f32.f16 %0, a0, b0, %0;\n fma.rn.f32.f16 %0, a1, b1, %0;\n"
        " fma.rn.f32.f16 %0, a2, b2, %0;\n fma.rn.f32.f16 %0, a3, b3, %0;\n"
        " fma.rn.f32.f16 %0, a4, b4, %0;\n fma.rn.f32.f16 %0, a5, b5, %0;\n"
        " fma.rn.f32.f16 %0, a6, b6, %0;\n fma.rn.f32.f16 %0, a7, b7, %0;\n}"
        : "+f"(acc)
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w));
  }
  return acc;
}

// Exact fp32 score: dot8 over the lane's 8 features, then the 8 lanes of a
// group add their partial sums by xor-shuffles over 1, 2 and 4, so all 8
// lanes hold the same sum.  Every exact score (finish kernel and warp
// re-selection) is this one rounding of the dot product.
template <typename T>
__device__ __forceinline__ float group_dot(const uint4& qg, const uint4& kc) {
  float acc = dot8<T>(qg, kc);
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

__device__ __forceinline__ float finite_or_zero(float x) { return isfinite(x) ? x : 0.f; }

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
__device__ __noinline__ void reselect_row(RowOut a, int64_t m, int topk, float scale, int64_t slice, int64_t gr, int64_t pr,
                                          const float* bias_row, int64_t seg_len, float* fv, int* fi, float* ftau,
                                          int lane) {
  const int g = lane & 7, grp = lane >> 3;
  const uint4 qg = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) + pr * D) + g);
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
    // biased: the final score, scaled then shifted by the key's segment bias
    if (bias_row && valid) s = __fadd_rn(__fmul_rn(s, scale), bias_row[key / seg_len]);
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
  if (bias_row) scale = 1.f;  // the list already holds final scores
  // softmax shift: the row maximum, or 0 when it is not finite (all scores
  // -inf gives LSE -inf; a NaN or +inf maximum gives NaN / +inf)
  const float mxs = finite_or_zero(fv[0] * scale);
  float part = 0.f;
  for (int j = lane; j < c0; j += kWarp) part += expf(fv[j] * scale - mxs);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  const float lse = mxs + logf(part);
  if (lane == 0) a.lse[gr] = lse;
  write_row<T>(static_cast<const T*>(a.v) + slice * m * D, [&](int j) { return fv[j]; }, [&](int j) { return fi[j]; },
               c0, scale, lse, static_cast<T*>(a.out) + pr * D, a.top_idx + gr * topk,
               a.top_scores ? a.top_scores + gr * topk : nullptr, lane);
  __syncwarp();
}

// kPrefilter: skip 32-key chunks in which no row of the warp has a hit.
// That pays only for small k: with k >= 8, some row of the warp has a hit in
// nearly every chunk and the test is pure overhead.
// kBias: each row's scores of a key tile are shifted by the bias of the
// tile's segment, fma(dot, scale, bias), before the filter (the finish kernel
// recomputes the exact fl(fl(dot * scale) + bias)).
template <typename T, bool kPrefilter, bool kBias>
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
  volatile uint32_t* scan_big = reinterpret_cast<volatile uint32_t*>(sm + OFF_MISC + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t slice, row0;
  int count;  // rows of this CTA (RS, fewer at a slice's end, 0 for a surplus grouped CTA)
  locate_tile(a.geo, blockIdx.x, RS, &slice, &row0, &count);
  if (count <= 0) return;
  const int64_t slice_row0 = slice_row_begin(a.geo, slice);
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
      if (!a.row_index) {  // else warps 2 and 3 gather the query rows
        mbar_arrive_expect_tx(q_full, NTILE * TILE_BYTES);
        for (int g = 0; g < NTILE; ++g) tma_load_2d(qs + g * TILE_BYTES, &tmap_q, 0, (int)(row0 + g * TQ), q_full);
      }
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % KSTAGES;
        const uint32_t ph = (uint32_t)(t / KSTAGES) & 1u;
        if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag, a.wait_limit_ns)) break;
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
  } else if (warp == 2 || warp == 3) {
    if (a.row_index) {
      // Grouped rows read through the permutation: the two warps gather the
      // CTA's query rows into the layout the TMA would have written (128-byte
      // rows, 16-byte chunk c of row r at chunk c ^ (r & 7)); rows past the
      // CTA's count are zero.  The copies are made visible to the tensor
      // cores' async proxy before q_full is signalled.
      const int t = (int)threadIdx.x - 2 * kWarp;
      const T* qrows = static_cast<const T*>(a.q);
      const uint32_t qbase = smem_addr(qs);
      for (int c = t; c < RS * (D / 8); c += 2 * kWarp) {
        const int r = c >> 3, ch = c & 7;
        const uint32_t dst = qbase + (uint32_t)(r / TQ) * TILE_BYTES + (uint32_t)(r % TQ) * (D * 2) +
                             ((uint32_t)(ch ^ (r & 7)) << 4);
        if (r < count)
          cp_async_16(dst, qrows + (int64_t)a.row_index[row0 + r] * D + ch * 8);
        else
          st_shared_zero16(dst);
      }
      cp_async_wait_all();
      fence_proxy_async_shared();
      named_bar_sync(1, 2 * kWarp);
      if (t == 0) mbar_arrive(q_full);
    }
    // The first CTA of each slice also checks the slice's keys for unsafe
    // magnitudes, with its two otherwise idle warps reading the key rows
    // from global memory (L2: the slice's CTAs are streaming them).
    if (row0 == slice_row0) {
      const uint4* kp = reinterpret_cast<const uint4*>(static_cast<const T*>(a.k) + slice * a.m * D);
      const int64_t total = a.m * (D / 8);
      const uint32_t add = (0x8000u - a.big16) * 0x00010001u;
      uint32_t big = 0;
      const int64_t step = 2 * kWarp;
      int64_t i = (int64_t)(warp - 2) * kWarp + lane;
      for (; i + 15 * step < total; i += 16 * step) {
        uint4 u[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) u[j] = __ldg(kp + i + j * step);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          big |= big_halves(u[j].x, add) | big_halves(u[j].y, add) | big_halves(u[j].z, add) | big_halves(u[j].w, add);
      }
      for (; i < total; i += step) {
        const uint4 u = __ldg(kp + i);
        big |= big_halves(u.x, add) | big_halves(u.y, add) | big_halves(u.z, add) | big_halves(u.w, add);
      }
      const bool any_big = __any_sync(0xffffffffu, big != 0u);
      if (warp == 3 && lane == 0) *scan_big = any_big ? 1u : 0u;
      named_bar_sync(1, 2 * kWarp);
      if (warp == 2 && lane == 0) a.unsafe[slice_row0] = (any_big || *scan_big) ? 1u : 0u;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc_f16(kBf16, TQ, TK);
      const uint32_t q_addr = smem_addr(qs);
      uint64_t* last_bar = nullptr;  // barrier of the last commit, for the abort path
      uint32_t last_ph = 0;
      if (mbar_wait(q_full, 0, abort_flag, a.wait_limit_ns)) {
        for (int t = 0; t < ntiles; ++t) {
          const int s = t % KSTAGES, b = t & 1;
          const uint32_t ph_s = ((uint32_t)(t >> 1) & 1u);
          if (!mbar_wait(&k_full[s], (uint32_t)(t / KSTAGES) & 1u, abort_flag, a.wait_limit_ns)) break;
          const uint32_t k_addr = smem_addr(ks + s * TILE_BYTES);
          bool stop = false;
#pragma unroll
          for (int g = 0; g < NTILE; ++g) {
            if (!mbar_wait(&s_empty[2 * g + b], ph_s ^ 1u, abort_flag, a.wait_limit_ns)) {
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
    const int tile_left = count - wg * TQ;
    const int rows = tile_left < 0 ? 0 : (tile_left < TQ ? tile_left : TQ);
    const uint32_t tm = tmem + ((uint32_t)(quarter * kWarp) << 16) + (uint32_t)(2 * wg * TK);
    uint64_t* my_full = s_full + 2 * wg;
    uint64_t* my_empty = s_empty + 2 * wg;
    const uint32_t lbase = smem_addr(list) + 4u * R;
    const uint32_t sbase = smem_addr(sm + OFF_STAGE) + 64u * R;
    const uint32_t sw = ((uint32_t)(R >> 1) & 3u) << 4;
    float tau = __int_as_float(0x7fc00000);  // "no threshold yet"
    uint32_t tb2 = packed_threshold(tau);
    int cnt = 0;
    bool dead = false;  // list could not be shrunk: exact re-selection at the end
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&my_full[b], (uint32_t)(t >> 1) & 1u, abort_flag, a.wait_limit_ns));
      if (!ok) break;
      tc_fence_after();
      const int64_t key_tile = (int64_t)t * TK;
      const int tile_valid = (int)((a.m - key_tile) < TK ? (a.m - key_tile) : TK);
      float tile_bias = 0.f;
      if (kBias && rl < rows)
        tile_bias = __ldg(a.seg_bias + (row0 + wg * TQ + rl) * a.segs + key_tile / a.seg_len);
      // One 32-column chunk at a time; the TMEM load of the next chunk is in
      // flight while the current one is filtered.  The loop body holds two
      // chunk steps (two register buffers) so that the hot path stays small
      // enough for the instruction cache.  The TMEM buffer is released once
      // its last chunk is in registers.
      auto chunk_step = [&](uint32_t(&v)[32], int c) {
        const int valid = tile_valid - c * 32;
        if (kBias) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(fmaf(__uint_as_float(v[i]), a.scale, tile_bias));
        }
        if (kPrefilter) {
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
        }
        uint32_t p[16];
        uint32_t m = hit_mask(v, tb2, p);
        if (dead) m = 0u;
        if (valid < 32) m &= valid > 0 ? (1u << valid) - 1u : 0u;
        const uint32_t key0 = (uint32_t)(key_tile + c * 32);
        if (__any_sync(0xffffffffu, __popc(m) > kDenseHits))
          append_dense(v, m, key0, lbase, cnt);
        else
          append_sparse(p, m, key0, sbase, sw, lbase, cnt);
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
            tb2 = packed_threshold(tau);
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
    // Hand the row to the finish kernel: its entry count (or kCandDead) and
    // the entries, four per 16-byte store (slots past the count are unused).
    if (rl < rows) {
      const int64_t gr = row0 + (int64_t)wg * TQ + rl;
      if (!ok) {
        a.cand_n[gr] = kCandAborted;
      } else if (dead) {
        a.cand_n[gr] = kCandDead;
      } else {
        uint4* dst = reinterpret_cast<uint4*>(a.cand + gr * CAP);
        for (int s = 0; s < cnt; s += 4)
          dst[s >> 2] = make_uint4(list[s * RS + R], list[(s + 1) * RS + R], list[(s + 2) * RS + R],
                                   list[(s + 3) * RS + R]);
        a.cand_n[gr] = cnt;
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

// ------------------------------------------------------------ finish ---
// One warp per query row (see the file comment).  Each warp keeps its row's
// survivors (key, exact score) and a 256-bin histogram in shared memory; the
// exact re-selection of marked rows reuses the survivor arrays.
constexpr int FW = 8;                      // warps per finish block
constexpr int NV = (CAP + kWarp - 1) / kWarp;  // list entries per lane
constexpr int FUNR = 4;                    // survivors in flight per lane group

struct FinArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int32_t* top_idx;
  float* lse;
  float* top_scores;
  const uint32_t* cand;
  const int32_t* cand_n;
  const uint32_t* unsafe;  // at each slice's first row, from the stream kernel's key check
  const int32_t* row_index;  // nullable: logical row -> query/output row
  const float* seg_bias;     // nullable: per (logical row, key segment), as in TcArgs
  int64_t seg_len;
  int segs;
  SliceGeometry geo;
  int64_t rows, m;
  int topk;
  float scale;
  uint32_t big16;
};

struct __align__(16) FinWarp {
  float sc[CAP];  // survivors' exact scores, then the selection's
  int si[CAP];    // their key indices
  int hist[256];
};
static_assert(sizeof(float) * CAP + sizeof(int) * CAP >= FIX_CAP * 8 + 16, "re-selection buffers exceed sc/si");

// The need-th largest (1 <= need <= count) of the warp's values whose `ok`
// is set, by 8-bit digits starting at the highest bit in which those values
// differ, one 256-bin shared-memory histogram per digit.  Only the first
// `nv` slots of each lane (warp-uniform) may be set.  *above receives how
// many values are strictly larger.
__device__ __forceinline__ uint32_t warp_kth_largest(const uint32_t (&v)[NV], const bool (&ok)[NV], int nv,
                                                     int need, int* hist, int lane, int* above) {
  uint32_t lo = 0xffffffffu, hi = 0u;
#pragma unroll
  for (int i = 0; i < NV; ++i)
    if (i < nv && ok[i]) {
      lo = min(lo, v[i]);
      hi = max(hi, v[i]);
    }
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  int gt = 0;
  uint32_t prefix = lo;
  if (hi != lo) {
    const int top = 31 - __clz(hi ^ lo);
    prefix = lo & ~(uint32_t)((2ull << top) - 1ull);  // the bits above `top`, common to all
    for (int lowbit = top - 7;; lowbit -= 8) {
      const int sh = lowbit < 0 ? 0 : lowbit;
      const uint32_t dmask = (1u << (lowbit + 8 - sh)) - 1u;
      reinterpret_cast<int4*>(hist)[2 * lane] = make_int4(0, 0, 0, 0);
      reinterpret_cast<int4*>(hist)[2 * lane + 1] = make_int4(0, 0, 0, 0);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < NV; ++i)
        if (i < nv && ok[i] && ((uint64_t)(v[i] ^ prefix) >> (lowbit + 8)) == 0)
          atomicAdd(&hist[(v[i] >> sh) & dmask], 1);
      __syncwarp();
      // lane L holds bins 255-8L down to 248-8L
      const int4 h0 = reinterpret_cast<const int4*>(hist)[62 - 2 * lane];
      const int4 h1 = reinterpret_cast<const int4*>(hist)[63 - 2 * lane];
      const int c[8] = {h1.w, h1.z, h1.y, h1.x, h0.w, h0.z, h0.y, h0.x};
      int tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) tot += c[i];
      int incl = tot;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int excl = incl - tot;
      const int src = __ffs(__ballot_sync(0xffffffffu, excl < need && need <= incl)) - 1;
      int dig = -1, before = 0, run = excl;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (dig < 0 && run + c[i] >= need) {
          dig = 255 - 8 * lane - i;
          before = run;
        }
        run += c[i];
      }
      dig = __shfl_sync(0xffffffffu, dig, src);
      before = __shfl_sync(0xffffffffu, before, src);
      prefix |= (uint32_t)dig << sh;
      need -= before;
      gt += before;
      __syncwarp();
      if (lowbit <= 0) break;
    }
  }
  *above = gt;
  return prefix;
}

template <typename T>
__global__ void __launch_bounds__(FW * kWarp, 4) fwd_tc_finish(FinArgs a) {
  __shared__ FinWarp sw[FW];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane & 7, grp = lane >> 3;
  const unsigned lt = (1u << lane) - 1u;
  FinWarp& w = sw[warp];
  for (int64_t r = (int64_t)blockIdx.x * FW + warp; r < a.rows; r += (int64_t)gridDim.x * FW) {
    const int cnt = a.cand_n[r];
    if (cnt == kCandAborted) {
      // the stream kernel gave up on this row (a bounded wait ran out, device
      // status bit 2): defined outputs that no caller can mistake for a
      // result — NaN output and LSE, index -1 (the backward skips it)
      for (int j = lane; j < a.topk; j += kWarp) {
        a.top_idx[r * a.topk + j] = -1;
        if (a.top_scores) a.top_scores[r * a.topk + j] = __int_as_float(0x7fc00000);
      }
      const int64_t orow = a.row_index ? (int64_t)a.row_index[r] : r;
      if (lane < D) static_cast<T*>(a.out)[orow * D + lane] = from_acc<T>(__int_as_float(0x7fc00000));
      if (lane + kWarp < D) static_cast<T*>(a.out)[orow * D + lane + kWarp] = from_acc<T>(__int_as_float(0x7fc00000));
      if (lane == 0) a.lse[r] = __int_as_float(0x7fc00000);
      continue;
    }
    const int64_t slice = slice_of_row(a.geo, r);
    const int64_t pr = a.row_index ? (int64_t)a.row_index[r] : r;  // query and output row
    const uint4 qg = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) + pr * D) + g);
    const uint32_t add = (0x8000u - a.big16) * 0x00010001u;
    const bool unsafe = __any_sync(0xffffffffu, (big_halves(qg.x, add) | big_halves(qg.y, add) |
                                                 big_halves(qg.z, add) | big_halves(qg.w, add)) != 0u) ||
                        a.unsafe[slice_row_begin(a.geo, slice)] != 0u;
    const float* brow = a.seg_bias ? a.seg_bias + r * a.segs : nullptr;
    bool bias_nan = false;  // a NaN bias makes NaN scores, which the stream filter does not rank
    if (brow)
      for (int j = lane; j < a.segs; j += kWarp) bias_nan |= brow[j] != brow[j];
    if (cnt < 0 || unsafe || __any_sync(0xffffffffu, bias_nan)) {
      uint8_t* fix = reinterpret_cast<uint8_t*>(&w);
      reselect_row<T>(RowOut{a.q, a.k, a.v, a.out, a.top_idx, a.lse, a.top_scores}, a.m, a.topk, a.scale, slice, r, pr,
                      brow, a.seg_len,
                      reinterpret_cast<float*>(fix), reinterpret_cast<int*>(fix + FIX_CAP * 4),
                      reinterpret_cast<float*>(fix + FIX_CAP * 8), lane);
      continue;
    }
    // bucket cut: keep the entries whose bucket reaches the k-th largest
    const int nv = (cnt + kWarp - 1) / kWarp;
    uint32_t e[NV], o[NV];
    bool ok[NV];
    const uint32_t* crow = a.cand + r * CAP;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int s = lane + kWarp * i;
      ok[i] = false;
      e[i] = 0u;
      if (i < nv) {
        ok[i] = s < cnt;
        e[i] = ok[i] ? crow[s] : 0u;
      }
      o[i] = ord_entry(e[i]) >> 16;
    }
    int above = 0;
    const uint32_t tb = cnt > a.topk ? warp_kth_largest(o, ok, nv, a.topk, w.hist, lane, &above) : 0u;
    int S = 0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i < nv) {
        const bool keep = ok[i] && o[i] >= tb;
        const unsigned b = __ballot_sync(0xffffffffu, keep);
        if (keep) w.si[S + __popc(b & lt)] = (int)(e[i] & 0xffffu);
        S += __popc(b);
      }
    }
    __syncwarp();
    // exact scores: group grp re-scores survivors grp, grp + 4, ...
    const T* kbase = static_cast<const T*>(a.k) + slice * a.m * D;
    for (int s0 = 0; s0 < S; s0 += 4 * FUNR) {
      uint4 kc[FUNR];
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        const int s = s0 + 4 * u + grp;
        kc[u] = make_uint4(0u, 0u, 0u, 0u);
        if (s < S) kc[u] = __ldg(reinterpret_cast<const uint4*>(kbase + (int64_t)w.si[s] * D) + g);
      }
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        const int s = s0 + 4 * u + grp;
        const float d = group_dot<T>(qg, kc[u]);
        if (g == 0 && s < S)
          w.sc[s] = brow ? __fadd_rn(__fmul_rn(d, a.scale), brow[w.si[s] / a.seg_len]) : d;
      }
    }
    __syncwarp();
    // exact cut to k: larger score first, lower key index on equal scores
    int sel = S;
    if (S > a.topk) {
      const int sv = (S + kWarp - 1) / kWarp;
      bool hk[NV];
      float xs[NV];
      int ks[NV];
      uint64_t rk[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int s = lane + kWarp * i;
        hk[i] = i < sv && s < S;
        xs[i] = hk[i] ? w.sc[s] : 0.f;
        ks[i] = hk[i] ? w.si[s] : 0;
        rk[i] = hk[i] ? rank_key(xs[i], (uint32_t)ks[i]) : ~0ull;
      }
      if (S - a.topk <= 8) {
        // few extra: drop the lowest-ranked one at a time (rank keys are
        // distinct, so each round removes exactly one)
        for (int d = S - a.topk; d > 0; --d) {
          uint64_t mn = ~0ull;
#pragma unroll
          for (int i = 0; i < NV; ++i)
            if (i < sv) mn = rk[i] < mn ? rk[i] : mn;
          const uint32_t mh = __reduce_min_sync(0xffffffffu, (uint32_t)(mn >> 32));
          const uint32_t ml = __reduce_min_sync(0xffffffffu, (uint32_t)(mn >> 32) == mh ? (uint32_t)mn : 0xffffffffu);
          const uint64_t low = ((uint64_t)mh << 32) | ml;
#pragma unroll
          for (int i = 0; i < NV; ++i)
            if (i < sv && rk[i] == low) {
              rk[i] = ~0ull;
              hk[i] = false;
            }
        }
      } else {
        uint32_t hv[NV], lv[NV];
        bool lk[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) hv[i] = (uint32_t)(rk[i] >> 32);
        int gt = 0;
        const uint32_t ts = warp_kth_largest(hv, hk, sv, a.topk, w.hist, lane, &gt);
        const int need = a.topk - gt;
        int eq = 0;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          lk[i] = hk[i] && hv[i] == ts;
          lv[i] = (uint32_t)rk[i];
          if (i < sv) eq += __popc(__ballot_sync(0xffffffffu, lk[i]));
        }
        uint32_t tl = 0u;  // the kept ties are those whose low word reaches tl
        if (eq > need) {
          int unused = 0;
          tl = warp_kth_largest(lv, lk, sv, need, w.hist, lane, &unused);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) hk[i] = hk[i] && (hv[i] > ts || (lk[i] && lv[i] >= tl));
      }
      __syncwarp();
      int pos = 0;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if (i < sv) {
          const unsigned b = __ballot_sync(0xffffffffu, hk[i]);
          if (hk[i]) {
            const int p = pos + __popc(b & lt);
            w.sc[p] = xs[i];
            w.si[p] = ks[i];
          }
          pos += __popc(b);
        }
      }
      __syncwarp();
      sel = pos;
    }
    // LSE; lane j holds selections j and j + 32 (k <= 64).  Biased scores are final.
    const float sc_mul = brow ? 1.f : a.scale;
    const bool v0 = lane < sel, v1 = lane + kWarp < sel;
    const float x0 = v0 ? w.sc[lane] : 0.f, x1 = v1 ? w.sc[lane + kWarp] : 0.f;
    const int k0 = v0 ? w.si[lane] : 0, k1 = v1 ? w.si[lane + kWarp] : 0;
    float mx = fmaxf(v0 ? x0 : __int_as_float(0xff800000), v1 ? x1 : __int_as_float(0xff800000));
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
    const float mxs = finite_or_zero(mx * sc_mul);
    float part = (v0 ? expf(x0 * sc_mul - mxs) : 0.f) + (v1 ? expf(x1 * sc_mul - mxs) : 0.f);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o2);
    const float lse = mxs + logf(part);
    if (lane == 0) a.lse[r] = lse;
    float* pw = reinterpret_cast<float*>(w.hist);  // softmax weight of each selection
    int32_t* idx_row = a.top_idx + r * a.topk;
    if (v0) {
      pw[lane] = expf(x0 * sc_mul - lse);
      idx_row[lane] = k0;
      if (a.top_scores) a.top_scores[r * a.topk + lane] = x0 * sc_mul;
    }
    if (v1) {
      pw[lane + kWarp] = expf(x1 * sc_mul - lse);
      idx_row[lane + kWarp] = k1;
      if (a.top_scores) a.top_scores[r * a.topk + lane + kWarp] = x1 * sc_mul;
    }
    __syncwarp();
    // softmax-weighted sum of the value rows: group grp takes selections
    // grp, grp + 4, ... in order; the groups are added by xor-shuffles
    const T* vbase = static_cast<const T*>(a.v) + slice * a.m * D;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < sel; j0 += 4 * FUNR) {
      uint4 vc[FUNR];
      float pj[FUNR];
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        const int j = j0 + 4 * u + grp;
        vc[u] = make_uint4(0u, 0u, 0u, 0u);
        pj[u] = 0.f;
        if (j < sel) {
          pj[u] = pw[j];
          vc[u] = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)w.si[j] * D) + g);
        }
      }
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        float f[8];
        unpack8<T>(vc[u], f);
#pragma unroll
        for (int h = 0; h < 8; ++h) acc[h] = fmaf(pj[u], f[h], acc[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 8);
      acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 16);
    }
    if (lane < 8) {
      uint4 u;
      T* ev = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int h = 0; h < 8; ++h) ev[h] = from_acc<T>(acc[h]);
      reinterpret_cast<uint4*>(static_cast<T*>(a.out) + pr * D)[g] = u;
    }
    __syncwarp();
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
int launch(const FwdLaunch& L) {
  CUtensorMap tq, tk;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const bool grouped = L.row_offsets != nullptr;
  // grouped: n is the total row count, slice s owns rows [row_offsets[s], row_offsets[s+1])
  const int64_t rows = grouped ? L.n : L.slices * L.n;
  if (rows <= 0) return SDK_OK;
  if (!make_rows_map(&tq, L.q, rows, bf16)) return SDK_ERR_CUDA;
  if (!make_rows_map(&tk, L.k, L.slices * L.m, bf16)) return SDK_ERR_CUDA;
  TcArgs a;
  a.q = L.q;
  a.k = L.k;
  a.row_index = L.row_index;
  a.geo = SliceGeometry{L.row_offsets, L.slices, L.n};
  a.m = L.m;
  a.topk = L.topk;
  a.status = L.status;
  a.wait_limit_ns = wait_limit_ns();
  a.seg_bias = static_cast<const float*>(L.seg_bias);
  a.seg_len = L.seg_len;
  a.segs = L.segs;
  a.scale = (float)L.scale;
  // grouped: at most ceil(rows / RS) + slices tiles; CTAs past the last exit at once
  const int64_t grid = grouped ? (rows + RS - 1) / RS + L.slices : L.slices * ((L.n + RS - 1) / RS);
  if (grid <= 0) return SDK_OK;
  if (grid > 0x7fffffff) return SDK_ERR_UNSUPPORTED;
  const bool bias = L.seg_bias != nullptr;
  auto kern = L.topk < 8 ? (bias ? fused_fwd_tc<T, true, true> : fused_fwd_tc<T, true, false>)
                         : (bias ? fused_fwd_tc<T, false, true> : fused_fwd_tc<T, false, false>);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
    return SDK_ERR_CUDA;
  const size_t need = (size_t)rows * (CAP * 4 + 8);
  void* ws = L.workspace;
  const bool pooled = ws == nullptr;
  if (pooled) {
    cudaMemPool_t pool = scratch_pool();
    if (!pool) return SDK_ERR_CUDA;
    if (cudaMallocFromPoolAsync(&ws, need, pool, L.stream) != cudaSuccess) return SDK_ERR_CUDA;
  } else if (L.workspace_bytes < need || !aligned16(ws)) {
    return SDK_ERR_INVALID_ARGUMENT;
  }
  // per row: CAP entries, a count and a flag (set at the first row of each slice)
  a.cand = static_cast<uint32_t*>(ws);
  a.cand_n = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + (size_t)rows * CAP * 4);
  a.unsafe = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + (size_t)rows * (CAP * 4 + 4));
  a.big16 = bf16 ? 0x5d80u : 0x7c00u;
  kern<<<(unsigned)grid, NT, SMEM_BYTES, L.stream>>>(tq, tk, a);
  int rc = cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
  if (rc == SDK_OK) {
    FinArgs f;
    f.q = L.q;
    f.k = L.k;
    f.v = L.v;
    f.out = L.out;
    f.top_idx = L.top_idx;
    f.lse = static_cast<float*>(L.lse);
    f.top_scores = static_cast<float*>(L.top_scores);
    f.cand = a.cand;
    f.cand_n = a.cand_n;
    f.unsafe = a.unsafe;
    f.row_index = L.row_index;
    f.seg_bias = a.seg_bias;
    f.seg_len = L.seg_len;
    f.segs = L.segs;
    f.geo = a.geo;
    f.big16 = a.big16;
    f.rows = rows;
    f.m = L.m;
    f.topk = L.topk;
    f.scale = (float)L.scale;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // One resident wave, grid-stride: the warps of all SMs then walk the rows
    // together, so each slice's key and value rows are gathered while they
    // are hot in L2 (a second wave re-reads them: 4.1 GB instead of 2.7 GB of
    // DRAM reads at 128 slices).
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fwd_tc_finish<T>, FW * kWarp, 0) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    const int64_t want = (rows + FW - 1) / FW, cap = (int64_t)sms * per_sm;
    fwd_tc_finish<T><<<(unsigned)(want < cap ? want : cap), FW * kWarp, 0, L.stream>>>(f);
    rc = cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
  }
  if (pooled && cudaFreeAsync(ws, L.stream) != cudaSuccess) rc = SDK_ERR_CUDA;
  return rc;
}

}  // namespace

namespace {
// The shape conditions of the tensor-core path (everything but pointers).
bool tensorcore_shape(int64_t rows, int64_t m, int d, int dv, int topk, int score_grid, int dtype) {
  if (dtype != SDK_DTYPE_BF16 && dtype != SDK_DTYPE_F16) return false;
  if (d != D || dv != D || score_grid != 0) return false;
  if (m < 1 || m > 65536 || topk < 1 || topk > 64 || rows < 1) return false;
  return rows <= 0x7fffff00;
}
}  // namespace

bool fwd_tensorcore_supports(const FwdLaunch& L) {
  if (L.n < 1) return false;
  // a segment bias needs whole key tiles per segment
  if (L.seg_bias && (L.segs < 1 || L.seg_len < 1 || L.seg_len % TK != 0 || L.seg_len * L.segs != L.m ||
                     !aligned16(L.seg_bias)))
    return false;
  if (!tensorcore_shape(L.row_offsets ? L.n : L.slices * L.n, L.m, L.d, L.dv, L.topk, L.score_grid, L.dtype))
    return false;
  if (L.slices * L.m > 0x7fffffff) return false;
  if (!aligned16(L.q) || !aligned16(L.k) || !aligned16(L.v) || !aligned16(L.out)) return false;
  return encode_fn() != nullptr;
}

size_t fwd_tensorcore_workspace(int64_t rows, int64_t m, int d, int dv, int topk, int score_grid, bool grouped,
                                int dtype) {
  (void)grouped;  // grouped and uniform slices need the same scratch per row
  if (!tensorcore_shape(rows, m, d, dv, topk, score_grid, dtype)) return 0;
  return (size_t)rows * (CAP * 4 + 8);
}

int fwd_tensorcore(const FwdLaunch& L) {
  if (L.dtype == SDK_DTYPE_BF16) return launch<__nv_bfloat16>(L);
  if (L.dtype == SDK_DTYPE_F16) return launch<__half>(L);
  return SDK_ERR_UNSUPPORTED;
}

}  // namespace sdk
