// Fused top-k attention forward on the 5th-generation tensor cores (sm_100a).
//
// One CTA owns 128 query rows of one (b, h) slice (d = dv = 64, bf16 or fp16)
// and streams the slice's keys twice in tiles of 256:
//
//   warp 0       TMA producer: the query tile once, then every K tile of
//                both passes into a 4-stage ring of 128-byte-swizzled
//                shared-memory buffers;
//   warp 1       allocates 512 TMEM columns and issues tcgen05.mma
//                (M=128, N=256, K=16 x 4) of S = Q·Kᵀ for every K tile into
//                one of two 256-column accumulators, committing to "S full"
//                / "stage free" mbarriers;
//   warps 2, 3   in the first CTA of each slice: the input magnitude check
//                of the slice's keys (below); for grouped rows: the gather of
//                the query rows through the permutation;
//   warps 4..19  selection: thread i of warps 4+j, 8+j, 12+j and 16+j
//                (j < 4) own query row 32j+i (TMEM lane); warp 4+4c+j reads
//                columns 64c..64c+63 of each 256-key tile.  Four selection
//                warps per SM sub-partition hide each other's latencies.
//
// Pass 1 records, per row, the maxima of disjoint groups of G keys (G chosen
// per call so that a row has at most 256 groups), rounded down to bf16.  The
// k-th largest group maximum tau is a lower bound of the row's k-th largest
// score: k different groups, so k different keys, reach it.  The four
// threads of a row find it by a bisection over the bf16 values, exchanging
// partial counts through shared memory.
//
// Pass 2 recomputes the scores and keeps the key of every score that reaches
// tau (a packed bf16 compare of the truncated scores: conservative), in the
// thread's quarter of the row's candidate list in global memory.  For
// Gaussian inputs about 1.15·k keys per row pass.  A second kernel, one warp
// per row, re-scores the candidates exactly from the gathered key rows (one
// fixed fp32 summation order), keeps the k best (larger score first, lower
// key index on ties), and writes the LSE, the indices and the
// softmax-weighted sum of the gathered value rows.  A row whose candidates
// overflow its list (heavily tied scores) is re-selected exactly by its warp
// over all keys.
//
// scale = 1/(T·sqrt(d)) > 0 is applied to each exact score, fl(dot·scale),
// or with a segment bias fl(fl(dot·scale)+bias), before the ranking.
#include <cuda.h>

#include <cmath>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sdk {
namespace {

using namespace sm100;

constexpr int TQ = 128;          // query rows per CTA (TMEM lanes, MMA M)
constexpr int TK = 256;          // keys per score tile (MMA N)
constexpr int NSEL = 4;          // selection threads per query row
constexpr int QK = TK / NSEL;    // keys of a tile per selection thread
constexpr int D = 64;            // feature width (one 128-byte swizzle row)
constexpr int KSTAGES = 4;
constexpr int CAP = 192;         // candidate keys per row
constexpr int CAPQ = CAP / NSEL; // candidate keys of each of the row's selection threads
constexpr int FIX_CAP = 128;     // exact list of a row re-selected by one warp
constexpr int NGW = 32;          // group-maximum words per selection thread (two bf16 each)
constexpr int NT = 128 + NSEL * 4 * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t Q_BYTES = TQ * D * 2;
constexpr uint32_t K_BYTES = TK * D * 2;

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + (int)Q_BYTES;
constexpr int OFF_GM = OFF_K + KSTAGES * (int)K_BYTES;     // [thread][word][row] group maxima
constexpr int OFF_XCH = OFF_GM + NSEL * NGW * TQ * 4;      // [slot][thread][row] the tau search's exchange
constexpr int OFF_BAR = OFF_XCH + 2 * NSEL * TQ * 4;
constexpr int NBARS = 1 + 2 * KSTAGES + 4;
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");
static_assert(OFF_GM % 1024 == 0 && OFF_K % 1024 == 0, "swizzled tiles need 1024-byte alignment");

// Count words of a row in the candidate buffer, one per selection thread:
// the number of keys it found (more than CAPQ: its part of the list
// overflowed, re-select the row exactly), or
constexpr int32_t kCandAborted = -2;  // a pipeline wait timed out: nothing to finish

struct TcArgs {
  const void* q;     // query rows, gathered through row_index when that is set
  const void* k;     // key rows, for the magnitude check
  const int32_t* row_index;  // nullable: logical row -> query row (grouped slices)
  uint16_t* cand;    // [rows][NSEL][CAPQ] candidate keys of each query row, per selection thread
  int32_t* cand_n;   // [rows][NSEL] key counts or kCandAborted
  uint32_t* unsafe;  // [rows], at each slice's first row: 1 when a key of the slice fails the magnitude check
  SliceGeometry geo;
  int64_t m;
  int topk;
  int glog;          // log2 of the keys per group maximum (5 .. 8)
  uint32_t big16;    // 16-bit magnitude field at which an element counts as unsafe
  unsigned int* status;
  uint64_t wait_limit_ns;  // bound of each pipeline wait (sdk_set_wait_limit)
  // kBias: score(r, j) = fl(fl(dot * scale) + seg_bias[r * segs + j / seg_len]),
  // seg_len a multiple of QK so that each thread's part of a tile lies in one segment
  const float* seg_bias;
  int64_t seg_len;
  int segs;
  float scale;
  int widen;  // scale is not a power of two (see the filter threshold)
};

// Input magnitude check.  With every |q|, |k| < 2^60 and finite, each of the
// 64 products is below 2^120 and their fp32 sum below 2^126, so no score can
// overflow to inf or become NaN; the stream passes then need no NaN
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

// ------------------------------------------------------------ pass helpers ---
constexpr uint32_t kBf16NegInf = 0xff80u;
constexpr uint32_t kBf16PosInf = 0x7f80u;

// The largest bf16 value <= x (x not NaN): truncation, one step further from
// zero for negative x with nonzero low bits.
__device__ __forceinline__ uint32_t bf16_floor(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u >> 16) + (((int32_t)u < 0 && (u & 0xffffu) != 0u) ? 1u : 0u);
}

// Order-preserving 16-bit code of a bf16 value and its inverse.
__device__ __forceinline__ uint32_t bf16_ord(uint32_t b) { return b ^ ((b & 0x8000u) ? 0xffffu : 0x8000u); }
__device__ __forceinline__ uint32_t bf16_of_ord(uint32_t o) { return o ^ ((o & 0x8000u) ? 0x8000u : 0xffffu); }

// Bit i set when key i's truncated score reaches the packed threshold tb2
// (one bf16 in both halves).  Word j packs the upper halves of keys j and
// j + 16; one byte permute, one packed compare and one logic op cover two
// keys.  Truncation is monotonic and tb2 is a bf16 value, so every key whose
// score reaches the threshold is set (and a few just below it, for negative
// scores).
__device__ __forceinline__ uint32_t hit_mask(const uint32_t (&v)[32], uint32_t tb2) {
  uint32_t m[4] = {0u, 0u, 0u, 0u};  // four independent chains, joined at the end
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t p = __byte_perm(v[j], v[j + 16], 0x7632);
    uint32_t w;
    asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(w) : "r"(p), "r"(tb2));
    m[j & 3] |= w & (0x00010001u << j);
  }
  return (m[0] | m[1]) | (m[2] | m[3]);
}

// Maxima of the four 8-key groups of a 32-key chunk.
__device__ __forceinline__ void max8x4(const uint32_t (&v)[32], float (&g)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t* x = v + 8 * j;
    const float a = max3_nan(__uint_as_float(x[0]), __uint_as_float(x[1]), __uint_as_float(x[2]));
    const float b = max3_nan(__uint_as_float(x[3]), __uint_as_float(x[4]), __uint_as_float(x[5]));
    g[j] = max3_nan(a, b, max_nan(__uint_as_float(x[6]), __uint_as_float(x[7])));
  }
}

// Number of packed bf16 values of `words` consecutive group-maximum words
// (stride TQ*4 bytes from `addr`) that reach the packed threshold p2.
__device__ __forceinline__ int count_ge(uint32_t addr, int words, uint32_t p2) {
  int c0 = 0, c1 = 0;
  int w = 0;
  for (; w + 4 <= words; w += 4) {
    uint32_t x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x[i]) : "r"(addr + (uint32_t)(w + i) * (TQ * 4u)) : "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t r;
      asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(x[i]), "r"(p2));
      if (i & 1) c1 += __popc(r); else c0 += __popc(r);
    }
  }
  for (; w < words; ++w) {
    uint32_t x, r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x) : "r"(addr + (uint32_t)w * (TQ * 4u)) : "memory");
    asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(p2));
    c0 += __popc(r);
  }
  return (c0 + c1) >> 4;  // 16 set bits per passing half
}

// Packed pass-2 threshold of one thread's half tile with segment bias b: a
// bf16 value t such that every raw dot d with fl(fl(d·scale) + b) >= tau
// has trunc16(d) >= t.  tau = -inf (no bound) admits every key; b = -inf
// with a finite tau admits none.  The margin covers the two roundings of the
// final score and the rounding of the quotient.
__device__ __forceinline__ uint32_t biased_threshold(float tau, float b, float scale) {
  if (tau == __int_as_float(0xff800000)) return kBf16NegInf * 0x00010001u;
  if (b == __int_as_float(0xff800000)) return kBf16PosInf * 0x00010001u;
  const float num = tau - b;
  const float margin = (fabsf(tau) + fabsf(b)) * 0x1p-16f + 0x1p-120f;
  const float t = __fdiv_rd(num - margin, scale);
  if (t != t) return kBf16NegInf * 0x00010001u;
  return bf16_floor(t) * 0x00010001u;
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
                                          int lane, int stride) {
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
    // the final score: scaled, then shifted by the key's segment bias
    s = __fmul_rn(s, scale);
    if (bias_row && valid) s = __fadd_rn(s, bias_row[key / seg_len]);
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
  // softmax shift: the row maximum, or 0 when it is not finite (all scores
  // -inf gives LSE -inf; a NaN or +inf maximum gives NaN / +inf)
  const float mxs = finite_or_zero(fv[0]);
  float part = 0.f;
  for (int j = lane; j < c0; j += kWarp) part += expf(fv[j] - mxs);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  const float lse = mxs + logf(part);
  if (lane == 0) a.lse[gr] = lse;
  write_row<T>(static_cast<const T*>(a.v) + slice * m * D, [&](int j) { return fv[j]; }, [&](int j) { return fi[j]; },
               c0, 1.f, lse, static_cast<T*>(a.out) + pr * D, a.top_idx + gr * stride,
               a.top_scores ? a.top_scores + gr * stride : nullptr, lane);
  __syncwarp();
}

// kBias: scores shifted per (row, key segment); see TcArgs.
template <typename T, bool kBias>
__global__ void __launch_bounds__(NT, 1)
    fused_fwd_tc(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                 TcArgs a) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* qs = sm + OFF_Q;
  uint8_t* ks = sm + OFF_K;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 1 + KSTAGES;
  uint64_t* s_full = bars + 1 + 2 * KSTAGES;  // [buffer]
  uint64_t* s_empty = s_full + 2;             // [buffer]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_MISC + 4);
  volatile uint32_t* scan_big = reinterpret_cast<volatile uint32_t*>(sm + OFF_MISC + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t slice, row0;
  int count;  // rows of this CTA (TQ, fewer at a slice's end, 0 for a surplus grouped CTA)
  locate_tile(a.geo, blockIdx.x, TQ, &slice, &row0, &count);
  if (count <= 0) return;
  const int64_t slice_row0 = slice_row_begin(a.geo, slice);
  const int ntiles = (int)((a.m + TK - 1) / TK);
  const int jobs = 2 * ntiles;  // both passes

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], NSEL * 4 * kWarp);
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
        mbar_arrive_expect_tx(q_full, Q_BYTES);
        tma_load_2d(qs, &tmap_q, 0, (int)row0, q_full);
      }
      for (int j = 0; j < jobs; ++j) {
        const int s = j % KSTAGES;
        const uint32_t ph = (uint32_t)(j / KSTAGES) & 1u;
        if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag, a.wait_limit_ns)) break;
        mbar_arrive_expect_tx(&k_full[s], K_BYTES);
        tma_load_2d(ks + s * K_BYTES, &tmap_k, 0, (int)(slice * a.m + (int64_t)(j % ntiles) * TK), &k_full[s]);
        ++issued;
      }
      if (*abort_flag) {
        // let the copies already in flight land before the CTA exits
        for (int j = (issued > KSTAGES ? issued - KSTAGES : 0); j < issued; ++j) {
          const uint64_t t0 = global_timer();
          while (!mbar_try_wait(&k_full[j % KSTAGES], (uint32_t)(j / KSTAGES) & 1u) &&
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
      for (int c = t; c < TQ * (D / 8); c += 2 * kWarp) {
        const int r = c >> 3, ch = c & 7;
        const uint32_t dst = qbase + (uint32_t)r * (D * 2) + ((uint32_t)(ch ^ (r & 7)) << 4);
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
        for (int j = 0; j < jobs; ++j) {
          const int s = j % KSTAGES, b = j & 1;
          const uint32_t ph_b = (uint32_t)(j >> 1) & 1u;
          if (!mbar_wait(&k_full[s], (uint32_t)(j / KSTAGES) & 1u, abort_flag, a.wait_limit_ns)) break;
          if (!mbar_wait(&s_empty[b], ph_b ^ 1u, abort_flag, a.wait_limit_ns)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_addr(ks + s * K_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_f16(tmem + (uint32_t)(b * TK), smem_desc_k128(q_addr + kk * 32), smem_desc_k128(k_addr + kk * 32),
                    idesc, kk > 0);
          mma_commit(&s_full[b]);
          mma_commit(&k_empty[s]);
          last_bar = &s_full[b];
          last_ph = ph_b;
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
    const int h = (warp - 4) >> 2, quarter = warp & 3;  // column quarter, lane quarter
    const int rl = quarter * kWarp + lane;  // row within the CTA == TMEM lane
    const bool live = rl < count;
    const int64_t gr = row0 + rl;
    const uint32_t tm = tmem + ((uint32_t)(quarter * kWarp) << 16) + (uint32_t)(h * QK);
    const uint32_t row_bar = 2u + (uint32_t)quarter;  // the four warps of this lane quarter
    // group maxima: value v of this thread at word v/2, half v%2 of column rl
    const uint32_t gm_base = smem_addr(sm + OFF_GM) + (uint32_t)(h * NGW * TQ + rl) * 4u;
    uint32_t* xch = reinterpret_cast<uint32_t*>(sm + OFF_XCH);
    const int gsh = a.glog - 5;  // a group is 2^gsh chunks of 32 keys of this thread
    const float neg_inf_f = __int_as_float(0xff800000);
    bool ok = true;

    // One 32-column chunk at a time; the other selection warps of the SM
    // sub-partition cover the TMEM load latency.  The TMEM buffer is
    // released once the tile's last chunk is in registers.  Chunks past the
    // last key (only in the last tile of a slice) take the masked variant.
    auto stream_tile = [&](int j, auto&& chunk) -> bool {
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)(j >> 1) & 1u, abort_flag, a.wait_limit_ns)))
        return false;
      tc_fence_after();
      const int t = j % ntiles;
      const int64_t key_q = (int64_t)t * TK + h * QK;
      const int q_valid = (int)(a.m - key_q < QK ? (a.m - key_q > 0 ? a.m - key_q : 0) : QK);
#pragma unroll
      for (int c = 0; c < QK / 32; ++c) {
        uint32_t v[32];
        tmem_load_32cols(tm + b * TK + c * 32, v);
        tmem_wait_load(v);
        if (c == QK / 32 - 1) {
          tc_fence_before();
          mbar_arrive(&s_empty[b]);
        }
        if (q_valid >= QK)
          chunk(v, key_q + c * 32, 32, std::true_type{});
        else
          chunk(v, key_q + c * 32, q_valid - c * 32, std::false_type{});
      }
      return true;
    };

    // ---- pass 1: group maxima (value v at word v/2, half v%2), rounded
    // down to bf16; the finite values' range and count are kept for the tau
    // search.
    int nv = 0;             // values written
    int cc = 0;             // chunks seen
    float run = neg_inf_f;  // running maximum of a group spanning chunks
    float lo_f = __int_as_float(0x7f800000), hi_f = neg_inf_f;
    int nfin = 0;
    auto put = [&](float x) {
      asm volatile("st.shared.u16 [%0], %1;"
                   ::"r"(gm_base + (uint32_t)(nv >> 1) * (TQ * 4u) + (uint32_t)(nv & 1) * 2u),
                   "h"((unsigned short)bf16_floor(x))
                   : "memory");
      const bool fin = x > neg_inf_f;  // NaN only in rows re-selected later
      hi_f = fmaxf(hi_f, x);
      lo_f = fminf(lo_f, fin ? x : __int_as_float(0x7f800000));
      nfin += fin ? 1 : 0;
      ++nv;
    };
    float bias1 = 0.f;
    for (int j = 0; j < ntiles && ok; ++j) {
      if (kBias && live) {
        const int64_t key_q = (int64_t)j * TK + h * QK;
        bias1 = key_q < a.m ? __ldg(a.seg_bias + gr * a.segs + key_q / a.seg_len) : 0.f;
      }
      ok = stream_tile(j, [&](uint32_t(&v)[32], int64_t, int valid, auto whole) {
        if constexpr (!decltype(whole)::value) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i >= valid) v[i] = 0xff800000u;
        }
        float g[4];
        max8x4(v, g);
        float x = max_nan(max3_nan(g[0], g[1], g[2]), g[3]);
        if (kBias) x = __fadd_rn(__fmul_rn(x, a.scale), bias1);
        run = max_nan(run, x);
        ++cc;
        if ((cc & ((1 << gsh) - 1)) == 0) {
          put(run);
          run = neg_inf_f;
        }
      });
    }
    if ((cc & ((1 << gsh) - 1)) != 0) put(run);  // a group cut short by the last tile
    if (nv & 1) {  // pad the last word's upper half
      asm volatile("st.shared.u16 [%0], %1;" ::"r"(gm_base + (uint32_t)(nv >> 1) * (TQ * 4u) + 2u),
                   "h"((unsigned short)kBf16NegInf)
                   : "memory");
    }
    uint32_t lo = nfin ? bf16_ord(bf16_floor(lo_f)) : 0xffffu;
    uint32_t hi = nfin ? bf16_ord(bf16_floor(hi_f)) : 0u;
    const int words = (nv + 1) >> 1;

    // ---- tau: the k-th largest group maximum of the row (all four
    // threads' values), by bisection over ordered bf16 codes; L always
    // satisfies count(>= L) >= k, H is the lowest code known to fail.  The
    // four threads of a row compute the same L and H, so the four warps of a
    // lane quarter meet the same number of barriers.
    xch[(0 * NSEL + h) * TQ + rl] = (lo & 0xffffu) | (hi << 16);
    xch[(1 * NSEL + h) * TQ + rl] = (uint32_t)nfin;
    named_bar_sync(row_bar, NSEL * kWarp);
    nfin = 0;
#pragma unroll
    for (int o = 0; o < NSEL; ++o) {
      const uint32_t pr = xch[(0 * NSEL + o) * TQ + rl];
      lo = min(lo, pr & 0xffffu);
      hi = max(hi, pr >> 16);
      nfin += (int)xch[(1 * NSEL + o) * TQ + rl];
    }
    uint32_t L = lo, H = hi + 1u;
    const bool bounded = nfin >= a.topk;  // else: no bound, every key is a candidate
    if (!bounded) {
      L = 0u;
      H = 1u;
    }
    while (__any_sync(0xffffffffu, H - L > 1u)) {
      const bool act = H - L > 1u;
      const uint32_t mid = (L + H) >> 1;
      const uint32_t p2 = bf16_of_ord(mid) * 0x00010001u;
      const int mine = act ? count_ge(gm_base, words, p2) : 0;
      named_bar_sync(row_bar, NSEL * kWarp);  // the other threads have read the previous exchange
      xch[h * TQ + rl] = (uint32_t)mine;
      named_bar_sync(row_bar, NSEL * kWarp);
      int c = 0;
#pragma unroll
      for (int o = 0; o < NSEL; ++o) c += (int)xch[o * TQ + rl];
      if (act) {
        if (c >= a.topk) L = mid; else H = mid;
      }
    }
    // Rows are ranked on fl(dot·scale).  When scale is not a power of two,
    // that rounding can tie a key below tau with one at or above it (and the
    // lower key index wins the tie), so the filter then starts one bf16 step
    // lower: every dot whose scaled value equals that of a dot >= tau lies
    // within a few fp32 ulps of it.
    if (!kBias && a.widen && L > bf16_ord(kBf16NegInf)) L -= 1u;
    const uint32_t tau_b = bounded ? bf16_of_ord(L) : kBf16NegInf;
    const float tau = __uint_as_float(tau_b << 16);

    // ---- pass 2: candidate keys, into this thread's part of the row's list
    const uint32_t tb2_plain = tau_b * 0x00010001u;
    uint16_t* crow = a.cand + gr * CAP + h * CAPQ;
    uint32_t cnt = 0;
    for (int j = ntiles; j < jobs && ok; ++j) {
      uint32_t tb2 = tb2_plain;
      if (kBias && live) {
        const int64_t key_q = (int64_t)(j - ntiles) * TK + h * QK;
        const float bias2 = key_q < a.m ? __ldg(a.seg_bias + gr * a.segs + key_q / a.seg_len) : 0.f;
        tb2 = biased_threshold(tau, bias2, a.scale);
      }
      ok = stream_tile(j, [&](uint32_t(&v)[32], int64_t key0, int valid, auto whole) {
        uint32_t m = hit_mask(v, tb2);
        if constexpr (!decltype(whole)::value) m &= valid >= 32 ? 0xffffffffu : (valid > 0 ? (1u << valid) - 1u : 0u);
        if (!live) m = 0u;
        // one hit of each lane per round, a warp-uniform number of rounds
        const uint32_t rounds = __reduce_max_sync(0xffffffffu, (uint32_t)__popc(m));
        for (uint32_t rd = 0; rd < rounds; ++rd) {
          const bool hit = m != 0u;
          const uint32_t i = hit ? 31u - __clz(m) : 0u;
          m ^= hit ? 1u << i : 0u;
          if (hit && cnt < (uint32_t)CAPQ) crow[cnt] = (uint16_t)((uint32_t)key0 + i);
          cnt += hit ? 1u : 0u;
        }
      });
    }
    // Hand this part of the row to the finish kernel: its count (more than
    // CAPQ: overflowed) or kCandAborted.
    named_bar_sync(row_bar, NSEL * kWarp);
    if (live) a.cand_n[NSEL * gr + h] = *abort_flag ? kCandAborted : (int32_t)cnt;
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
// candidates (key, exact score) in shared memory; the exact re-selection of
// a row whose list overflowed reuses the same arrays.
constexpr int FW = 8;             // warps per finish block
constexpr int FUNR = 4;           // key or value rows in flight per lane group
constexpr int NV = CAP / kWarp;   // candidates per lane

struct FinArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int32_t* top_idx;
  float* lse;
  float* top_scores;
  const uint16_t* cand;
  const int32_t* cand_n;
  const uint32_t* unsafe;  // at each slice's first row, from the stream kernel's key check
  const int32_t* row_index;  // nullable: logical row -> query/output row
  const float* seg_bias;     // nullable: per (logical row, key segment), as in TcArgs
  const int32_t* row_k;      // nullable: per logical row, the number of keys to keep
  int64_t seg_len;
  int segs;
  SliceGeometry geo;
  int64_t rows, m;
  int topk;
  float scale;
  uint32_t big16;
};

struct __align__(16) FinWarp {
  float sc[CAP];  // candidates' exact scores, then the selection's (list order)
  int si[CAP];    // their key indices
  float pw[64];   // softmax weight of each selection
  float pad[4];
};
static_assert(sizeof(float) * CAP + sizeof(int) * CAP >= FIX_CAP * 8, "re-selection buffers exceed sc/si");

// Order-preserving 32-bit form of a score (NaN highest, -0 == +0).
__device__ __forceinline__ uint32_t ord_score(float x) {
  if (x != x) return 0xffffffffu;
  const uint32_t u = __float_as_uint(x + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Keeps the `topk` best of the row's `cnt` candidates in w.sc / w.si
// (larger score first, lower key index on ties; cnt >= topk), in list order,
// at the front of w.sc / w.si; returns the largest score.  NVT candidates per
// lane.  The lowest-ranked candidate is dropped until topk remain: the
// lowest ordered score, and among equal scores the highest key index.
template <int NVT>
__device__ __forceinline__ float cut_candidates(int cnt, int topk, FinWarp& w, int lane) {
  float xs[NVT];
  int ks[NVT];
  uint32_t os[NVT];
  bool hk[NVT];
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int s = lane + kWarp * i;
    hk[i] = s < cnt;
    xs[i] = hk[i] ? w.sc[s] : 0.f;
    ks[i] = hk[i] ? w.si[s] : 0;
    os[i] = ord_score(xs[i]);
  }
  __syncwarp();  // every lane holds its candidates before the compaction below overwrites them
  for (int dn = cnt - topk; dn > 0; --dn) {
    uint32_t mn = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < NVT; ++i) mn = hk[i] ? min(mn, os[i]) : mn;
    mn = __reduce_min_sync(0xffffffffu, mn);
    int kx = -1;
#pragma unroll
    for (int i = 0; i < NVT; ++i) kx = (hk[i] && os[i] == mn) ? max(kx, ks[i]) : kx;
    kx = __reduce_max_sync(0xffffffffu, kx);
#pragma unroll
    for (int i = 0; i < NVT; ++i) hk[i] = hk[i] && !(os[i] == mn && ks[i] == kx);
  }
  const unsigned lt = (1u << lane) - 1u;
  int pos = 0;
  float mx = __int_as_float(0xff800000);
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const unsigned bal = __ballot_sync(0xffffffffu, hk[i]);
    if (hk[i]) {
      const int p = pos + __popc(bal & lt);
      w.sc[p] = xs[i];
      w.si[p] = ks[i];
      mx = fmaxf(mx, xs[i]);
    }
    pos += __popc(bal);
  }
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  return mx;
}

template <typename T>
__global__ void __launch_bounds__(FW * kWarp, 4) fwd_tc_finish(FinArgs a) {
  __shared__ FinWarp sw[FW];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane & 7, grp = lane >> 3;
  FinWarp& w = sw[warp];
  for (int64_t r = (int64_t)blockIdx.x * FW + warp; r < a.rows; r += (int64_t)gridDim.x * FW) {
    const int4 cq = reinterpret_cast<const int4*>(a.cand_n)[r];
    const int c0 = cq.x, c1 = cq.y, c2 = cq.z, c3 = cq.w;
    if (c0 == kCandAborted || c1 == kCandAborted || c2 == kCandAborted || c3 == kCandAborted) {
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
    const int cnt = c0 + c1 + c2 + c3;
    const int64_t slice = slice_of_row(a.geo, r);
    const int64_t pr = a.row_index ? (int64_t)a.row_index[r] : r;  // query and output row
    const uint4 qg = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) + pr * D) + g);
    const uint32_t add = (0x8000u - a.big16) * 0x00010001u;
    const bool unsafe = __any_sync(0xffffffffu, (big_halves(qg.x, add) | big_halves(qg.y, add) |
                                                 big_halves(qg.z, add) | big_halves(qg.w, add)) != 0u) ||
                        a.unsafe[slice_row_begin(a.geo, slice)] != 0u;
    const float* brow = a.seg_bias ? a.seg_bias + r * a.segs : nullptr;
    bool bias_bad = false;  // NaN or +inf biases are ranked by the exact path only
    if (brow)
      for (int j = lane; j < a.segs; j += kWarp) bias_bad |= !(brow[j] < __int_as_float(0x7f800000));
    // keys this row keeps (adaptive k); its other index slots are -1
    const int kr = a.row_k ? min(max(a.row_k[r], 1), a.topk) : a.topk;
    for (int j = kr + lane; j < a.topk; j += kWarp) {
      a.top_idx[r * a.topk + j] = -1;
      if (a.top_scores) a.top_scores[r * a.topk + j] = __int_as_float(0xff800000);
    }
    if (min(min(c0, c1), min(c2, c3)) < 0 || max(max(c0, c1), max(c2, c3)) > CAPQ || cnt < a.topk || unsafe ||
        __any_sync(0xffffffffu, bias_bad)) {
      uint8_t* fix = reinterpret_cast<uint8_t*>(&w);
      reselect_row<T>(RowOut{a.q, a.k, a.v, a.out, a.top_idx, a.lse, a.top_scores}, a.m, kr, a.scale, slice, r, pr,
                      brow, a.seg_len, reinterpret_cast<float*>(fix), reinterpret_cast<int*>(fix + FIX_CAP * 4),
                      w.pad, lane, a.topk);
      continue;
    }
    // the candidates of the four selection threads, in list order
    const uint16_t* crow = a.cand + r * CAP;
    const int o1 = c0, o2 = c0 + c1, o3 = c0 + c1 + c2;
    for (int s = lane; s < cnt; s += kWarp)
      w.si[s] = (int)crow[s < o1 ? s : (s < o2 ? CAPQ + (s - o1) : (s < o3 ? 2 * CAPQ + (s - o2) : 3 * CAPQ + (s - o3)))];
    __syncwarp();
    // exact scores: group grp re-scores candidates grp, grp + 4, ... from the
    // gathered key rows (eight lanes per 128-byte row, one fixed summation order)
    const T* kbase = static_cast<const T*>(a.k) + slice * a.m * D;
    for (int s0 = 0; s0 < cnt; s0 += 4 * FUNR) {
      uint4 kc[FUNR];
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        const int s = s0 + 4 * u + grp;
        kc[u] = make_uint4(0u, 0u, 0u, 0u);
        if (s < cnt) kc[u] = __ldg(reinterpret_cast<const uint4*>(kbase + (int64_t)w.si[s] * D) + g);
      }
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        const int s = s0 + 4 * u + grp;
        const float d = group_dot<T>(qg, kc[u]);
        // the final score, as the generic kernel forms it: fl(dot·scale),
        // shifted by the key's segment bias when there is one
        const float x = __fmul_rn(d, a.scale);
        if (g == 0 && s < cnt) w.sc[s] = brow ? __fadd_rn(x, brow[w.si[s] / a.seg_len]) : x;
      }
    }
    __syncwarp();
    // the k best, in list order
    const float mx = cnt <= 3 * kWarp ? cut_candidates<3>(cnt, kr, w, lane) : cut_candidates<NV>(cnt, kr, w, lane);
    const int sel = kr;
    // LSE; lane j holds selections j and j + 32 (k <= 64)
    const bool v0 = lane < sel, v1 = lane + kWarp < sel;
    const float x0 = v0 ? w.sc[lane] : 0.f, x1 = v1 ? w.sc[lane + kWarp] : 0.f;
    const int k0 = v0 ? w.si[lane] : 0, k1 = v1 ? w.si[lane + kWarp] : 0;
    const float mxs = finite_or_zero(mx);
    float part = (v0 ? expf(x0 - mxs) : 0.f) + (v1 ? expf(x1 - mxs) : 0.f);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o2);
    const float lse = mxs + logf(part);
    if (lane == 0) a.lse[r] = lse;
    int32_t* idx_row = a.top_idx + r * a.topk;
    if (v0) {
      w.pw[lane] = expf(x0 - lse);
      idx_row[lane] = k0;
      if (a.top_scores) a.top_scores[r * a.topk + lane] = x0;
    }
    if (v1) {
      w.pw[lane + kWarp] = expf(x1 - lse);
      idx_row[lane + kWarp] = k1;
      if (a.top_scores) a.top_scores[r * a.topk + lane + kWarp] = x1;
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
          pj[u] = w.pw[j];
          vc[u] = __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)w.si[j] * D) + g);
        }
      }
#pragma unroll
      for (int u = 0; u < FUNR; ++u) {
        float f[8];
        unpack8<T>(vc[u], f);
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) acc[hh] = fmaf(pj[u], f[hh], acc[hh]);
      }
    }
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) {
      acc[hh] += __shfl_xor_sync(0xffffffffu, acc[hh], 8);
      acc[hh] += __shfl_xor_sync(0xffffffffu, acc[hh], 16);
    }
    if (lane < 8) {
      uint4 u;
      T* ev = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) ev[hh] = from_acc<T>(acc[hh]);
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

// Row-major [rows, 64] 16-bit matrix, boxes of `box_rows` rows, 128-byte swizzle.
bool make_rows_map(CUtensorMap* map, const void* base, int64_t rows, bool bf16, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {(cuuint32_t)D, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// log2 of the keys per group maximum: the smallest group (32 .. 256 keys)
// that leaves each selection thread at most 2·NGW values.
int group_log(int64_t m) {
  const int64_t chunks = ((m + TK - 1) / TK) * (QK / 32);  // 32-key chunks per selection thread
  for (int gl = 5; gl < 8; ++gl)
    if (((chunks + (1 << (gl - 5)) - 1) >> (gl - 5)) <= 2 * NGW) return gl;
  return 8;
}

// candidate keys, NSEL counts and the slice check word
size_t workspace_per_row() { return (size_t)CAP * sizeof(uint16_t) + 4 * NSEL + 4; }

template <typename T>
int launch(const FwdLaunch& L) {
  CUtensorMap tq, tk;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const bool grouped = L.row_offsets != nullptr;
  // grouped: n is the total row count, slice s owns rows [row_offsets[s], row_offsets[s+1])
  const int64_t rows = grouped ? L.n : L.slices * L.n;
  if (rows <= 0) return SDK_OK;
  if (!make_rows_map(&tq, L.q, rows, bf16, TQ)) return SDK_ERR_CUDA;
  if (!make_rows_map(&tk, L.k, L.slices * L.m, bf16, TK)) return SDK_ERR_CUDA;
  TcArgs a;
  a.q = L.q;
  a.k = L.k;
  a.row_index = L.row_index;
  a.geo = SliceGeometry{L.row_offsets, L.slices, L.n};
  a.m = L.m;
  a.topk = L.topk;
  a.glog = group_log(L.m);
  a.status = L.status;
  a.wait_limit_ns = wait_limit_ns();
  a.seg_bias = static_cast<const float*>(L.seg_bias);
  a.seg_len = L.seg_len;
  a.segs = L.segs;
  a.scale = (float)L.scale;
  {
    int e2 = 0;
    a.widen = std::frexp(a.scale, &e2) != 0.5f;
  }
  // grouped: at most ceil(rows / TQ) + slices tiles; CTAs past the last exit at once
  const int64_t grid = grouped ? (rows + TQ - 1) / TQ + L.slices : L.slices * ((L.n + TQ - 1) / TQ);
  if (grid <= 0) return SDK_OK;
  if (grid > 0x7fffffff) return SDK_ERR_UNSUPPORTED;
  const bool bias = L.seg_bias != nullptr;
  auto kern = bias ? fused_fwd_tc<T, true> : fused_fwd_tc<T, false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
    return SDK_ERR_CUDA;
  const size_t need = (size_t)rows * workspace_per_row();
  void* ws = L.workspace;
  const bool pooled = ws == nullptr;
  if (pooled) {
    cudaMemPool_t pool = scratch_pool();
    if (!pool) return SDK_ERR_CUDA;
    if (cudaMallocFromPoolAsync(&ws, need, pool, L.stream) != cudaSuccess) return SDK_ERR_CUDA;
  } else if (L.workspace_bytes < need || !aligned16(ws)) {
    return SDK_ERR_INVALID_ARGUMENT;
  }
  // per row: CAP candidate keys, NSEL counts and a flag (set at the first row of each slice)
  uint8_t* wb = static_cast<uint8_t*>(ws);
  a.cand = reinterpret_cast<uint16_t*>(wb);
  a.cand_n = reinterpret_cast<int32_t*>(wb + (size_t)rows * CAP * sizeof(uint16_t));
  a.unsafe = reinterpret_cast<uint32_t*>(wb + (size_t)rows * (CAP * sizeof(uint16_t) + 4 * NSEL));
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
    f.row_k = L.row_k;
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
    // are hot in L2.
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
  // a segment bias needs whole tile quarters per segment
  if (L.seg_bias && (L.segs < 1 || L.seg_len < 1 || L.seg_len % QK != 0 || L.seg_len * L.segs != L.m ||
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
  return (size_t)rows * workspace_per_row();
}

int fwd_tensorcore(const FwdLaunch& L) {
  if (L.dtype == SDK_DTYPE_BF16) return launch<__nv_bfloat16>(L);
  if (L.dtype == SDK_DTYPE_F16) return launch<__half>(L);
  return SDK_ERR_UNSUPPORTED;
}

}  // namespace sdk
