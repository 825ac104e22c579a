// Dense affinity scores = q·kᵀ (fp32) on the 5th-generation tensor cores,
// for fp16 query and key rows: the stand-alone stage op of the reference's
// tiled_affinity (kernels/fused_topk_attn.py:227-287), whose fp16 path runs
// tl.dot on the tensor cores.
//
// One CTA writes a 128 × 256 tile of the score matrix:
//
//   warp 0     TMA producer: per 64-feature chunk of d, the 128 query rows and
//              the 256 key rows (128-byte swizzle; rows and features past the
//              ends read as zero) into a 2-stage ring;
//   warp 1     allocates 256 TMEM columns and issues tcgen05.mma
//              (M=128, N=256, K=16 x 4 per chunk) into one fp32 accumulator;
//   warps 4-7  epilogue: warp 4+j reads TMEM lanes 32j..32j+31 (query rows)
//              32 columns at a time and stores them as fp32, 128 contiguous
//              bytes per thread and chunk.
//
// Features past d read as zero in both operands, so d needs no padding; the
// tensor maps need 16-byte aligned bases, row strides that are multiples of 8
// halves and d >= 64 (one whole box of features); other calls take the
// CUDA-core kernel of stages.cu.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace sdk {
namespace {

using namespace sm100;

constexpr int AM = 128;        // query rows per CTA (MMA M, TMEM lanes)
constexpr int AN = 256;        // key rows per CTA (MMA N, TMEM columns)
constexpr int AF = 64;         // features per chunk (one 128-byte swizzle row)
constexpr int ASTAGES = 2;
constexpr int ANT = 256;
constexpr uint32_t A_BYTES = AM * AF * 2;
constexpr uint32_t B_BYTES = AN * AF * 2;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int OFF_BARS = ASTAGES * (int)STAGE_BYTES;
constexpr int SMEM_TOTAL = OFF_BARS + 128 + 1024;  // + alignment slack

struct AffArgs {
  float* s;
  int64_t n, m;
  int chunks;
  bool vec4;  // 16-byte stores are aligned (m % 4 == 0, 16-byte aligned output)
  unsigned int* status;
  uint64_t wait_limit_ns;
};

__global__ void __launch_bounds__(ANT, 1)
    affinity_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, AffArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BARS);
  uint64_t* full = bars;                // [stage]
  uint64_t* empty = bars + ASTAGES;     // [stage]
  uint64_t* acc_full = bars + 2 * ASTAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ASTAGES + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.y * AM, col0 = (int64_t)blockIdx.x * AN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ASTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, AN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int c = 0; c < a.chunks; ++c) {
        const int s = c % ASTAGES;
        if (!mbar_wait(&empty[s], ((uint32_t)(c / ASTAGES) & 1u) ^ 1u, abort_flag, a.wait_limit_ns)) break;
        uint8_t* st = sm + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        tma_load_2d(st, &tq, c * AF, (int)row0, &full[s]);
        tma_load_2d(st + A_BYTES, &tk, c * AF, (int)col0, &full[s]);
        ++issued;
      }
      if (*abort_flag) {
        // let the copies already in flight land before the CTA exits
        for (int c = (issued > ASTAGES ? issued - ASTAGES : 0); c < issued; ++c) {
          const uint64_t t0 = global_timer();
          while (!mbar_try_wait(&full[c % ASTAGES], (uint32_t)(c / ASTAGES) & 1u) &&
                 global_timer() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc_f16(false, AM, AN);
      bool done = true;
      for (int c = 0; c < a.chunks; ++c) {
        const int s = c % ASTAGES;
        if (!mbar_wait(&full[s], (uint32_t)(c / ASTAGES) & 1u, abort_flag, a.wait_limit_ns)) {
          done = false;
          break;
        }
        tc_fence_after();
        const uint32_t qa = smem_addr(sm + s * STAGE_BYTES), ka = qa + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < AF / 16; ++kk)
          mma_f16(tmem, smem_desc_k128(qa + kk * 32), smem_desc_k128(ka + kk * 32), idesc, c > 0 || kk > 0);
        mma_commit(&empty[s]);
      }
      // the accumulator is complete when the last MMAs are (or, after an
      // abort, when those issued so far are: TMEM is then not read)
      mma_commit(acc_full);
      if (!done) {
        const uint64_t t0 = global_timer();
        while (!mbar_try_wait(acc_full, 0) && global_timer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag, a.wait_limit_ns));
    if (ok && !*abort_flag) {
      tc_fence_after();
      const int64_t r = row0 + q * kWarp + lane;
      float* srow = a.s + r * a.m;
#pragma unroll 1
      for (int c = 0; c < AN / 32; ++c) {
        uint32_t v[32];
        tmem_load_32cols(tmem + ((uint32_t)(q * kWarp) << 16) + (uint32_t)(c * 32), v);
        tmem_wait_load(v);
        const int64_t c0 = col0 + c * 32;
        if (r < a.n) {
          if (a.vec4 && c0 + 32 <= a.m) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              reinterpret_cast<uint4*>(srow + c0)[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c0 + i < a.m) srow[c0 + i] = __uint_as_float(v[i]);
          }
        }
      }
    }
  }
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) raise_device_status(a.status, kStatusWaitTimeout);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, AN);
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

// [rows, d] fp16 rows `stride` halves apart, boxes of 64 features × box_rows rows.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int d, int64_t stride, int box_rows) {
  EncodeFn fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  const cuuint32_t box[2] = {(cuuint32_t)AF, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool affinity_tensorcore_supports(const void* q, const void* k, int64_t n, int64_t m, int d, int64_t qs, int64_t ks,
                                  int dtype) {
  if (dtype != SDK_DTYPE_F16) return false;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k) & 15)) return false;
  if (qs % 8 || ks % 8 || d < AF || d > 65535) return false;
  if (n > 0x7fffffff || m > 0x7fffffff || (n + AM - 1) / AM > 65535) return false;
  return encoder() != nullptr;
}

int affinity_tensorcore(const void* q, const void* k, float* scores, int64_t n, int64_t m, int d, int64_t qs,
                        int64_t ks, cudaStream_t stream) {
  CUtensorMap tq, tk;
  if (!make_map(&tq, q, n, d, qs, AM) || !make_map(&tk, k, m, d, ks, AN)) return SDK_ERR_CUDA;
  AffArgs a;
  a.s = scores;
  a.n = n;
  a.m = m;
  a.chunks = (d + AF - 1) / AF;
  a.vec4 = (m % 4 == 0) && ((reinterpret_cast<uintptr_t>(scores) & 15) == 0);
  a.status = device_status_ptr();
  a.wait_limit_ns = wait_limit_ns();
  if (cudaFuncSetAttribute(affinity_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL) !=
      cudaSuccess)
    return SDK_ERR_CUDA;
  const dim3 grid((unsigned)((m + AN - 1) / AN), (unsigned)((n + AM - 1) / AM));
  affinity_tc_kernel<<<grid, ANT, SMEM_TOTAL, stream>>>(tq, tk, a);
  return cudaPeekAtLastError() == cudaSuccess ? SDK_OK : SDK_ERR_CUDA;
}

}  // namespace sdk
