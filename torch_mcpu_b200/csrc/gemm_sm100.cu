// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   C[M, N] = A[M, K] . B[N, K]^T      (bf16 in, fp32 accumulate, bf16 out)
//
// This is the mcpu device's aten::mm / aten::addmm for the MLP
// (csrc/aten/ops/mm.cpp:13-98 of kzwrime/torch_mcpu, which calls at::mm_out
// on host views) and, with the SwiGLU epilogue, the fused gate/up projection
// + silu_and_mul of the gated MLP.
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A 128x64 and B 256x64 tiles (128-byte swizzle)
//               into a 4-stage shared-memory ring.
//   warp 1      allocates 512 TMEM columns, then one thread issues
//               tcgen05.mma (M=128, N=256, K=16) into one of two TMEM
//               accumulators and commits each stage back to the producer.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns the
//               32 TMEM lanes = rows its warp index selects), convert, store.
// Two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
// Tiles are walked m-fastest so the CTAs working at one time share the same
// weight (B) tiles through L2.
//
// Every mbarrier wait is bounded; a wait that runs out sets the device error
// flag, the CTA drains what it issued and returns.
#include <cuda.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "sm100.cuh"
#include "silu_bf16.cuh"

namespace mcpu {
namespace gemm {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;         // two 128x256 fp32 accumulators
constexpr int THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

enum Epilogue { kPlain = 0, kSwiGLU = 1, kBias = 2 };

__device__ int g_error = 0;

struct Params {
  int M, N, K;       // N = columns of B (for SwiGLU: 2 x output columns)
  void* C;           // bf16 [M, ldc]
  long long ldc;     // elements
  const void* bias;  // bf16 [N] for kBias
  int epilogue;
  int tiles_m, tiles_n;
};

struct Smem {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* tiles = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  Smem* s = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &s->abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s->full[i], 1);
      mbar_init(&s->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->tmem_full[i], 1);
      mbar_init(&s->tmem_empty[i], 128);
    }
    mbar_init(&s->drain, 1);
    s->abort = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&s->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s->tmem_base;

  const int num_tiles = p.tiles_m * p.tiles_n;
  const int KB = (p.K + BK - 1) / BK;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, armed_parity = 0;  // per stage: ever armed / parity of last arm
    for (int t = blockIdx.x; t < num_tiles && !*abort; t += gridDim.x) {
      const int m_blk = t % p.tiles_m, n_blk = t / p.tiles_m;
      for (int kb = 0; kb < KB; ++kb) {
        if (!mbar_wait(&s->empty[stage], phase ^ 1u, abort)) break;
        uint8_t* sa = tiles + stage * STAGE_BYTES;
        mbar_arrive_expect_tx(&s->full[stage], STAGE_BYTES);
        tma_load_2d(sa, &tmA, &s->full[stage], kb * BK, m_blk * BM);
        tma_load_2d(sa + A_BYTES, &tmB, &s->full[stage], kb * BK, n_blk * BN);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // drain: every armed stage's copies have landed before the CTA exits
    for (int i = 0; i < STAGES; ++i) {
      if (!(armed & (1u << i))) continue;
      const uint32_t par = (armed_parity >> i) & 1u;
      for (uint32_t n = 0; n < kSpinLimit && !mbar_try_wait(&s->full[i], par); ++n) {
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_bf16(BM, BN);
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&s->tmem_empty[acc], acc_phase ^ 1u, abort)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + acc * BN;
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        if (!mbar_wait(&s->full[stage], phase, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(tiles + stage * STAGE_BYTES);
        const uint64_t adesc = smem_desc_k128(sa);
        const uint64_t bdesc = smem_desc_k128(sa + A_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // +32 bytes along K per step = +2 in the descriptor's address field
          umma_bf16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
        }
        umma_commit(&s->empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      umma_commit(&s->tmem_full[acc]);
    }
    // all issued MMAs complete before TMEM is released
    umma_commit(&s->drain);
    for (uint32_t n = 0; n < kSpinLimit && !mbar_try_wait(&s->drain, 0); ++n) {
    }
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue
    const int slice = warp & 3;  // TMEM lanes [32*slice, 32*slice+32)
    const int row_in_tile = slice * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&s->tmem_full[acc], acc_phase, abort)) break;
      tc_fence_after();
      const int m_blk = t % p.tiles_m, n_blk = t / p.tiles_m;
      const long long grow = static_cast<long long>(m_blk) * BM + row_in_tile;
      const bool row_ok = grow < p.M;
      const uint32_t tbase = tmem_base + acc * BN + (static_cast<uint32_t>(slice * 32) << 16);
      uint16_t* crow = static_cast<uint16_t*>(p.C) + grow * p.ldc;
      if (p.epilogue == kSwiGLU) {
        // columns [0,128) of the tile are gate, [128,256) the matching up
        const int out_cols = p.N / 2;
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + BN / 2 + c, u);
          tmem_ld_wait();
          const long long col0 = static_cast<long long>(n_blk) * (BN / 2) + c;
          if (row_ok) {
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // gate and up rounded to bf16 (the GEMMs' outputs), then
              // bf16(bf16(silu(gate)) * up); roundings two at a time
              const uint32_t g2 = pack_bf16x2(__uint_as_float(g[2 * j]), __uint_as_float(g[2 * j + 1]));
              const uint32_t u2 = pack_bf16x2(__uint_as_float(u[2 * j]), __uint_as_float(u[2 * j + 1]));
              const uint32_t s2 = pack_bf16x2(silu_for_bf16(__uint_as_float(g2 << 16)),
                                              silu_for_bf16(__uint_as_float(g2 & 0xFFFF0000u)));
              o[j] = pack_bf16x2(__fmul_rn(__uint_as_float(s2 << 16), __uint_as_float(u2 << 16)),
                                 __fmul_rn(__uint_as_float(s2 & 0xFFFF0000u), __uint_as_float(u2 & 0xFFFF0000u)));
            }
            if (col0 + 32 <= out_cols) {
              uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < out_cols)
                  crow[col0 + j] = static_cast<uint16_t>((o[j >> 1] >> (16 * (j & 1))) & 0xFFFF);
            }
          }
        }
      } else {
        const uint16_t* bias = static_cast<const uint16_t*>(p.bias);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_ld_wait();
          const long long col0 = static_cast<long long>(n_blk) * BN + c;
          if (row_ok && col0 < p.N) {
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v0 = __uint_as_float(r[2 * j]), v1 = __uint_as_float(r[2 * j + 1]);
              if (p.epilogue == kBias) {
                const long long c0 = col0 + 2 * j;
                v0 = __fadd_rn(v0, c0 < p.N ? bf16_bits_to_float(bias[c0]) : 0.0f);
                v1 = __fadd_rn(v1, c0 + 1 < p.N ? bf16_bits_to_float(bias[c0 + 1]) : 0.0f);
              }
              o[j] = pack_bf16x2(v0, v1);
            }
            if (col0 + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N)
                  crow[col0 + j] = static_cast<uint16_t>((o[j >> 1] >> (16 * (j & 1))) & 0xFFFF);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&s->tmem_empty[acc]);
    }
  }

  if (threadIdx.x == 0 && s->abort) atomicExch(&g_error, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] { fn = reinterpret_cast<EncodeTiledFn>(driver_entry("cuTensorMapEncodeTiled")); });
  return fn;
}

// K-major bf16 matrix [rows, K] with row pitch `ld` elements; box 64 x box_rows.
static orError_t make_map(CUtensorMap* m, const void* ptr, long long rows, long long K, long long ld,
                          int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_last_error("mm: cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return orErrorUnknown;
  }
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), gdim, gstride,
                   box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("mm: cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    return orErrorInvalidValue;
  }
  return orSuccess;
}

static int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

orError_t launch(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc,
                 long long M, long long N, long long K, int epilogue, const void* bias,
                 cudaStream_t st, int max_ctas) {
  MCPU_ARG_CHECK(M > 0 && N > 0 && K > 0, "mm: empty problem should not reach the kernel");
  MCPU_ARG_CHECK(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), "mm: dimension too large");
  MCPU_ARG_CHECK(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(B) % 16 == 0,
                 "mm: operands must be 16-byte aligned");
  MCPU_ARG_CHECK((lda * 2) % 16 == 0 && (ldb * 2) % 16 == 0,
                 "mm: row pitches of A and B must be multiples of 8 elements (TMA stride rule)");
  MCPU_ARG_CHECK(reinterpret_cast<uintptr_t>(C) % 16 == 0 && (ldc * 2) % 16 == 0,
                 "mm: output must be 16-byte aligned with a row pitch multiple of 8 elements");
  if (epilogue == kSwiGLU)
    MCPU_ARG_CHECK(N % BN == 0, "gemm_swiglu: 2 x intermediate (%lld) must be a multiple of %d", N, BN);
  CUtensorMap ta, tb;
  orError_t e = make_map(&ta, A, M, K, lda, BM);
  if (e != orSuccess) return e;
  e = make_map(&tb, B, N, K, ldb, BN);
  if (e != orSuccess) return e;
  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = C;
  p.ldc = ldc;
  p.bias = bias;
  p.epilogue = epilogue;
  p.tiles_m = static_cast<int>((M + BM - 1) / BM);
  p.tiles_n = static_cast<int>((N + BN - 1) / BN);
  const int tiles = p.tiles_m * p.tiles_n;
  int ctas = sm_count();
  if (max_ctas > 0 && max_ctas < ctas) ctas = max_ctas;
  if (tiles < ctas) ctas = tiles;
  gemm_bf16_kernel<<<ctas, THREADS, SMEM_BYTES, st>>>(ta, tb, p);
  return from_cuda(cudaGetLastError(), "mm launch");
}

}  // namespace gemm
}  // namespace mcpu

using namespace mcpu;

extern "C" orError_t mcpu_mm(const void* a, const void* b, void* out, int64_t M, int64_t N, int64_t K,
                             int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_BFLOAT16, "mm: only bfloat16 is supported (dtype code %d)", dtype);
  MCPU_ARG_CHECK(M >= 0 && N >= 0 && K >= 0, "mm: negative size");
  if (M == 0 || N == 0) return orSuccess;
  MCPU_ARG_CHECK(a && b && out, "mm: NULL tensor pointer");
  if (K == 0) return from_cuda(cudaMemsetAsync(out, 0, M * N * 2, as_cuda(stream)), "mm zero-K");
  return gemm::launch(a, K, b, K, out, N, M, N, K, gemm::kPlain, nullptr, as_cuda(stream), 0);
}

extern "C" orError_t mcpu_addmm(const void* bias, const void* a, const void* b, void* out, int64_t M,
                                int64_t N, int64_t K, int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_BFLOAT16, "addmm: only bfloat16 is supported (dtype code %d)", dtype);
  MCPU_ARG_CHECK(M >= 0 && N >= 0 && K > 0, "addmm: bad size");
  if (M == 0 || N == 0) return orSuccess;
  MCPU_ARG_CHECK(a && b && out && bias, "addmm: NULL tensor pointer");
  return gemm::launch(a, K, b, K, out, N, M, N, K, gemm::kBias, bias, as_cuda(stream), 0);
}

extern "C" orError_t mcpu_gemm_swiglu(const void* x, const void* w_gate_up, void* out, int64_t M,
                                      int64_t I, int64_t K, int dtype, orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_BFLOAT16, "gemm_swiglu: only bfloat16 is supported");
  MCPU_ARG_CHECK(M >= 0 && I > 0 && K > 0, "gemm_swiglu: bad size");
  if (M == 0) return orSuccess;
  MCPU_ARG_CHECK(x && w_gate_up && out, "gemm_swiglu: NULL tensor pointer");
  return gemm::launch(x, K, w_gate_up, K, out, I, M, 2 * I, K, gemm::kSwiGLU, nullptr,
                      as_cuda(stream), 0);
}

orError_t gemm::read_error(int* flag, bool reset) {
  MCPU_CUDA_TRY(cudaMemcpyFromSymbol(flag, gemm::g_error, sizeof(int)), "gemm error flag");
  if (reset) {
    const int zero = 0;
    MCPU_CUDA_TRY(cudaMemcpyToSymbol(gemm::g_error, &zero, sizeof(int)), "gemm error flag reset");
  }
  return orSuccess;
}
