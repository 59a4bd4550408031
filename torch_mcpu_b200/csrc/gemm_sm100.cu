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
//
// The same kernel, instantiated with kAR = true, is the row-parallel down
// projection of the TP MLP fused with the SUM all-reduce of its partials
// over NVLink (mcpu_mm_allreduce):
//   phase A  each epilogue warp converts its 32 accumulator rows to bf16 and
//            writes them, staged through shared memory as full 128-byte
//            lines, into the window of the slice's owner rank; then, after
//            a warp barrier, it bumps the owner's four unit counters
//            (release, system scope: cumulative over the warp's stores);
//   phase B  four more warps per CTA (warps 6-9), running beside the GEMM
//            from the start, take this rank's units (8 rows x 256 columns
//            of a slice) in tile order: wait until all ranks' partials have
//            arrived, sum them in fp32 in rank order, round once to bf16
//            and store the rows into every rank's output; at the end, a
//            warp barrier and one release increment of every rank's done
//            counter;
//   finish   one thread waits for its own done counter to reach the number
//            of units, so the launch ends only when this rank's output is
//            complete.
// Counters are reset by their consumer, so a window is reusable by the next
// call (and by a replayed CUDA graph) without host work.  The launch is
// cooperative: every CTA is resident, so no wait depends on an unscheduled
// block.
#include <cuda.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "peer.cuh"
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
constexpr int REDUCER_WARPS = 4;                       // kAR: phase-B warps 6..9
constexpr int THREADS_AR = THREADS + 32 * REDUCER_WARPS;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

enum Epilogue { kPlain = 0, kSwiGLU = 1, kBias = 2 };

__device__ int g_error = 0;

// ---- fused all-reduce (kAR): window layout and work units
namespace ar {
constexpr int kSliceRows = 32;                               // one epilogue warp's TMEM lanes
constexpr int kUnitRows = 8;                                 // rows one phase-B unit reduces
constexpr int kUnitsPerSlice = kSliceRows / kUnitRows;       // 4
constexpr long long kRowBytes = BN * 2;                      // 512: one slice row of bf16
constexpr long long kSliceBytes = kSliceRows * kRowBytes;    // 16 KB
constexpr long long kUnitBytes = kUnitRows * kRowBytes;      // 4 KB
constexpr long long kCountersOff = 256;                      // u32 done counter at 0
constexpr long long kAlign = 4096;
constexpr int kStagingBytes = 4 * kSliceRows * 128;          // 4 warps x 32 rows x 64 bf16

inline long long align_up(long long v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Leading bytes of a window that hold the done counter and one counter per
// unit of the largest problem the window can hold; fixed for a window, so a
// later call with another M finds its counters at zero.
inline long long control_bytes(unsigned long long bytes, int world) {
  const long long max_slots =
      static_cast<long long>(bytes / (static_cast<unsigned long long>(world) * kSliceBytes)) + 1;
  return align_up(kCountersOff + max_slots * kUnitsPerSlice * 4);
}

struct Layout {
  int tiles_m, tiles_n, n_slices, slots;
  long long recv_off, y_off, total;
};

// Every rank: [control][recv: world x slots slices][y: M x N bf16].  Slice s
// (= tile * 4 + warp) belongs to rank s % world at slot s / world; rank q's
// partial of it lands at recv + (q * slots + slot) * kSliceBytes.
inline Layout layout(long long M, long long N, int world, unsigned long long bytes) {
  Layout L;
  L.tiles_m = static_cast<int>((M + BM - 1) / BM);
  L.tiles_n = static_cast<int>(N / BN);
  L.n_slices = L.tiles_m * L.tiles_n * kUnitsPerSlice;
  L.slots = (L.n_slices + world - 1) / world;
  L.recv_off = control_bytes(bytes, world);
  L.y_off = align_up(L.recv_off + static_cast<long long>(world) * L.slots * kSliceBytes);
  L.total = L.y_off + M * N * 2;
  return L;
}
}  // namespace ar

struct ArParams {
  uint8_t* base[MCPU_SYMM_MAX_RANKS];  // every rank's window, as mapped here
  int rank, world;
  int slots;
  unsigned int units_total;           // units of the whole problem = done target
  long long recv_off, y_off;
};

struct Params {
  int M, N, K;       // N = columns of B (for SwiGLU: 2 x output columns)
  void* C;           // bf16 [M, ldc]
  long long ldc;     // elements
  const void* bias;  // bf16 [N] for kBias
  int epilogue;
  int tiles_m, tiles_n;
  ArParams ar;       // kAR only
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

static_assert(sizeof(Smem) <= 256, "barrier block overflows its slot");
constexpr int SMEM_BYTES_AR = SMEM_BYTES + ar::kStagingBytes;

__device__ __forceinline__ void add_bf16x8(float (&a)[8], const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a[2 * j] = __fadd_rn(a[2 * j], __uint_as_float(w[j] << 16));
    a[2 * j + 1] = __fadd_rn(a[2 * j + 1], __uint_as_float(w[j] & 0xFFFF0000u));
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&a)[8]) {
  return make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                    pack_bf16x2(a[6], a[7]));
}

// One unit of phase B: rows [row0, row0 + 8) x 256 columns.  Every rank's
// bf16 partial of those rows is read from this rank's slots (RB rows x WMAX
// ranks = 16 loads of 16 bytes in flight per lane), summed in fp32 in rank
// order, rounded once and stored into every rank's output (own copy first).
template <int WMAX>
__device__ __forceinline__ void ar_reduce_unit(const Params& p, const uint8_t* src, long long src_stride,
                                               long long row0, long long col_bytes) {
  using namespace ar;
  constexpr int RB = (16 / WMAX) < kUnitRows ? (16 / WMAX) : kUnitRows;
  const int world = p.ar.world, rank = p.ar.rank;
  const long long ypitch = static_cast<long long>(p.N) * 2;
#pragma unroll 1
  for (int r0 = 0; r0 < kUnitRows; r0 += RB) {
    uint4 v[RB][WMAX];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
#pragma unroll
      for (int q = 0; q < WMAX; ++q)
        if (q < world) v[i][q] = peer::ld_cg_v4(src + q * src_stride + (r0 + i) * kRowBytes);
    }
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < WMAX; ++q)
        if (q < world) add_bf16x8(a, v[i][q]);
      const uint4 o = pack_bf16x8(a);
      const long long g = row0 + r0 + i;
      if (g < p.M) {
        for (int d = 0; d < world; ++d) {
          const int dr = rank + d < world ? rank + d : rank + d - world;
          peer::st_v4(p.ar.base[dr] + p.ar.y_off + col_bytes + g * ypitch, o);
        }
      }
    }
  }
}

// Phase B for one reducer warp (rslot of nr per CTA), running from the
// start of the launch beside the GEMM: takes this rank's units in order,
// waits until all ranks' partials of each have arrived, reduces and
// broadcasts it; then one fence and one done increment per rank for all
// its units.  One thread of the grid then waits until this rank's output
// is complete.
__device__ __forceinline__ void ar_reducer(const Params& p, int rslot, int nr, int lane) {
  using namespace ar;
  const int world = p.ar.world, rank = p.ar.rank;
  uint32_t* counters = reinterpret_cast<uint32_t*>(p.ar.base[rank] + kCountersOff);
  const long long src_stride = static_cast<long long>(p.ar.slots) * kSliceBytes;
  const int n_slices = p.tiles_m * p.tiles_n * kUnitsPerSlice;
  const int units = p.ar.slots * kUnitsPerSlice;
  bool ok = true;
  uint32_t processed = 0;
  for (int k = blockIdx.x * nr + rslot; k < units; k += gridDim.x * nr) {
    const int slot = k / kUnitsPerSlice, sub = k % kUnitsPerSlice;
    const int sidx = slot * world + rank;
    if (sidx >= n_slices) break;  // k only grows
    uint32_t got = 1;
    if (lane == 0) {
      got = peer::wait_geq_sys(counters + k, static_cast<uint32_t>(world)) ? 1u : 0u;
      if (got) peer::st_relaxed_sys(counters + k, 0u);
    }
    got = __shfl_sync(0xFFFFFFFFu, got, 0);
    __syncwarp();  // orders lane 0's acquire before the other lanes' loads
    if (!got) {
      ok = false;
      break;
    }
    const int t = sidx / kUnitsPerSlice, ws = sidx % kUnitsPerSlice;
    const long long row0 = static_cast<long long>(t % p.tiles_m) * BM + ws * kSliceRows + sub * kUnitRows;
    const long long col_bytes = static_cast<long long>(t / p.tiles_m) * BN * 2 + lane * 16;
    const uint8_t* src = p.ar.base[rank] + p.ar.recv_off + slot * kSliceBytes + sub * kUnitBytes + lane * 16;
    if (world <= 2)  // two instances only: more make the kernel spill
      ar_reduce_unit<2>(p, src, src_stride, row0, col_bytes);
    else
      ar_reduce_unit<8>(p, src, src_stride, row0, col_bytes);
    ++processed;
  }
  if (processed) {
    // the warp barrier orders every lane's stores before the signalling
    // lanes' release (release is cumulative): no per-lane system fence
    __syncwarp();
    if (lane < world) peer::red_add_release_sys(reinterpret_cast<uint32_t*>(p.ar.base[lane]), processed);
  }
  if (!ok) {
    if (lane == 0) atomicOr(&g_error, 2);
    return;
  }
  if (blockIdx.x == 0 && rslot == 0 && lane == 0) {
    uint32_t* done = reinterpret_cast<uint32_t*>(p.ar.base[rank]);
    if (peer::wait_geq_sys(done, p.ar.units_total))
      peer::st_relaxed_sys(done, 0u);
    else
      atomicOr(&g_error, 2);
  }
}

template <bool kAR>
__global__ void __launch_bounds__(kAR ? THREADS_AR : THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* tiles = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  Smem* s = reinterpret_cast<Smem*>(tiles + STAGES * STAGE_BYTES);
  uint8_t* staging = tiles + STAGES * STAGE_BYTES + 256;  // kAR only
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
  } else if (warp >= 2 && warp < 6) {
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
      if constexpr (kAR) {
        using namespace ar;
        // this warp's 32 rows of the tile are slice t*4+slice, owned by rank
        // (t*4+slice) % world; rows past M are zeros (TMA fill) and are sent
        // all the same, the owner skips them
        const int sidx = t * kUnitsPerSlice + slice;
        const int owner = sidx % p.ar.world, slot = sidx / p.ar.world;
        uint8_t* dst = p.ar.base[owner] + p.ar.recv_off +
                       (static_cast<long long>(p.ar.rank) * p.ar.slots + slot) * kSliceBytes;
        uint8_t* stg = staging + slice * (kSliceRows * 128);
        (void)row_ok;
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          uint32_t r0[32], r1[32];
          tmem_ld32(tbase + c, r0);
          tmem_ld32(tbase + c + 32, r1);
          tmem_ld_wait();
          // lane = row: 64 bf16 as eight 16-byte vectors, vector index XOR
          // row so the 8 lanes of a shared-memory phase hit distinct banks
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((q ^ (lane & 7)) << 4)) =
                make_uint4(pack_bf16x2(__uint_as_float(r0[8 * q]), __uint_as_float(r0[8 * q + 1])),
                           pack_bf16x2(__uint_as_float(r0[8 * q + 2]), __uint_as_float(r0[8 * q + 3])),
                           pack_bf16x2(__uint_as_float(r0[8 * q + 4]), __uint_as_float(r0[8 * q + 5])),
                           pack_bf16x2(__uint_as_float(r0[8 * q + 6]), __uint_as_float(r0[8 * q + 7])));
            *reinterpret_cast<uint4*>(stg + lane * 128 + (((q + 4) ^ (lane & 7)) << 4)) =
                make_uint4(pack_bf16x2(__uint_as_float(r1[8 * q]), __uint_as_float(r1[8 * q + 1])),
                           pack_bf16x2(__uint_as_float(r1[8 * q + 2]), __uint_as_float(r1[8 * q + 3])),
                           pack_bf16x2(__uint_as_float(r1[8 * q + 4]), __uint_as_float(r1[8 * q + 5])),
                           pack_bf16x2(__uint_as_float(r1[8 * q + 6]), __uint_as_float(r1[8 * q + 7])));
          }
          __syncwarp();
          // 8 lanes per row: each store instruction writes four whole
          // 128-byte lines of the owner's slot
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int row = i * 4 + (lane >> 3), cq = lane & 7;
            const uint4 v = *reinterpret_cast<const uint4*>(stg + row * 128 + ((cq ^ (row & 7)) << 4));
            peer::st_v4(dst + row * kRowBytes + (c >> 6) * 128 + cq * 16, v);
          }
          __syncwarp();
        }
        tc_fence_before();
        mbar_arrive(&s->tmem_empty[acc]);
        // every lane's stores are ordered before the signalling lanes'
        // release by the warp barrier (release is cumulative)
        __syncwarp();
        if (lane < kUnitsPerSlice)
          peer::red_add_release_sys(
              reinterpret_cast<uint32_t*>(p.ar.base[owner] + kCountersOff) + slot * kUnitsPerSlice + lane, 1u);
        continue;
      }
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
  } else if (kAR && warp >= 6) {
    // ------------------------------------------------ reducers (kAR)
    ar_reducer(p, warp - 6, REDUCER_WARPS, lane);
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
  MCPU_CUDA_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_bf16_kernel<false>), SMEM_BYTES),
                "mm shared-memory attribute");
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
  gemm_bf16_kernel<false><<<ctas, THREADS, SMEM_BYTES, st>>>(ta, tb, p);
  return from_cuda(cudaGetLastError(), "mm launch");
}

// C = sum over ranks of A_r . B_r^T into every rank's window (kAR).
orError_t launch_allreduce(const void* A, const void* B, long long M, long long N, long long K,
                           const mcpuSymmWindow* w, void** out, cudaStream_t st) {
  MCPU_ARG_CHECK(w != nullptr && out != nullptr, "mm_allreduce: NULL window or output slot");
  MCPU_ARG_CHECK(w->world >= 1 && w->world <= MCPU_SYMM_MAX_RANKS, "mm_allreduce: world %d outside 1..%d",
                 w->world, MCPU_SYMM_MAX_RANKS);
  MCPU_ARG_CHECK(w->rank >= 0 && w->rank < w->world, "mm_allreduce: rank %d outside 0..%d", w->rank,
                 w->world - 1);
  for (int r = 0; r < w->world; ++r)
    MCPU_ARG_CHECK(w->base[r] != nullptr && reinterpret_cast<uintptr_t>(w->base[r]) % 256 == 0,
                   "mm_allreduce: window of rank %d is NULL or not 256-byte aligned", r);
  MCPU_ARG_CHECK(M > 0 && N > 0 && K > 0, "mm_allreduce: M, N and K must be positive");
  MCPU_ARG_CHECK(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), "mm_allreduce: dimension too large");
  MCPU_ARG_CHECK(N % BN == 0, "mm_allreduce: N (%lld) must be a multiple of %d", N, BN);
  MCPU_ARG_CHECK(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(B) % 16 == 0,
                 "mm_allreduce: operands must be 16-byte aligned");
  MCPU_ARG_CHECK((K * 2) % 16 == 0, "mm_allreduce: K must be a multiple of 8 (TMA stride rule)");
  const ar::Layout L = ar::layout(M, N, w->world, w->bytes);
  MCPU_ARG_CHECK(static_cast<unsigned long long>(L.total) <= w->bytes,
                 "mm_allreduce: the window holds %llu bytes, an %lld x %lld output over %d ranks needs %lld",
                 static_cast<unsigned long long>(w->bytes), M, N, w->world, L.total);
  MCPU_ARG_CHECK(static_cast<long long>(L.n_slices) * ar::kUnitsPerSlice < (1LL << 31),
                 "mm_allreduce: too many units");
  CUtensorMap ta, tb;
  orError_t e = make_map(&ta, A, M, K, K, BM);
  if (e != orSuccess) return e;
  e = make_map(&tb, B, N, K, K, BN);
  if (e != orSuccess) return e;
  MCPU_CUDA_TRY(ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_bf16_kernel<true>), SMEM_BYTES_AR),
                "mm_allreduce shared-memory attribute");
  int per_sm = 0;
  MCPU_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_bf16_kernel<true>, THREADS_AR,
                                                              SMEM_BYTES_AR),
                "mm_allreduce occupancy");
  MCPU_ARG_CHECK(per_sm >= 1, "mm_allreduce: the kernel does not fit on an SM");
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = nullptr;
  p.ldc = N;
  p.bias = nullptr;
  p.epilogue = kPlain;
  p.tiles_m = L.tiles_m;
  p.tiles_n = L.tiles_n;
  for (int r = 0; r < MCPU_SYMM_MAX_RANKS; ++r)
    p.ar.base[r] = r < w->world ? static_cast<uint8_t*>(w->base[r]) : nullptr;
  p.ar.rank = w->rank;
  p.ar.world = w->world;
  p.ar.slots = L.slots;
  p.ar.units_total = static_cast<unsigned int>(L.n_slices * ar::kUnitsPerSlice);
  p.ar.recv_off = L.recv_off;
  p.ar.y_off = L.y_off;
  // one CTA per SM, all resident (cooperative): phase B of a CTA waits on
  // phase A of CTAs here and on the other ranks
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(THREADS_AR);
  cfg.dynamicSmemBytes = SMEM_BYTES_AR;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MCPU_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<true>, ta, tb, p), "mm_allreduce launch");
  *out = static_cast<uint8_t*>(w->base[w->rank]) + L.y_off;
  return orSuccess;
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

extern "C" orError_t mcpu_mm_allreduce(const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                                       int dtype, const mcpuSymmWindow* window, void** out,
                                       orStream_t stream) {
  MCPU_ARG_CHECK(dtype == MCPU_BFLOAT16, "mm_allreduce: only bfloat16 is supported (dtype code %d)", dtype);
  MCPU_ARG_CHECK(a && b, "mm_allreduce: NULL tensor pointer");
  return gemm::launch_allreduce(a, b, M, N, K, window, out, as_cuda(stream));
}

extern "C" orError_t mcpu_mm_allreduce_window_bytes(int64_t M, int64_t N, int world, uint64_t* bytes) {
  MCPU_ARG_CHECK(bytes != nullptr, "mm_allreduce_window_bytes: NULL output");
  MCPU_ARG_CHECK(M > 0 && N > 0 && N % gemm::BN == 0, "mm_allreduce_window_bytes: bad M, N");
  MCPU_ARG_CHECK(world >= 1 && world <= MCPU_SYMM_MAX_RANKS, "mm_allreduce_window_bytes: bad world");
  // the control block grows with the window: iterate to a size that holds
  // the layout computed for itself
  unsigned long long b = 0;
  for (int i = 0; i < 64; ++i) {
    const long long need = gemm::ar::layout(M, N, world, b).total;
    if (static_cast<unsigned long long>(need) <= b) break;
    b = static_cast<unsigned long long>(gemm::ar::align_up(need));
  }
  *bytes = b;
  return orSuccess;
}

extern "C" orError_t mcpu_mm_allreduce_control_bytes(uint64_t bytes, int world, uint64_t* control_bytes) {
  MCPU_ARG_CHECK(control_bytes != nullptr, "mm_allreduce_control_bytes: NULL output");
  MCPU_ARG_CHECK(world >= 1 && world <= MCPU_SYMM_MAX_RANKS, "mm_allreduce_control_bytes: bad world");
  *control_bytes = static_cast<uint64_t>(gemm::ar::control_bytes(bytes, world));
  return orSuccess;
}

orError_t gemm::read_error(int* flag, bool reset) {
  MCPU_CUDA_TRY(cudaMemcpyFromSymbol(flag, gemm::g_error, sizeof(int)), "gemm error flag");
  if (reset) {
    const int zero = 0;
    MCPU_CUDA_TRY(cudaMemcpyToSymbol(gemm::g_error, &zero, sizeof(int)), "gemm error flag reset");
  }
  return orSuccess;
}
