// grouped_topk: specialised TMA-fed kernel + exact worklist kernel
// (included by grouped_topk.cu).
//
// Hot kernel.  A G-lane segment serves one token (G a compile-time power of
// two); a 128-thread CTA holds 128/G tokens per tile and loops over tiles
// persistently while one thread keeps a 2-stage TMA ring of [128/G, E] tiles
// filled.  Lane g of a segment owns group g.  The expert pick works on the
// candidate list (keys >= L0 - delta, see grouped_topk_tma.cuh) ranked by
// direct comparison.  A token whose fast result cannot be certified, or whose
// candidate list overflows, is appended to a worklist and left to the exact
// kernel; the hot kernel itself carries no exact-arithmetic code.
//
// Exact kernel.  One warp per worklist row: exact keys (correctly rounded
// sigmoid, or the exact softmax definition), group pick and k rounds of warp
// argmax, all through per-warp shared memory.  It is launched right behind the
// hot kernel with programmatic dependent launch and waits on the hot kernel's
// completion (griddepcontrol.wait) before reading the worklist; the last CTA
// to finish resets the worklist counter for the next call on the stream.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kHotThreads = 128;
constexpr int kHotStages = 2;
constexpr int kCandStride = kCap + 1;  // padded: segments of a warp hit distinct banks

struct Worklist {
  int* count;         // rows appended by the hot kernel
  unsigned* done;     // CTA ticket of the exact kernel
  int* rows;          // capacity >= num_tokens
};

struct HotLayout {
  int tile_bytes, bias_off, ck_off, ci_off, selk_off, seli_off, wbuf_off, ninth_off, bar_off, total;
};

__host__ __device__ inline HotLayout hot_layout(int tpt, int E, int esz) {
  HotLayout L;
  L.tile_bytes = (tpt * E * esz + 1023) & ~1023;
  int off = kHotStages * L.tile_bytes;
  L.bias_off = off;
  off += (E * 4 + 15) & ~15;
  L.ck_off = off;
  off += tpt * kCandStride * 4;
  L.ci_off = off;
  off += ((tpt * kCandStride * 2) + 15) & ~15;
  L.selk_off = off;
  off += tpt * (kMaxK + 1) * 4;
  L.seli_off = off;
  off += tpt * (kMaxK + 1) * 4;
  L.wbuf_off = off;
  off += tpt * (kMaxK + 1) * 4;
  L.ninth_off = off;
  off += ((tpt * 4) + 15) & ~15;
  L.bar_off = off;
  off += kHotStages * 8 + 16;
  L.total = off + 1024;
  return L;
}

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename InT, int G, int GS_MAX, bool kFast>
__global__ void __launch_bounds__(kHotThreads, 4) grouped_topk_hot_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const int tiles, const Worklist wl) {
  constexpr bool kBf16 = sizeof(InT) == 2;
  constexpr int VE = 16 / sizeof(InT);
  constexpr int NCH_MAX = (GS_MAX + VE - 1) / VE;
  constexpr int TPT = kHotThreads / G;
  constexpr unsigned kSegBits = (G == 32) ? 0xFFFFFFFFu : ((1u << G) - 1u);

  pdl_launch_dependents();  // the exact kernel may be scheduled now; it waits for us

  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (ra & 1023)) & 1023);
  const HotLayout L = hot_layout(TPT, p.E, sizeof(InT));
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  float* ck = reinterpret_cast<float*>(base + L.ck_off);
  uint16_t* ci = reinterpret_cast<uint16_t*>(base + L.ci_off);
  float* selk = reinterpret_cast<float*>(base + L.selk_off);
  int* seli = reinterpret_cast<int*>(base + L.seli_off);
  float* wbuf = reinterpret_cast<float*>(base + L.wbuf_off);
  float* ninth = reinterpret_cast<float*>(base + L.ninth_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_off);
  int* abort_flag = reinterpret_cast<int*>(base + L.bar_off + kHotStages * 8);

  const int GS = p.GS, K = p.K, E = p.E, TG = p.TG;
  const int lane = threadIdx.x & 31;
  const int tok = threadIdx.x / G;
  const int g = threadIdx.x & (G - 1);
  const unsigned segmask = kSegBits << (lane & ~(G - 1));
  const bool has_bias = p.bias != nullptr;
  const int box_bytes = TPT * E * static_cast<int>(sizeof(InT));
  const int nch = GS / VE;
  const int gshift = g % (nch > 0 ? nch : 1);
  const bool vec_layout = (GS % VE) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHotStages; ++s) sm100::mbar_init(&full[s], 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&tm);
  }
  for (int i = threadIdx.x; i < E; i += blockDim.x) sbias[i] = has_bias ? p.bias[i] : 0.0f;
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.x < tiles) {
    sm100::mbar_arrive_expect_tx(&full[0], box_bytes);
    sm100::tma_load_2d(base, &tm, &full[0], 0, blockIdx.x * TPT);
  }

  int i = 0;
  for (;; ++i) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= tiles) break;
    const int st = i & 1;
    if (threadIdx.x == 0) {
      const int tn = t + gridDim.x;
      if (tn < tiles) {
        sm100::mbar_arrive_expect_tx(&full[st ^ 1], box_bytes);
        sm100::tma_load_2d(base + (st ^ 1) * L.tile_bytes, &tm, &full[st ^ 1], 0, tn * TPT);
      }
    }
    if (!sm100::mbar_wait(&full[st], (i >> 1) & 1, abort_flag)) break;

    const long long token = static_cast<long long>(t) * TPT + tok;
    const bool valid = token < p.T;
    const InT* row = reinterpret_cast<const InT*>(base + st * L.tile_bytes) + tok * E;
    const InT* grp = row + g * GS;
    const float* bgrp = sbias + g * GS;

    float row_max = 0.0f, row_sum = 1.0f;
    if (p.scoring == MCPU_SCORING_SOFTMAX) {
      float m = -INFINITY;
      for (int j = 0; j < GS; ++j) m = fmaxf(m, smem_elem<InT>(grp, j));
#pragma unroll
      for (int off = 1; off < G; off <<= 1) m = fmaxf(m, __shfl_xor_sync(segmask, m, off, G));
      row_max = m;
      float sum = 0.0f;
      for (int j = 0; j < GS; ++j) sum = __fadd_rn(sum, expf(smem_elem<InT>(grp, j) - row_max));
#pragma unroll
      for (int off = 1; off < G; off <<= 1) sum = __fadd_rn(sum, __shfl_xor_sync(segmask, sum, off, G));
      row_sum = sum;
    }

    // ---- keys + the group's two best, chunk by chunk from shared memory
    float key[GS_MAX];
    float m1 = -INFINITY, m2 = -INFINITY;
    if (vec_layout) {
#pragma unroll
      for (int c = 0; c < NCH_MAX; ++c) {
        int cc = c + gshift;
        if (cc >= nch) cc -= nch;
        float xv[VE], bv[VE];
        if (c < nch) {
          const uint4 raw = *reinterpret_cast<const uint4*>(grp + cc * VE);
          if constexpr (kBf16) {
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              xv[2 * q] = __uint_as_float(w[q] << 16);
              xv[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
            }
          } else {
            xv[0] = __uint_as_float(raw.x);
            xv[1] = __uint_as_float(raw.y);
            xv[2] = __uint_as_float(raw.z);
            xv[3] = __uint_as_float(raw.w);
          }
#pragma unroll
          for (int q = 0; q < VE; q += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(bgrp + cc * VE + q);
            bv[q] = b4.x;
            bv[q + 1] = b4.y;
            bv[q + 2] = b4.z;
            bv[q + 3] = b4.w;
          }
        }
#pragma unroll
        for (int q = 0; q < VE; ++q) {
          const int s = c * VE + q;
          if (s >= GS_MAX) continue;
          float k = -INFINITY;
          if (c < nch) {
            if constexpr (kFast) {
              k = fast_key(xv[q], bv[q]);
            } else if (has_bias) {
              float sc = p.scoring == MCPU_SCORING_SIGMOID
                             ? sigmoid_exact_call(xv[q])
                             : __fdiv_rn(expf(xv[q] - row_max), row_sum);
              if (kBf16) sc = round_bf16(sc);
              k = __fadd_rn(sc, bv[q]);
            } else {
              k = xv[q];
            }
          }
          key[s] = k;
          m2 = fmaxf(m2, fminf(m1, k));
          m1 = fmaxf(m1, k);
        }
      }
    } else {
#pragma unroll
      for (int s = 0; s < GS_MAX; ++s) {
        float k = -INFINITY;
        if (s < GS) {
          const float xv = smem_elem<InT>(grp, s), bv = bgrp[s];
          if constexpr (kFast) {
            k = fast_key(xv, bv);
          } else if (has_bias) {
            float sc = p.scoring == MCPU_SCORING_SIGMOID ? sigmoid_exact_call(xv)
                                                         : __fdiv_rn(expf(xv - row_max), row_sum);
            if (kBf16) sc = round_bf16(sc);
            k = __fadd_rn(sc, bv);
          } else {
            k = xv;
          }
        }
        key[s] = k;
        m2 = fmaxf(m2, fminf(m1, k));
        m1 = fmaxf(m1, k);
      }
    }
    auto local_of = [&](int s) -> int {
      if (!vec_layout) return s;
      const int c = s / VE;
      int cc = c + gshift;
      if (cc >= nch) cc -= nch;
      return cc * VE + (s - c * VE);
    };

    // ---- group pick (ties to the lower group index)
    const float gs = has_bias ? __fadd_rn(m1, m2) : m1;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const float o = __shfl_sync(segmask, gs, j, G);
      rank += (o > gs) || (o == gs && j < g);
    }
    const bool gsel = rank < TG;
    bool ok = true;
    if constexpr (kFast) {
      float lo = gsel ? gs : INFINITY, hi = gsel ? -INFINITY : gs;
#pragma unroll
      for (int off = 1; off < G; off <<= 1) {
        lo = fminf(lo, __shfl_xor_sync(segmask, lo, off, G));
        hi = fmaxf(hi, __shfl_xor_sync(segmask, hi, off, G));
      }
      if (hi != -INFINITY) ok = (lo - hi) > (0x1p-18f + 0x1p-19f * fmaxf(fabsf(lo), fabsf(hi)));
    }

    // ---- candidates: keys >= L0 - delta in the selected groups
    float l0 = gsel ? m2 : INFINITY;
#pragma unroll
    for (int off = 1; off < G; off <<= 1) l0 = fminf(l0, __shfl_xor_sync(segmask, l0, off, G));
    if (!(GS >= 2 && 2 * TG >= K)) l0 = -INFINITY;
    const float thr = kFast ? l0 - (0x1p-19f + 0x1p-20f * fabsf(l0)) : l0;
    int c = 0;
#pragma unroll
    for (int s = 0; s < GS_MAX; ++s) c += (gsel && key[s] >= thr) ? 1 : 0;
    int incl = c;
#pragma unroll
    for (int off = 1; off < G; off <<= 1) {
      const int o = __shfl_up_sync(segmask, incl, off, G);
      if (g >= off) incl += o;
    }
    const int C = __shfl_sync(segmask, incl, G - 1, G);
    float* tck = ck + tok * kCandStride;
    uint16_t* tci = ci + tok * kCandStride;
    float* tsk = selk + tok * (kMaxK + 1);
    int* tsi = seli + tok * (kMaxK + 1);
    const bool fits = C <= kCap;
    if (fits) {
      int pos = incl - c;
#pragma unroll
      for (int s = 0; s < GS_MAX; ++s) {
        if (gsel && key[s] >= thr) {
          tck[pos] = key[s];
          tci[pos] = static_cast<uint16_t>(g * GS + local_of(s));
          ++pos;
        }
      }
      __syncwarp(segmask);
      for (int q = g; q < C; q += G) {
        const float v = tck[q];
        const int iv = tci[q];
        int r = 0;
        for (int k2 = 0; k2 < C; ++k2) r += ranks_before(tck[k2], tci[k2], v, iv) ? 1 : 0;
        if (r < K) {
          tsk[r] = v;
          tsi[r] = iv;
        } else if (r == K) {
          ninth[tok] = v;
        }
      }
      __syncwarp(segmask);
      if (kFast && C > K) {
        const float k8 = tsk[K - 1], k9 = ninth[tok];
        ok = ok && (k8 - k9) > (0x1p-19f + 0x1p-20f * fmaxf(fabsf(k8), fabsf(k9)));
      }
    }
    const bool certified = fits && ok;

    if (!certified) {
      if (g == 0 && valid) wl.rows[atomicAdd(wl.count, 1)] = static_cast<int>(token);
    } else {
      float* tw = wbuf + tok * (kMaxK + 1);
      for (int k = g; k < K; k += G) {
        const float xv = smem_elem<InT>(row, tsi[k]);
        float sc;
        if (p.scoring == MCPU_SCORING_SIGMOID)
          sc = kFast ? sigmoid_accurate(xv) : sigmoid_exact_call(xv);
        else
          sc = __fdiv_rn(expf(xv - row_max), row_sum);
        tw[k] = kBf16 ? round_bf16(sc) : sc;
      }
      __syncwarp(segmask);
      float sum = 0.0f;
      if (p.renorm) {
        for (int k = 0; k < K; ++k) sum = __fadd_rn(sum, tw[k]);
        if (kBf16) sum = round_bf16(sum);
      }
      if (valid) {
        for (int k = g; k < K; k += G) {
          float w = tw[k];
          if (p.renorm) {
            w = __fdiv_rn(w, sum);
            if (kBf16) w = round_bf16(w);
          }
          if (p.scale != 1.0f) {
            w = __fmul_rn(w, p.scale);
            if (kBf16) w = round_bf16(w);
          }
          p.w_out[token * K + k] = w;
          p.id_out[token * K + k] = tsi[k];
        }
      }
    }
    __syncthreads();
  }

  if (threadIdx.x == 0 && *abort_flag) {
    // a wait ran out: record it, then let the copies this CTA issued land
    atomicExch(&g_router_error, 1);
    for (int j = i; j <= i + 1; ++j) {
      if (blockIdx.x + j * gridDim.x >= tiles) continue;
      for (uint32_t n = 0; n < sm100::kSpinLimit && !sm100::mbar_try_wait(&full[j & 1], (j >> 1) & 1);
           ++n) {
      }
    }
  }
}

// ------------------------------------------------------------------ exact kernel
constexpr int kExactWarps = 4;

template <typename InT>
__global__ void __launch_bounds__(kExactWarps * 32) grouped_topk_exact_kernel(const Params p,
                                                                             const Worklist wl) {
  extern __shared__ float xsm[];  // per warp: key[E], score[E], gsc[G]
  pdl_wait();                      // the hot kernel's worklist is complete and visible
  constexpr bool kBf16 = sizeof(InT) == 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.E, G = p.G, GS = p.GS, K = p.K;
  float* skey = xsm + warp * (2 * E + G);
  float* ssc = skey + E;
  float* sgs = ssc + E;
  const int n = *reinterpret_cast<volatile int*>(wl.count);
  const int nwarps = gridDim.x * kExactWarps;
  const bool has_bias = p.bias != nullptr;
  for (int item = blockIdx.x * kExactWarps + warp; item < n; item += nwarps) {
    const long long token = wl.rows[item];
    const InT* row = reinterpret_cast<const InT*>(p.gating) + token * E;
    float row_max = 0.0f, row_sum = 1.0f;
    if (p.scoring == MCPU_SCORING_SOFTMAX) {
      float m = -INFINITY;
      for (int e = lane; e < E; e += 32) m = fmaxf(m, load_one<InT>(row + e));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
      row_max = m;
      // fixed summation order: lane-strided partial sums, then a fixed tree
      float s = 0.0f;
      for (int e = lane; e < E; e += 32) s = __fadd_rn(s, expf(load_one<InT>(row + e) - row_max));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, off));
      row_sum = s;
    }
    for (int e = lane; e < E; e += 32) {
      const float xv = load_one<InT>(row + e);
      float sc = p.scoring == MCPU_SCORING_SIGMOID ? sigmoid_exact_call(xv)
                                                   : __fdiv_rn(expf(xv - row_max), row_sum);
      if (kBf16) sc = round_bf16(sc);
      ssc[e] = sc;
      skey[e] = has_bias ? __fadd_rn(sc, __ldg(p.bias + e)) : xv;
    }
    __syncwarp();
    for (int gi = lane; gi < G; gi += 32) {
      float m1 = -INFINITY, m2 = -INFINITY;
      for (int j = 0; j < GS; ++j) {
        const float v = skey[gi * GS + j];
        m2 = fmaxf(m2, fminf(m1, v));
        m1 = fmaxf(m1, v);
      }
      sgs[gi] = has_bias ? __fadd_rn(m1, m2) : m1;
    }
    __syncwarp();
    // group pick: rank of each group among all G (ties to the lower index)
    unsigned long long sel_lo = 0;  // bit g: group g selected (G <= 64 supported here)
    for (int gi = lane; gi < G; gi += 32) {
      const float v = sgs[gi];
      int r = 0;
      for (int j = 0; j < G; ++j) r += ranks_before(sgs[j], j, v, gi) ? 1 : 0;
      if (r < p.TG) sel_lo |= 1ull << gi;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sel_lo |= __shfl_xor_sync(0xFFFFFFFFu, sel_lo, off);
    // k rounds of warp argmax over the experts of the selected groups
    float lk = INFINITY;
    int li = -1;
    int ids[kMaxK];
#pragma unroll
    for (int r = 0; r < kMaxK; ++r) ids[r] = 0;
    for (int r = 0; r < K; ++r) {
      float bk = -INFINITY;
      int bi = 0x7FFFFFFF;
      for (int e = lane; e < E; e += 32) {
        if (!((sel_lo >> (e / GS)) & 1ull)) continue;
        const float v = skey[e];
        const bool after = v < lk || (v == lk && e > li);
        if (after && ranks_before(v, e, bk, bi)) {
          bk = v;
          bi = e;
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ok2 = __shfl_xor_sync(0xFFFFFFFFu, bk, off);
        const int oi2 = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
        if (ranks_before(ok2, oi2, bk, bi)) {
          bk = ok2;
          bi = oi2;
        }
      }
#pragma unroll
      for (int q = 0; q < kMaxK; ++q)
        if (q == r) ids[q] = bi;
      lk = bk;
      li = bi;
    }
    if (lane == 0) {
      float w[kMaxK];
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < kMaxK; ++k) {
        w[k] = k < K ? ssc[ids[k]] : 0.0f;
        if (k < K) sum = __fadd_rn(sum, w[k]);
      }
      if (kBf16) sum = round_bf16(sum);
#pragma unroll
      for (int k = 0; k < kMaxK; ++k) {
        if (k >= K) continue;
        float v = w[k];
        if (p.renorm) {
          v = __fdiv_rn(v, sum);
          if (kBf16) v = round_bf16(v);
        }
        if (p.scale != 1.0f) {
          v = __fmul_rn(v, p.scale);
          if (kBf16) v = round_bf16(v);
        }
        p.w_out[token * K + k] = v;
        p.id_out[token * K + k] = ids[k];
      }
      atomicAdd(&g_exact_rows, 1ull);
    }
    __syncwarp();
  }
  // the last CTA to finish resets the worklist for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned ticket = atomicAdd(wl.done, 1u);
    if (ticket == gridDim.x - 1) {
      *wl.count = 0;
      *wl.done = 0u;
      __threadfence();
    }
  }
}

}  // namespace router
}  // namespace mcpu
