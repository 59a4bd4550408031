// grouped_topk: the specialised TMA-fed kernel (included by grouped_topk.cu).
//
// A G-lane segment serves one token (G a compile-time power of two); a
// 128-thread CTA holds 128/G tokens per tile and loops over tiles
// persistently while one thread keeps a 2-stage TMA ring of [128/G, E] tiles
// filled.  Lane g of a segment owns group g and keeps its experts' keys in
// registers.
//
// Expert pick: every selected group contributes its two best experts, so with
// 2 * topk_group >= topk the k-th best candidate is at least L0 = min over
// selected groups of the group's second-best key; only keys >= L0 - delta can
// be among the top k.  Each lane marks those slots in a 32-bit mask, writes
// them (as 64-bit packed value/index keys) to the token's list in shared
// memory, and every candidate is ranked by direct comparison.
//
// Exactness (fp32 sigmoid + bias): the fast keys are within eps(|key|) =
// 2^-21 + 2^-22 |key| of the exact ones.  When both selection margins exceed
// 4 eps the fast pick is provably the exact pick.  Otherwise the row is
// refined in place: exact keys are computed only for the experts that can
// still matter (within 4 eps of a group's second best, to get exact group
// scores, and the candidate list), and the pick is redone on exact keys.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kHotThreads = 128;
constexpr int kHotStages = 2;
constexpr int kCandStride = kCap + 1;  // padded: the segments of a warp hit distinct banks

struct HotLayout {
  int tile_bytes, bias_off, cand_off, sel_off, wbuf_off, bar_off, total;
};

__host__ __device__ inline HotLayout hot_layout(int tpt, int E, int esz) {
  HotLayout L;
  L.tile_bytes = (tpt * E * esz + 1023) & ~1023;
  int off = kHotStages * L.tile_bytes;
  L.bias_off = off;
  off += (E * 4 + 15) & ~15;
  L.cand_off = off;
  off += tpt * kCandStride * 8;
  L.sel_off = off;
  off += tpt * (kMaxK + 1) * 8;
  L.wbuf_off = off;
  off += ((tpt * (kMaxK + 1) * 4) + 15) & ~15;
  L.bar_off = off;
  off += kHotStages * 8 + 16;
  L.total = off + 1024;
  return L;
}

__device__ __forceinline__ unsigned long long pack_key(float f, int idx) {
  return (static_cast<unsigned long long>(orderable(f)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ int packed_index(unsigned long long k) {
  return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k));
}
__device__ __forceinline__ float packed_value(unsigned long long k) {
  const uint32_t u = static_cast<uint32_t>(k >> 32);
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

// Error bound of a fast key against the exact one: |fast - exact| <= eps(|key|).
__device__ __forceinline__ float key_eps(float mag) { return 0x1p-21f + 0x1p-22f * mag; }

template <typename InT, int G, int GS_MAX, bool kFast>
__global__ void __launch_bounds__(kHotThreads, 6) grouped_topk_hot_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const int tiles) {
  constexpr bool kBf16 = sizeof(InT) == 2;
  constexpr int VE = 16 / sizeof(InT);
  constexpr int NCH_MAX = (GS_MAX + VE - 1) / VE;
  constexpr int TPT = kHotThreads / G;
  constexpr unsigned kSegBits = (G == 32) ? 0xFFFFFFFFu : ((1u << G) - 1u);
  static_assert(GS_MAX <= 32, "slot masks are 32 bits");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (ra & 1023)) & 1023);
  const HotLayout L = hot_layout(TPT, p.E, sizeof(InT));
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(base + L.cand_off);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(base + L.sel_off);
  float* wbuf = reinterpret_cast<float*>(base + L.wbuf_off);
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
  const bool two_best = GS >= 2 && 2 * TG >= K;

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
    auto live = [&](int s) -> bool { return vec_layout ? (s / VE) < nch : s < GS; };
    auto local_of = [&](int s) -> int {
      if (!vec_layout) return s;
      const int c = s / VE;
      int cc = c + gshift;
      if (cc >= nch) cc -= nch;
      return cc * VE + (s - c * VE);
    };
    // key of local expert j of this lane's group: the ranking key of the
    // kernel's mode, or (exact = true) the exact key
    auto key_of = [&](int j, bool exact) -> float {
      const float xv = smem_elem<InT>(grp, j);
      if (kFast && !exact) return fast_key(xv, bgrp[j]);
      if (!has_bias) return xv;
      float sc = p.scoring == MCPU_SCORING_SIGMOID ? sigmoid_exact_call(xv)
                                                   : __fdiv_rn(expf(xv - row_max), row_sum);
      if (kBf16) sc = round_bf16(sc);
      return __fadd_rn(sc, bgrp[j]);
    };

    // ---- keys (fast, or exact in the exact-key modes) + the group's two best
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
        const float k = s < GS ? key_of(s, !kFast) : -INFINITY;
        key[s] = k;
        m2 = fmaxf(m2, fminf(m1, k));
        m1 = fmaxf(m1, k);
      }
    }

    unsigned long long* tc = cand + tok * kCandStride;
    unsigned long long* ts = sel + tok * (kMaxK + 1);
    bool exact = !kFast;  // are the group scores and candidate keys exact?
    bool slow = false;
#pragma unroll 1
    for (;;) {
      float gsv, m2v;
      if (kFast && exact) {
        // exact two best of this group: only experts whose fast key is within
        // 4 eps of the fast second best can be among the exact two best
        const float lim = m2 - 4.0f * key_eps(fabsf(m2));
        uint32_t near = 0;
#pragma unroll
        for (int s = 0; s < GS_MAX; ++s) near |= (key[s] >= lim) ? (1u << s) : 0u;
        float e1 = -INFINITY, e2 = -INFINITY;
#pragma unroll 1
        for (uint32_t m = near; m; m &= m - 1) {
          const float ke = key_of(local_of(__ffs(m) - 1), true);
          e2 = fmaxf(e2, fminf(e1, ke));
          e1 = fmaxf(e1, ke);
        }
        gsv = __fadd_rn(e1, e2);
        m2v = e2;
      } else {
        gsv = has_bias ? __fadd_rn(m1, m2) : m1;
        m2v = m2;
      }
      // group pick (ties to the lower group index)
      int rank = 0;
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const float o = __shfl_sync(segmask, gsv, j, G);
        rank += (o > gsv) || (o == gsv && j < g);
      }
      const bool gsel = rank < TG;
      bool ok = true;
      if (!exact) {
        float lo = gsel ? gsv : INFINITY, hi = gsel ? -INFINITY : gsv;
#pragma unroll
        for (int off = 1; off < G; off <<= 1) {
          lo = fminf(lo, __shfl_xor_sync(segmask, lo, off, G));
          hi = fmaxf(hi, __shfl_xor_sync(segmask, hi, off, G));
        }
        if (hi != -INFINITY) ok = (lo - hi) > 4.0f * key_eps(fmaxf(fabsf(lo), fabsf(hi)));
      }
      // candidates: keys >= L0 - delta in the selected groups, where
      // L0 = min over selected groups of the second best key
      float l0 = gsel ? m2v : INFINITY;
#pragma unroll
      for (int off = 1; off < G; off <<= 1) l0 = fminf(l0, __shfl_xor_sync(segmask, l0, off, G));
      if (!two_best) l0 = -INFINITY;
      const float thr = kFast ? l0 - 4.0f * key_eps(fabsf(l0)) : l0;
      uint32_t mask = 0;
#pragma unroll
      for (int s = 0; s < GS_MAX; ++s) mask |= (key[s] >= thr) ? (1u << s) : 0u;
      if (!gsel) mask = 0;
      const int c = __popc(mask);
      int incl = c;
#pragma unroll
      for (int off = 1; off < G; off <<= 1) {
        const int o = __shfl_up_sync(segmask, incl, off, G);
        if (g >= off) incl += o;
      }
      const int C = __shfl_sync(segmask, incl, G - 1, G);
      if (C > kCap) {
        if (!exact) {  // many near-equal keys: settle it on exact keys
          exact = true;
          slow = true;
          continue;
        }
        // degenerate input (more than kCap exact near-ties): k rounds of
        // segment argmax over exact keys, evaluated slot by slot
        uint32_t livemask = 0;
#pragma unroll
        for (int s = 0; s < GS_MAX; ++s) livemask |= live(s) ? (1u << s) : 0u;
        if (!gsel) livemask = 0;
        unsigned long long last = ~0ull;
#pragma unroll 1
        for (int r = 0; r < K; ++r) {
          unsigned long long best = 0;
#pragma unroll 1
          for (uint32_t m = livemask; m; m &= m - 1) {
            const int j = local_of(__ffs(m) - 1);
            const unsigned long long pk = pack_key(kFast ? key_of(j, true) : key_of(j, !kFast), g * GS + j);
            if (pk < last && pk > best) best = pk;
          }
#pragma unroll
          for (int off = 1; off < G; off <<= 1) {
            const unsigned long long o = __shfl_xor_sync(segmask, best, off, G);
            best = o > best ? o : best;
          }
          if (g == 0) ts[r] = best;
          last = best;
        }
        __syncwarp(segmask);
        break;
      }
      // write this lane's candidates at its prefix position
      int pos = incl - c;
      for (uint32_t m = mask; m; m &= m - 1) {
        const int j = local_of(__ffs(m) - 1);
        tc[pos++] = pack_key(key_of(j, exact), g * GS + j);
      }
      __syncwarp(segmask);
      // rank every candidate against all others (packed keys: one compare)
      for (int q = g; q < C; q += G) {
        const unsigned long long v = tc[q];
        int r = 0;
        for (int k2 = 0; k2 < C; ++k2) r += tc[k2] > v ? 1 : 0;
        if (r <= K) ts[r] = v;
      }
      __syncwarp(segmask);
      if (!exact) {
        if (C > K) {
          const float k8 = packed_value(ts[K - 1]), k9 = packed_value(ts[K]);
          ok = ok && (k8 - k9) > 4.0f * key_eps(fmaxf(fabsf(k8), fabsf(k9)));
        }
        if (!ok) {
          exact = true;
          slow = true;
          continue;
        }
      }
      break;
    }
    if (slow && g == 0 && valid) atomicAdd(&g_exact_rows, 1ull);

    // ---- weights, renormalisation, scaling, stores
    float* tw = wbuf + tok * (kMaxK + 1);
    for (int k = g; k < K; k += G) {
      const float xv = smem_elem<InT>(row, packed_index(ts[k]));
      float sc;
      if (p.scoring == MCPU_SCORING_SIGMOID)
        sc = (kFast && !slow) ? sigmoid_accurate(xv) : sigmoid_exact_call(xv);
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
        p.id_out[token * K + k] = packed_index(ts[k]);
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

}  // namespace router
}  // namespace mcpu
