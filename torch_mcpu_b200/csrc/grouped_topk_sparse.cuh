// grouped_topk for fp32 logits, sigmoid scoring with a correction bias: the
// sparse-key kernel (included by grouped_topk.cu).
//
// Same tiling as the hot kernel (a G-lane segment per token, lane g owns
// group g, persistent 128-thread CTAs fed by a 2-stage TMA ring), but the
// sigmoid is evaluated only for the experts that can matter.  sigmoid is
// increasing, so from the raw logits alone each lane bounds its group:
//
//   the group's second-best key  >= lb2 = sigmoid(x2) + min bias,
//   the group score (top-2 sum)  in [sigmoid(x1) + sigmoid(x2) + 2 min bias,
//                                    sigmoid(x1) + sigmoid(x2) + 2 max bias]
//
// (x1 >= x2 the group's two largest logits).  A group whose upper bound is
// below topk_group lower bounds of other groups cannot be picked; over the
// others, R = min lb2 bounds the k-th best candidate from below (each picked
// group holds two keys >= its second best).  No expert whose key is below
// min(R, own lb2) can be among its group's two best or among the candidates,
// so each lane keeps only the experts with
//
//   sigmoid(x) + max bias >= min(R, lb2) - margin,  i.e.  x >= logit(...)
//
// (about 4 of 32 for N(0,1) logits) and computes their fast keys into
// registers (kSparseSlots slots; more than that keeps the best ones and
// records the largest key it dropped).  From there the pick is the hot
// kernel's: group pick, candidate list >= L0 - 4 eps, ranking, margin
// certification, and in-place exact refinement of uncertain tokens.  The
// margin (16 times the fast-key error bound) keeps every excluded expert
// below every threshold the exact refinement uses, so the exclusion never
// changes a result.  Tokens with many near-equal keys (dropped keys near a
// threshold, or more than kCap candidates on exact keys) take a fully exact
// pick over all experts.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kSparseThreads = 128;
constexpr int kSparseSlots = 12;
constexpr int kSparseCandStride = 36;  // kCap + 4 zero pads, 16-byte rows

struct SparseLayout {
  int tile_bytes, bias_off, cand_off, sel_off, wbuf_off, bar_off, total;
};

__host__ __device__ inline SparseLayout sparse_layout(int tpt, int E) {
  SparseLayout L;
  L.tile_bytes = (tpt * E * 4 + 1023) & ~1023;
  int off = 2 * L.tile_bytes;
  L.bias_off = off;
  off += (E * 4 + 15) & ~15;
  L.cand_off = off;
  off += tpt * kSparseCandStride * 8;
  L.sel_off = off;
  off += tpt * (kMaxK + 1) * 8;
  L.wbuf_off = off;
  off += ((tpt * (kMaxK + 1) * 4) + 15) & ~15;
  L.bar_off = off;
  off += 2 * 8 + 16;
  L.total = off + 1024;
  return L;
}

// Prefilter margin: 16 times the fast-key error bound key_eps.
__device__ __forceinline__ float pre_margin(float mag) { return 0x1p-17f + 0x1p-18f * mag; }

__device__ __forceinline__ float lg2_approx(float v) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// A t with sigmoid(t) <= y, close to logit(y); -inf when y is tiny or NaN.
// y is first lowered to at most 1 - 2^-16 (a smaller y only lowers t).  The
// approximate logarithms are good to about 2^-21 (1 + |t|); t is lowered by
// 2^-12 (1 + |t|).
__device__ __forceinline__ float logit_floor(float y) {
  if (!(y > 0x1p-60f)) return -INFINITY;
  y = fminf(y, 1.0f - 0x1p-16f);
  const float t = 0.69314718f * (lg2_approx(y) - lg2_approx(1.0f - y));
  return t - 0x1p-12f * (1.0f + fabsf(t));
}

// Exact key of local expert j: the reference's fp32 sigmoid plus the bias.
__device__ __forceinline__ float exact_key(const float* grp, const float* bgrp, int j) {
  return __fadd_rn(sigmoid_exact_call(grp[j]), bgrp[j]);
}

// The whole pick on exact keys over every expert: exact group scores, group
// pick, then k rounds of segment argmax.  For inputs with many near-equal
// keys only; ts[0..K) receives the packed picks.
template <int G, int GS_MAX>
__device__ __noinline__ void sparse_full_exact(const float* grp, const float* bgrp, int g, int GS,
                                               int TG, int K, unsigned segmask,
                                               unsigned long long* ts) {
  float k[GS_MAX];
  float e1 = -INFINITY, e2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < GS_MAX; ++j) {
    k[j] = j < GS ? exact_key(grp, bgrp, j) : -INFINITY;
    e2 = fmaxf(e2, fminf(e1, k[j]));
    e1 = fmaxf(e1, k[j]);
  }
  const float gsv = __fadd_rn(e1, e2);
  int rank = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const float o = __shfl_sync(segmask, gsv, j, G);
    rank += (o > gsv) || (o == gsv && j < g);
  }
  const bool gsel = rank < TG;
  unsigned long long last = ~0ull;
  for (int r = 0; r < K; ++r) {
    unsigned long long best = 0;
    if (gsel) {
#pragma unroll
      for (int j = 0; j < GS_MAX; ++j) {
        if (j >= GS) continue;
        const unsigned long long pk = pack_key(k[j], g * GS + j);
        if (pk < last && pk > best) best = pk;
      }
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
}

template <int G, int GS_MAX>
__global__ void __launch_bounds__(kSparseThreads, 5) grouped_topk_sparse_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const int tiles) {
  constexpr int VE = 4;
  constexpr int NCH_MAX = GS_MAX / VE;
  constexpr int TPT = kSparseThreads / G;
  constexpr unsigned kSegBits = (G == 32) ? 0xFFFFFFFFu : ((1u << G) - 1u);
  static_assert(GS_MAX <= 32 && GS_MAX % VE == 0, "slot masks are 32 bits, vectors of 4");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (ra & 1023)) & 1023);
  const SparseLayout L = sparse_layout(TPT, p.E);
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(base + L.cand_off);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(base + L.sel_off);
  float* wbuf = reinterpret_cast<float*>(base + L.wbuf_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_off);
  int* abort_flag = reinterpret_cast<int*>(base + L.bar_off + 2 * 8);

  const int GS = p.GS, K = p.K, E = p.E, TG = p.TG;
  const int lane = threadIdx.x & 31;
  const int tok = threadIdx.x / G;
  const int g = threadIdx.x & (G - 1);
  const unsigned segmask = kSegBits << (lane & ~(G - 1));
  const int box_bytes = TPT * E * 4;
  const int nch = GS / VE;
  const int gshift = g % nch;
  const bool two_best = 2 * TG >= K;
  uint32_t live = 0;
#pragma unroll
  for (int s = 0; s < GS_MAX; ++s) live |= (s < GS) ? (1u << s) : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) sm100::mbar_init(&full[s], 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&tm);
  }
  for (int i = threadIdx.x; i < E; i += blockDim.x) sbias[i] = p.bias[i];
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.x < tiles) {
    sm100::mbar_arrive_expect_tx(&full[0], box_bytes);
    sm100::tma_load_2d(base, &tm, &full[0], 0, blockIdx.x * TPT);
  }
  const float* bgrp = sbias + g * GS;
  float bmin = INFINITY, bmax = -INFINITY;
  for (int j = 0; j < GS; ++j) {
    bmin = fminf(bmin, bgrp[j]);
    bmax = fmaxf(bmax, bgrp[j]);
  }
  // local index of slot s: the lane's 4-element chunks are visited starting
  // at chunk g so that the lanes of a segment hit distinct banks
  auto local_of = [&](int s) -> int {
    int cc = (s / VE) + gshift;
    if (cc >= nch) cc -= nch;
    return cc * VE + (s & (VE - 1));
  };

  bool ok = true;
  if (blockIdx.x < tiles) ok = sm100::mbar_wait(&full[0], 0, abort_flag);
  int i = 0;
  int last_issued = blockIdx.x < tiles ? 0 : -1;  // ring position of the newest load
  if (!__syncthreads_or(!ok)) {
    for (;; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      if (t >= tiles) break;
      const int st = i & 1;
      const int tn = t + gridDim.x;
      if (tn < tiles) last_issued = i + 1;
      if (threadIdx.x == 0 && tn < tiles) {
        sm100::mbar_arrive_expect_tx(&full[st ^ 1], box_bytes);
        sm100::tma_load_2d(base + (st ^ 1) * L.tile_bytes, &tm, &full[st ^ 1], 0, tn * TPT);
      }

      const long long token = static_cast<long long>(t) * TPT + tok;
      const bool valid = token < p.T;
      const float* row = reinterpret_cast<const float*>(base + st * L.tile_bytes) + tok * E;
      const float* grp = row + g * GS;

      // ---- pass 1: the group's two largest logits, and the bounds
      float xr[GS_MAX];
      float x1 = -INFINITY, x2 = -INFINITY;
#pragma unroll
      for (int c = 0; c < NCH_MAX; ++c) {
        int cc = c + gshift;
        if (cc >= nch) cc -= nch;
        float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        if (c < nch) v = *reinterpret_cast<const float4*>(grp + cc * VE);
        xr[c * 4 + 0] = v.x;
        xr[c * 4 + 1] = v.y;
        xr[c * 4 + 2] = v.z;
        xr[c * 4 + 3] = v.w;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          x2 = fmaxf(x2, fminf(x1, xr[c * 4 + q]));
          x1 = fmaxf(x1, xr[c * 4 + q]);
        }
      }
      const float s1 = sigmoid_fast(x1), s2 = sigmoid_fast(x2);
      const float l2 = __fadd_rn(s2, bmin);
      const float lb2 = l2 - pre_margin(fabsf(l2));
      const float ssum = __fadd_rn(s1, s2);
      const float glo = __fadd_rn(ssum, 2.0f * bmin), ghi = __fadd_rn(ssum, 2.0f * bmax);
      const float lo = glo - 2.0f * pre_margin(fabsf(glo));
      const float hi = ghi + 2.0f * pre_margin(fabsf(ghi));
      int above = 0;  // groups whose score is surely above this group's
#pragma unroll
      for (int j = 0; j < G; ++j) above += __shfl_sync(segmask, lo, j, G) > hi ? 1 : 0;
      float rsel = above < TG ? lb2 : INFINITY;
#pragma unroll
      for (int off = 1; off < G; off <<= 1) rsel = fminf(rsel, __shfl_xor_sync(segmask, rsel, off, G));
      if (!two_best) rsel = -INFINITY;
      const float rr = fminf(lb2, rsel);
      const float y = (rr - bmax) - 2.0f * pre_margin(fabsf(rr) + fabsf(bmax) + 1.0f);
      const float tx = logit_floor(y);
      uint32_t cm = 0;
#pragma unroll
      for (int s = 0; s < GS_MAX; ++s) cm |= (xr[s] >= tx) ? (1u << s) : 0u;
      cm &= live;

      // ---- fast keys of the kept experts, into slots
      float sf[kSparseSlots];
      int sj[kSparseSlots];
#pragma unroll
      for (int c = 0; c < kSparseSlots; ++c) {
        sf[c] = -INFINITY;
        sj[c] = -1;
      }
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int c = 0; c < kSparseSlots; ++c) {
        if (!__any_sync(0xFFFFFFFFu, cm != 0u)) break;
        if (cm) {
          const int j = local_of(__ffs(cm) - 1);
          cm &= cm - 1;
          const float f = fast_key(grp[j], bgrp[j]);
          sf[c] = f;
          sj[c] = j;
          m2 = fmaxf(m2, fminf(m1, f));
          m1 = fmaxf(m1, f);
        }
      }
      float dropf = -INFINITY;  // largest fast key not kept in a slot
      if (__any_sync(0xFFFFFFFFu, cm != 0u)) {
        for (; cm; cm &= cm - 1) {
          const int j = local_of(__ffs(cm) - 1);
          const float f = fast_key(grp[j], bgrp[j]);
          m2 = fmaxf(m2, fminf(m1, f));
          m1 = fmaxf(m1, f);
          unsigned long long mn = ~0ull;
          int mc = 0;
#pragma unroll
          for (int c = 0; c < kSparseSlots; ++c) {
            const unsigned long long pk = pack_key(sf[c], g * GS + sj[c]);
            if (pk < mn) {
              mn = pk;
              mc = c;
            }
          }
          if (pack_key(f, g * GS + j) > mn) {
            dropf = fmaxf(dropf, packed_value(mn));
#pragma unroll
            for (int c = 0; c < kSparseSlots; ++c) {
              if (c == mc) {
                sf[c] = f;
                sj[c] = j;
              }
            }
          } else {
            dropf = fmaxf(dropf, f);
          }
        }
      }

      unsigned long long* tc = cand + tok * kSparseCandStride;
      unsigned long long* ts = sel + tok * (kMaxK + 1);
      bool exact = false, slow = false, whole = false;
#pragma unroll 1
      for (;;) {
        float gsv, m2v;
        if (exact) {
          // exact two best: only slots within 4 eps of the fast second best
          const float lim = m2 - 4.0f * key_eps(fabsf(m2));
          float e1 = -INFINITY, e2 = -INFINITY;
#pragma unroll
          for (int c = 0; c < kSparseSlots; ++c) {
            if (sj[c] >= 0 && sf[c] >= lim) {
              const float ke = exact_key(grp, bgrp, sj[c]);
              e2 = fmaxf(e2, fminf(e1, ke));
              e1 = fmaxf(e1, ke);
            }
          }
          gsv = __fadd_rn(e1, e2);
          m2v = e2;
        } else {
          gsv = __fadd_rn(m1, m2);
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
        bool certain = true;
        if (!exact) {
          float glo2 = gsel ? gsv : INFINITY, ghi2 = gsel ? -INFINITY : gsv;
#pragma unroll
          for (int off = 1; off < G; off <<= 1) {
            glo2 = fminf(glo2, __shfl_xor_sync(segmask, glo2, off, G));
            ghi2 = fmaxf(ghi2, __shfl_xor_sync(segmask, ghi2, off, G));
          }
          if (ghi2 != -INFINITY)
            certain = (glo2 - ghi2) > 4.0f * key_eps(fmaxf(fabsf(glo2), fabsf(ghi2)));
        }
        float l0 = gsel ? m2v : INFINITY;
#pragma unroll
        for (int off = 1; off < G; off <<= 1) l0 = fminf(l0, __shfl_xor_sync(segmask, l0, off, G));
        if (!two_best) l0 = -INFINITY;
        const float thr = l0 - 4.0f * key_eps(fabsf(l0));
        // a dropped key near a threshold: settle the token on all exact keys
        const float need = gsel ? fminf(thr, m2) : m2;
        if (__any_sync(segmask, dropf >= need - 8.0f * key_eps(fabsf(need)))) {
          whole = true;
          break;
        }
        uint32_t mask = 0;
#pragma unroll
        for (int c = 0; c < kSparseSlots; ++c) mask |= (sj[c] >= 0 && sf[c] >= thr) ? (1u << c) : 0u;
        if (!gsel) mask = 0;
        const int cnt = __popc(mask);
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < G; off <<= 1) {
          const int o = __shfl_up_sync(segmask, incl, off, G);
          if (g >= off) incl += o;
        }
        const int C = __shfl_sync(segmask, incl, G - 1, G);
        if (C > kCap) {
          if (!exact) {
            exact = true;
            slow = true;
            continue;
          }
          whole = true;
          break;
        }
        int pos = incl - cnt;
#pragma unroll
        for (int c = 0; c < kSparseSlots; ++c) {
          if (mask & (1u << c)) {
            tc[pos++] = pack_key(exact ? exact_key(grp, bgrp, sj[c]) : sf[c], g * GS + sj[c]);
          }
        }
        const int C4 = (C + 3) & ~3;
        if (g < C4 - C) tc[C + g] = 0ull;  // zero pads rank below every key
        __syncwarp(segmask);
        // rank every candidate against all others (packed keys: one compare)
        for (int q = g; q < C; q += G) {
          const unsigned long long v = tc[q];
          int r = 0;
          for (int k2 = 0; k2 < C4; k2 += 4) {
            const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(tc + k2);
            const ulonglong2 b = *reinterpret_cast<const ulonglong2*>(tc + k2 + 2);
            r += (a.x > v) + (a.y > v) + (b.x > v) + (b.y > v);
          }
          if (r <= K) ts[r] = v;
        }
        __syncwarp(segmask);
        if (!exact) {
          if (C > K) {
            const float k8 = packed_value(ts[K - 1]), k9 = packed_value(ts[K]);
            certain = certain && (k8 - k9) > 4.0f * key_eps(fmaxf(fabsf(k8), fabsf(k9)));
          }
          if (!certain) {
            exact = true;
            slow = true;
            continue;
          }
        }
        break;
      }
      if (whole) {
        slow = true;
        sparse_full_exact<G, GS_MAX>(grp, bgrp, g, GS, TG, K, segmask, ts);
      }
      if (slow && g == 0 && valid) atomicAdd(&g_exact_rows, 1ull);

      // ---- weights, renormalisation, scaling, stores
      float* tw = wbuf + tok * (kMaxK + 1);
      for (int k = g; k < K; k += G) {
        const float xv = row[packed_index(ts[k])];
        tw[k] = slow ? sigmoid_exact_call(xv) : sigmoid_accurate(xv);
      }
      __syncwarp(segmask);
      float sum = 0.0f;
      if (p.renorm) {
        for (int k = 0; k < K; ++k) sum = __fadd_rn(sum, tw[k]);
      }
      if (valid) {
        for (int k = g; k < K; k += G) {
          float w = tw[k];
          if (p.renorm) w = __fdiv_rn(w, sum);
          if (p.scale != 1.0f) w = __fmul_rn(w, p.scale);
          p.w_out[token * K + k] = w;
          p.id_out[token * K + k] = packed_index(ts[k]);
        }
      }
      // next tile landed (every thread's own bounded wait), and every thread
      // is done with this one before its buffer is refilled
      bool nok = true;
      if (tn < tiles) nok = sm100::mbar_wait(&full[st ^ 1], ((i + 1) >> 1) & 1, abort_flag);
      if (__syncthreads_or(!nok)) {
        ++i;
        break;
      }
    }
  }

  if (threadIdx.x == 0 && *abort_flag) {
    // a wait ran out: record it, then let the copies this CTA issued land
    atomicExch(&g_router_error, 1);
    for (int j = i; j <= last_issued; ++j) {
      for (uint32_t n = 0; n < sm100::kSpinLimit && !sm100::mbar_try_wait(&full[j & 1], (j >> 1) & 1);
           ++n) {
      }
    }
  }
}

}  // namespace router
}  // namespace mcpu
