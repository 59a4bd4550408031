// grouped_topk, TMA-fed persistent variant (included by grouped_topk.cu).
//
// Each CTA loops over tiles of `tpt` tokens (tpt * G = 256 threads).  One
// thread streams the tiles [tpt, E] into a 2-stage shared-memory ring with
// cp.async.bulk.tensor; the others read their group's experts from shared
// memory (16-byte chunks in a rotated order so the G lanes of a token hit
// distinct banks).
//
// Expert pick without sorting: with every selected group contributing its
// two best experts (2 * topk_group >= topk), the k-th best candidate is at
// least L0 = min over selected groups of the group's second-best key.  Only
// keys >= L0 - delta can be among the top k (delta = the fast path's margin),
// typically 10-14 of the 128 experts of the selected groups.  Those
// candidates go to a per-token list in shared memory and each is ranked by
// direct comparison (ties to the lower index).  The margin between the k-th
// and (k+1)-th key certifies the fast result; when only k candidates exist
// the delta in the filter certifies it.  Rows that cannot be certified, or
// whose candidate list overflows, run the exact recomputation and a k-round
// argmax.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kCap = 32;      // candidate slots per token
constexpr int kStages = 2;    // TMA ring depth
constexpr int kMaxK = 16;

struct TmaLayout {
  int tile_bytes;   // one stage, rounded to 1024
  int bias_off, ck_off, ci_off, selk_off, seli_off, wbuf_off, ninth_off, bar_off;
  int total;        // dynamic shared memory bytes (incl. 1024 alignment slack)
};

__host__ __device__ inline TmaLayout tma_layout(int tpt, int E, int esz) {
  TmaLayout L;
  const int box = tpt * E * esz;
  L.tile_bytes = (box + 1023) & ~1023;
  int off = kStages * L.tile_bytes;
  L.bias_off = off;
  off += ((E * 4 + 15) & ~15);
  L.ck_off = off;
  off += tpt * kCap * 4;
  L.ci_off = off;
  off += tpt * kCap * 2;
  off = (off + 15) & ~15;
  L.selk_off = off;
  off += tpt * kMaxK * 4;
  L.seli_off = off;
  off += tpt * kMaxK * 4;
  L.wbuf_off = off;
  off += tpt * kMaxK * 4;
  L.ninth_off = off;
  off += tpt * 4;
  off = (off + 15) & ~15;
  L.bar_off = off;
  off += kStages * 8 + 16;
  L.total = off + 1024;
  return L;
}

template <typename InT>
__device__ __forceinline__ float smem_elem(const InT* row, int i);
template <>
__device__ __forceinline__ float smem_elem<float>(const float* row, int i) { return row[i]; }
template <>
__device__ __forceinline__ float smem_elem<__nv_bfloat16>(const __nv_bfloat16* row, int i) {
  return bf16_bits_to_float(reinterpret_cast<const uint16_t*>(row)[i]);
}

// (a, ia) ranks before (b, ib)
__device__ __forceinline__ bool ranks_before(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia < ib);
}

template <typename InT, int GS_MAX, bool kFast>
__global__ void __launch_bounds__(kThreads, 3) grouped_topk_tma_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const int tiles, const int tpt) {
  constexpr bool kBf16 = sizeof(InT) == 2;
  constexpr int VE = 16 / sizeof(InT);     // elements per 16-byte chunk
  constexpr int NCH_MAX = (GS_MAX + VE - 1) / VE;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (ra & 1023)) & 1023);
  const TmaLayout L = tma_layout(tpt, p.E, sizeof(InT));
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  float* ck = reinterpret_cast<float*>(base + L.ck_off);
  uint16_t* ci = reinterpret_cast<uint16_t*>(base + L.ci_off);
  float* selk = reinterpret_cast<float*>(base + L.selk_off);
  int* seli = reinterpret_cast<int*>(base + L.seli_off);
  float* wbuf = reinterpret_cast<float*>(base + L.wbuf_off);
  float* ninth = reinterpret_cast<float*>(base + L.ninth_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_off);
  int* abort_flag = reinterpret_cast<int*>(base + L.bar_off + kStages * 8);

  const int G = p.G, GS = p.GS, K = p.K, E = p.E;
  const int lane = threadIdx.x & 31;
  const int tok = threadIdx.x / G;
  const int g = threadIdx.x & (G - 1);
  const unsigned segmask = (G == 32) ? 0xFFFFFFFFu : (((1u << G) - 1u) << (lane & ~(G - 1)));
  const bool has_bias = p.bias != nullptr;
  const int box_bytes = tpt * E * static_cast<int>(sizeof(InT));
  const int nch = GS / VE;
  const int gshift = g % (nch > 0 ? nch : 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) sm100::mbar_init(&full[s], 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tensormap(&tm);
  }
  for (int i = threadIdx.x; i < E; i += blockDim.x) sbias[i] = has_bias ? p.bias[i] : 0.0f;
  __syncthreads();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages - 1; ++s) {
      const int t = blockIdx.x + s * gridDim.x;
      if (t < tiles) {
        sm100::mbar_arrive_expect_tx(&full[s], box_bytes);
        sm100::tma_load_2d(base + s * L.tile_bytes, &tm, &full[s], 0, t * tpt);
      }
    }
  }

  int i = 0;
  for (;; ++i) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= tiles) break;
    const int st = i % kStages;
    if (threadIdx.x == 0) {
      const int tn = t + (kStages - 1) * gridDim.x;
      if (tn < tiles) {
        const int sn = (i + kStages - 1) % kStages;
        sm100::mbar_arrive_expect_tx(&full[sn], box_bytes);
        sm100::tma_load_2d(base + sn * L.tile_bytes, &tm, &full[sn], 0, tn * tpt);
      }
    }
    if (!sm100::mbar_wait(&full[st], (i / kStages) & 1, abort_flag)) break;

    const long long token = static_cast<long long>(t) * tpt + tok;
    const bool valid = token < p.T;
    const InT* row = reinterpret_cast<const InT*>(base + st * L.tile_bytes) + tok * E;
    const InT* grp = row + g * GS;
    const float* bgrp = sbias + g * GS;

    // ---- this lane's experts: slot s = c*VE + q holds local expert
    //      ((c + gshift) % nch) * VE + q  (vector layout) or s (scalar)
    const bool vec_layout = (GS % VE) == 0;
    auto local_of = [&](int s) -> int {
      if (!vec_layout) return s;
      const int c = s / VE;
      int cc = c + gshift;
      if (cc >= nch) cc -= nch;
      return cc * VE + (s - c * VE);
    };
    auto slot_ok = [&](int s) -> bool { return vec_layout ? (s / VE) < nch : s < GS; };
    // logit of slot s, read from the staged tile
    auto logit = [&](int s) -> float { return smem_elem<InT>(grp, local_of(s)); };

    // softmax statistics (whole row)
    float row_max = 0.0f, row_sum = 1.0f;
    if (p.scoring == MCPU_SCORING_SOFTMAX) {
      float m = -INFINITY;
      for (int j = 0; j < GS; ++j) m = fmaxf(m, smem_elem<InT>(grp, j));
      row_max = seg_max(m, segmask, G);
      float sum = 0.0f;
      for (int j = 0; j < GS; ++j) sum = __fadd_rn(sum, expf(smem_elem<InT>(grp, j) - row_max));
      row_sum = seg_sum(sum, segmask, G);
    }

    // ranking keys, chunk by chunk from shared memory
    float key[GS_MAX];
    auto compute_keys = [&](bool exact) {
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
              if (kFast && !exact) {
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
          }
        }
      } else {
#pragma unroll
        for (int s = 0; s < GS_MAX; ++s) {
          float k = -INFINITY;
          if (s < GS) {
            const float xv = smem_elem<InT>(grp, s), bv = bgrp[s];
            if (kFast && !exact) {
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
        }
      }
    };
    (void)logit;

    bool slow = false;
    bool exact_keys = !kFast;
    compute_keys(!kFast);
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      if (pass == 1) {
        compute_keys(true);  // exact recomputation of the fp32 sigmoid + bias keys
        exact_keys = true;
      }
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int s = 0; s < GS_MAX; ++s) {
        m2 = fmaxf(m2, fminf(m1, key[s]));
        m1 = fmaxf(m1, key[s]);
      }
      const float gs = has_bias ? __fadd_rn(m1, m2) : m1;
      int rank = 0;
      for (int j = 0; j < G; ++j) {
        const float o = __shfl_sync(segmask, gs, j, G);
        rank += (o > gs) || (o == gs && j < g);
      }
      const bool gsel = rank < p.TG;
      bool ok = true;
      if (!exact_keys) {
        const float lo = seg_min(gsel ? gs : INFINITY, segmask, G);
        const float hi = seg_max(gsel ? -INFINITY : gs, segmask, G);
        if (hi != -INFINITY) ok = (lo - hi) > (0x1p-18f + 0x1p-19f * fmaxf(fabsf(lo), fabsf(hi)));
      }
      // candidate filter
      float l0 = -INFINITY;
      if (GS >= 2 && 2 * p.TG >= K) l0 = seg_min(gsel ? m2 : INFINITY, segmask, G);
      const float delta = exact_keys ? 0.0f : (0x1p-19f + 0x1p-20f * fabsf(l0));
      const float thr = l0 - delta;
      int c = 0;
#pragma unroll
      for (int s = 0; s < GS_MAX; ++s) c += (gsel && key[s] >= thr) ? 1 : 0;
      int incl = c;
      for (int off = 1; off < G; off <<= 1) {
        const int o = __shfl_up_sync(segmask, incl, off, G);
        if (g >= off) incl += o;
      }
      const int C = __shfl_sync(segmask, incl, G - 1, G);
      float* tck = ck + tok * kCap;
      uint16_t* tci = ci + tok * kCap;
      float* tsk = selk + tok * kMaxK;
      int* tsi = seli + tok * kMaxK;
      if (C <= kCap) {
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
        if (!exact_keys && C > K) {
          const float k8 = tsk[K - 1], k9 = ninth[tok];
          ok = ok && (k8 - k9) > (0x1p-19f + 0x1p-20f * fmaxf(fabsf(k8), fabsf(k9)));
        }
      } else if (!exact_keys) {
        ok = false;  // too many near-equal candidates: decide on exact keys
      } else {
        // k rounds of segment argmax (exact keys: a strict total order)
        float lk = INFINITY;
        int li = -1;
        for (int r = 0; r < K; ++r) {
          float bk = -INFINITY;
          int bi = 0x7FFFFFFF;
#pragma unroll
          for (int s = 0; s < GS_MAX; ++s) {
            const int idx = g * GS + local_of(s);
            const bool after = key[s] < lk || (key[s] == lk && idx > li);
            if (gsel && slot_ok(s) && after && ranks_before(key[s], idx, bk, bi)) {
              bk = key[s];
              bi = idx;
            }
          }
          for (int off = 1; off < G; off <<= 1) {
            const float ok2 = __shfl_xor_sync(segmask, bk, off, G);
            const int oi2 = __shfl_xor_sync(segmask, bi, off, G);
            if (ranks_before(ok2, oi2, bk, bi)) {
              bk = ok2;
              bi = oi2;
            }
          }
          if (g == 0) {
            tsk[r] = bk;
            tsi[r] = bi;
          }
          lk = bk;
          li = bi;
        }
        __syncwarp(segmask);
      }
      if (ok) break;
      slow = true;  // uncertified fast result: one exact pass
    }
    if (slow && g == 0 && valid) atomicAdd(&g_exact_rows, 1ull);

    // ---- weights, renormalisation, scaling, stores
    float* tw = wbuf + tok * kMaxK;
    const int* tsi = seli + tok * kMaxK;
    for (int k = g; k < K; k += G) {
      const float xv = smem_elem<InT>(row, tsi[k]);
      float sc;
      if (p.scoring == MCPU_SCORING_SIGMOID) {
        sc = (kFast && !slow) ? sigmoid_accurate(xv) : sigmoid_exact_call(xv);
      } else {
        sc = __fdiv_rn(expf(xv - row_max), row_sum);
      }
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
    __syncthreads();
  }

  if (threadIdx.x == 0) {
    if (*abort_flag) atomicExch(&g_router_error, 1);
    // loads still in flight (only after an abort) land before the CTA exits
    for (int s = 1; s < kStages; ++s) {
      const int t = blockIdx.x + (i + s - 1) * gridDim.x;
      if (t < tiles && *abort_flag) {
        const int sn = (i + s - 1) % kStages;
        for (uint32_t n = 0; n < sm100::kSpinLimit &&
                             !sm100::mbar_try_wait(&full[sn], ((i + s - 1) / kStages) & 1);
             ++n) {
        }
      }
    }
  }
}

}  // namespace router
}  // namespace mcpu
