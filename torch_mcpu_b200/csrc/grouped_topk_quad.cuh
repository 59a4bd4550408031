// grouped_topk for fp32 logits, sigmoid scoring with a correction bias and 8
// groups (DeepSeek-V3's router): the quad kernel (included by
// grouped_topk.cu).
//
// Work split.  Four lanes serve one token (lane q of the quad owns groups 2q
// and 2q + 1), so a warp serves 8 tokens per tile and the per-token pick
// work is shared by 8 tokens per warp instruction.  Every warp streams its
// own tiles [8 tokens, E] through ONE shared-memory buffer filled by TMA:
// the buffer is needed only until the token's candidates are extracted, so
// it is handed back to TMA then, and the next tile lands while the warp
// ranks candidates and writes weights.  One buffer per warp keeps 20 warps
// resident per SM (three tiles per warp for 65536 tokens).  Waits are bounded; warps never wait for one another.
//
// Per token:
//   keys    every fast key sigmoid_fast(x) + bias is computed once and written
//           over its logit; each lane keeps its two groups' two best keys;
//   groups  the quad gathers the 8 group scores (sum of the two best keys)
//           and ranks its own groups (ties to the lower group index);
//   experts L0 = smallest second-best key of the picked groups; each picked
//           group holds two keys >= L0, so the k-th best key is >= L0 and only
//           keys >= L0 - 4 eps are candidates (about 11 per token); quad lane
//           q collects those of the q-th picked group as 64-bit (orderable
//           value, inverted index) keys, and each candidate is ranked by
//           direct comparison;
//   exactness fast keys are within eps = 2^-21 + 2^-22 |key| of the
//           reference's fp32 keys.  A group margin under 4 eps re-picks the
//           groups on exact keys (experts within 4 eps of a group's second
//           best); a k-th/k+1-th margin under 4 eps re-ranks the candidates on
//           exact keys.  Exact keys are the reference's sigmoid (correctly
//           rounded exp) of the logit re-read from global memory.  More than
//           kCap near-equal candidates take a fully exact pick over all
//           experts (also from global memory);
//   weights the sigmoid of each pick is recovered from its fast key (key -
//           bias) or, on the exact paths, recomputed; renormalised over the
//           quad and scaled.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kQuadThreads = 128;  // 4 warps per CTA (5 CTAs, 20 warps per SM)
constexpr int kQuadTokens = 8;     // tokens per warp tile
constexpr int kQuadCandStride = kCap;

struct QuadLayout {
  int tile_bytes;  // one [8, E] fp32 tile
  int warp_bytes;  // tile + candidate and pick lists + barrier of one warp
  int cand_off, sel_off, bar_off;
  int bias_off;
  int total;
};

__host__ __device__ inline QuadLayout quad_layout(int E, int K) {
  QuadLayout L;
  L.tile_bytes = (kQuadTokens * E * 4 + 127) & ~127;
  int off = L.tile_bytes;
  L.cand_off = off;
  off += kQuadTokens * kQuadCandStride * 8;
  L.sel_off = off;
  off += kQuadTokens * (K + 1) * 8;
  L.bar_off = off;
  off += 16;
  L.warp_bytes = (off + 127) & ~127;
  L.bias_off = (kQuadThreads / 32) * L.warp_bytes;
  L.total = L.bias_off + ((E * 4 + 127) & ~127) + 128;
  return L;
}

// Weight sigmoid from the logit: the fast sigmoid is within about 3e-6
// relative of the reference's for x >= -80; further out, the division form.
__device__ __forceinline__ float quad_weight_sigmoid(float x) {
  return x >= -80.0f ? sigmoid_fast(x) : sigmoid_accurate(x);
}

// Exact key of expert e from its logit in global memory: the reference's
// fp32 sigmoid plus the bias.
__device__ __forceinline__ float quad_exact_key(const float* gx, const float* sbias, int e) {
  return __fadd_rn(sigmoid_exact_call(__ldg(gx + e)), sbias[e]);
}

// The whole pick on exact keys over every expert of the token (for inputs
// with many near-equal keys): exact group scores, group pick, then k rounds
// of quad argmax, re-evaluating the exact keys from the logits in global
// memory in every round (this path is for degenerate inputs only).
template <int GS_MAX>
__device__ __noinline__ void quad_full_exact(const float* gx, const float* sbias, int q, int GS, int TG,
                                             int K, unsigned quadmask, unsigned long long* ts) {
  float gs[2];
  bool gsel[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gg = 2 * q + h;
    float e1 = -INFINITY, e2 = -INFINITY;
    for (int j = 0; j < GS; ++j) {
      const float k = quad_exact_key(gx, sbias, gg * GS + j);
      e2 = fmaxf(e2, fminf(e1, k));
      e1 = fmaxf(e1, k);
    }
    gs[h] = __fadd_rn(e1, e2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gg = 2 * q + h;
    int r = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float o = __shfl_sync(quadmask, gs[j & 1], j >> 1, 4);
      r += (o > gs[h]) || (o == gs[h] && j < gg);
    }
    gsel[h] = r < TG;
  }
  unsigned long long last = ~0ull;
  for (int r = 0; r < K; ++r) {
    unsigned long long best = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!gsel[h]) continue;
      const int gg = 2 * q + h;
      for (int j = 0; j < GS; ++j) {
        const unsigned long long pk = pack_key(quad_exact_key(gx, sbias, gg * GS + j), gg * GS + j);
        if (pk < last && pk > best) best = pk;
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      const unsigned long long o = __shfl_xor_sync(quadmask, best, off, 4);
      best = o > best ? o : best;
    }
    if (q == 0) ts[r] = best;
    last = best;
  }
  __syncwarp(quadmask);
}

// Ranks the C candidates of tc (C <= kCap, zero-padded to CP entries) into
// ts[0..K] (rank K: the (k+1)-th key).  Lane q ranks entries q, q + 4, ...
__device__ __forceinline__ void quad_rank(const unsigned long long* tc, unsigned long long* ts, int C,
                                          int CP, int K, int q, unsigned quadmask) {
  bool ranked = false;
  if (C <= 16) {
    // on the value words alone; distinct values give distinct ranks, which
    // the rank sum C (C - 1) / 2 confirms
    unsigned long long v[4];
    uint32_t vh[4];
    int r[4] = {0, 0, 0, 0};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = tc[q + 4 * u];
      vh[u] = static_cast<uint32_t>(v[u] >> 32);
    }
#pragma unroll
    for (int k2 = 0; k2 < 16; k2 += 2) {
      const uint4 a = *reinterpret_cast<const uint4*>(tc + k2);  // {lo0, hi0, lo1, hi1}
#pragma unroll
      for (int u = 0; u < 4; ++u) r[u] += (a.y > vh[u]) + (a.w > vh[u]);
    }
    int rs = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) rs += (q + 4 * u < C) ? r[u] : 0;
    rs += __shfl_xor_sync(quadmask, rs, 1, 4);
    rs += __shfl_xor_sync(quadmask, rs, 2, 4);
    if (rs == C * (C - 1) / 2) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (q + 4 * u < C && r[u] <= K) ts[r[u]] = v[u];
      ranked = true;
    }
  }
  if (!ranked) {
    // equal values, or more than 16 candidates: full 64-bit keys
    for (int e = q; e < C; e += 4) {
      const unsigned long long v = tc[e];
      int r = 0;
      for (int k2 = 0; k2 < CP; k2 += 2) {
        const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(tc + k2);
        r += (a.x > v) + (a.y > v);
      }
      if (r <= K) ts[r] = v;
    }
  }
  __syncwarp(quadmask);
}

template <int GS_MAX>
__global__ void __launch_bounds__(kQuadThreads, 5) grouped_topk_quad_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const long long wtiles) {
  constexpr int VE = 4;
  constexpr int NCH_MAX = GS_MAX / VE;
  static_assert(GS_MAX <= 32 && GS_MAX % VE == 0, "bit masks are 32 bits, vectors of 4");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((128 - (ra & 127)) & 127);
  const QuadLayout L = quad_layout(p.E, p.K);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* wb = base + warp * L.warp_bytes;
  float* tile = reinterpret_cast<float*>(wb);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(wb + L.cand_off);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(wb + L.sel_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(wb + L.bar_off);
  int* abort_flag = reinterpret_cast<int*>(wb + L.bar_off + 8);
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);

  const int GS = p.GS, K = p.K, E = p.E, TG = p.TG;
  const int t = lane >> 2;  // token of the tile
  const int q = lane & 3;   // quad lane: groups 2q, 2q + 1
  const unsigned quadmask = 0xFu << (lane & ~3);
  const int tile_bytes = kQuadTokens * E * 4;
  const int nch = GS / VE;
  const int rot = lane % nch;  // chunk rotation: the 8 lanes of a phase hit distinct banks
  const long long gw = static_cast<long long>(blockIdx.x) * (kQuadThreads / 32) + warp;
  const long long nw = static_cast<long long>(gridDim.x) * (kQuadThreads / 32);
  const float* gating = static_cast<const float*>(p.gating);

  if (lane == 0) {
    sm100::mbar_init(full, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    if (gw < wtiles) {
      sm100::mbar_arrive_expect_tx(full, tile_bytes);
      sm100::tma_load_2d(tile, &tm, full, 0, static_cast<int>(gw * kQuadTokens));
    }
  }
  for (int i = threadIdx.x; i < E; i += blockDim.x) sbias[i] = p.bias[i];
  __syncthreads();  // the only CTA-wide barrier: bias staged, barriers initialised

  long long i = 0;
  bool inflight = gw < wtiles;  // a copy into the buffer is outstanding
  for (;; ++i) {
    const long long wt = gw + i * nw;
    if (wt >= wtiles) break;
    const bool ok = sm100::mbar_wait(full, static_cast<uint32_t>(i & 1), abort_flag);
    if (!__all_sync(0xFFFFFFFFu, ok)) break;
    inflight = false;

    const long long token = wt * kQuadTokens + t;
    const bool valid = token < p.T;
    float* row = tile + t * E;
    const float* gx = gating + (valid ? token : 0) * static_cast<long long>(E);

    // ---- keys: computed once, written over the logits; two best per group
    float m1[2], m2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float* gp = row + (2 * q + h) * GS;
      const float* bp = sbias + (2 * q + h) * GS;
      float a1 = -INFINITY, a2 = -INFINITY, b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
      for (int c = 0; c < NCH_MAX; ++c) {
        if (c < nch) {
          int cc = c + rot;
          if (cc >= nch) cc -= nch;
          const float4 x4 = *reinterpret_cast<const float4*>(gp + cc * VE);
          const float4 b4 = *reinterpret_cast<const float4*>(bp + cc * VE);
          float4 k4;
          k4.x = fast_key(x4.x, b4.x);
          k4.y = fast_key(x4.y, b4.y);
          k4.z = fast_key(x4.z, b4.z);
          k4.w = fast_key(x4.w, b4.w);
          *reinterpret_cast<float4*>(gp + cc * VE) = k4;
          a2 = fmaxf(a2, fminf(a1, k4.x));
          a1 = fmaxf(a1, k4.x);
          b2 = fmaxf(b2, fminf(b1, k4.y));
          b1 = fmaxf(b1, k4.y);
          a2 = fmaxf(a2, fminf(a1, k4.z));
          a1 = fmaxf(a1, k4.z);
          b2 = fmaxf(b2, fminf(b1, k4.w));
          b1 = fmaxf(b1, k4.w);
        }
      }
      m1[h] = fmaxf(a1, b1);
      m2[h] = fmaxf(fminf(a1, b1), fmaxf(a2, b2));
    }

    // ---- group pick; on a margin under 4 eps, again on exact keys
    float gs[2] = {__fadd_rn(m1[0], m2[0]), __fadd_rn(m1[1], m2[1])};
    float m2v[2] = {m2[0], m2[1]};
    bool exact = false;
    bool gsel[2];
    float l0;
#pragma unroll 1
    for (;;) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[2 * j] = __shfl_sync(quadmask, gs[0], j, 4);
        o[2 * j + 1] = __shfl_sync(quadmask, gs[1], j, 4);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gg = 2 * q + h;
        int r = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) r += (o[j] > gs[h]) || (o[j] == gs[h] && j < gg);
        gsel[h] = r < TG;
      }
      float glo = fminf(gsel[0] ? gs[0] : INFINITY, gsel[1] ? gs[1] : INFINITY);
      float ghi = fmaxf(gsel[0] ? -INFINITY : gs[0], gsel[1] ? -INFINITY : gs[1]);
      l0 = fminf(gsel[0] ? m2v[0] : INFINITY, gsel[1] ? m2v[1] : INFINITY);
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) {
        glo = fminf(glo, __shfl_xor_sync(quadmask, glo, off, 4));
        ghi = fmaxf(ghi, __shfl_xor_sync(quadmask, ghi, off, 4));
        l0 = fminf(l0, __shfl_xor_sync(quadmask, l0, off, 4));
      }
      if (exact || ghi == -INFINITY || (glo - ghi) > 4.0f * key_eps(fmaxf(fabsf(glo), fabsf(ghi)))) break;
      // exact two best of each group: only experts whose fast key is within
      // 4 eps of the fast second best can be among them
      exact = true;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gg = 2 * q + h;
        const float lim = m2[h] - 4.0f * key_eps(fabsf(m2[h]));
        float e1 = -INFINITY, e2 = -INFINITY;
        for (int j = 0; j < GS; ++j) {
          if (row[gg * GS + j] >= lim) {
            const float ke = quad_exact_key(gx, sbias, gg * GS + j);
            e2 = fmaxf(e2, fminf(e1, ke));
            e1 = fmaxf(e1, ke);
          }
        }
        gs[h] = __fadd_rn(e1, e2);
        m2v[h] = e2;
      }
    }
    const float thr = l0 - 4.0f * key_eps(fabsf(l0));

    // ---- candidates: keys >= thr; quad lane q scans the q-th (and q + 4-th)
    // picked group
    uint32_t selbits = (gsel[0] ? 1u << (2 * q) : 0u) | (gsel[1] ? 2u << (2 * q) : 0u);
    selbits |= __shfl_xor_sync(quadmask, selbits, 1, 4);
    selbits |= __shfl_xor_sync(quadmask, selbits, 2, 4);
    int cg[2] = {-1, -1};
    {
      int n = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if ((selbits >> b) & 1u) {
          if (n == q) cg[0] = b;
          if (n == q + 4) cg[1] = b;
          ++n;
        }
      }
    }
    uint32_t cm[2] = {0u, 0u};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (cg[h] < 0) continue;
      const float* gp = row + cg[h] * GS;
#pragma unroll
      for (int c = 0; c < NCH_MAX; ++c) {
        if (c < nch) {
          int cc = c + rot;
          if (cc >= nch) cc -= nch;
          const float4 k4 = *reinterpret_cast<const float4*>(gp + cc * VE);
          const uint32_t b = (k4.x >= thr ? 1u : 0u) | (k4.y >= thr ? 2u : 0u) | (k4.z >= thr ? 4u : 0u) |
                             (k4.w >= thr ? 8u : 0u);
          cm[h] |= b << (cc * VE);
        }
      }
    }
    const int cnt = __popc(cm[0]) + __popc(cm[1]);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      const int v = __shfl_up_sync(quadmask, incl, off, 4);
      if (q >= off) incl += v;
    }
    const int C = __shfl_sync(quadmask, incl, 3, 4);
    unsigned long long* tc = cand + t * kQuadCandStride;
    unsigned long long* ts = sel + t * (K + 1);
    const bool whole = C > kCap;
    if (!whole) {
      int pos = incl - cnt;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (cg[h] < 0) continue;
        for (uint32_t m = cm[h]; m; m &= m - 1) {
          const int e = cg[h] * GS + __ffs(m) - 1;
          const float v = exact ? quad_exact_key(gx, sbias, e) : row[e];
          tc[pos++] = pack_key(v, e);
        }
      }
    }

    // ---- the tile is no longer needed: hand the buffer to the next tile
    __syncwarp();
    if (lane == 0) {
      const long long nt = wt + nw;
      if (nt < wtiles) {
        sm100::mbar_arrive_expect_tx(full, tile_bytes);
        sm100::tma_load_2d(tile, &tm, full, 0, static_cast<int>(nt * kQuadTokens));
      }
    }
    inflight = wt + nw < wtiles;

    // ---- rank, certify the k-th/k+1-th margin, else re-rank on exact keys
    bool slow = exact;
    if (whole) {
      slow = true;
      quad_full_exact<GS_MAX>(gx, sbias, q, GS, TG, K, quadmask, ts);
    } else {
      const int CP = C <= 16 ? 16 : ((C + 3) & ~3);
      for (int e = C + q; e < CP; e += 4) tc[e] = 0ull;
      __syncwarp(quadmask);
      quad_rank(tc, ts, C, CP, K, q, quadmask);
      if (!exact && C > K) {
        const float k8 = packed_value(ts[K - 1]), k9 = packed_value(ts[K]);
        if (!((k8 - k9) > 4.0f * key_eps(fmaxf(fabsf(k8), fabsf(k9))))) {
          slow = true;
          for (int e = q; e < C; e += 4) {
            const int idx = packed_index(tc[e]);
            tc[e] = pack_key(quad_exact_key(gx, sbias, idx), idx);
          }
          __syncwarp(quadmask);
          quad_rank(tc, ts, C, CP, K, q, quadmask);
        }
      }
    }
    if (slow && q == 0 && valid) atomicAdd(&g_exact_rows, 1ull);

    // ---- weights: lane q owns outputs q, q + 4, q + 8, q + 12 (< K).  From
    // a fast key, sigmoid = key - bias is within 2^-20 relative while it is
    // at least |key| / 16; otherwise, and on the exact paths, it is
    // recomputed from the logit.
    float wv[4];
    int id[4];
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = q + 4 * u;
      wv[u] = 0.0f;
      id[u] = 0;
      if (k < K) {
        const unsigned long long pk = ts[k];
        id[u] = packed_index(pk);
        const float key = packed_value(pk);
        float sg = __fsub_rn(key, sbias[id[u]]);
        if (slow) {
          sg = sigmoid_exact_call(__ldg(gx + id[u]));
        } else if (!(sg >= 0.0625f * fabsf(key))) {
          sg = quad_weight_sigmoid(__ldg(gx + id[u]));
        }
        wv[u] = sg;
        sum = __fadd_rn(sum, sg);
      }
    }
    if (p.renorm) {
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) sum = __fadd_rn(sum, __shfl_xor_sync(quadmask, sum, off, 4));
    }
    if (valid) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k = q + 4 * u;
        if (k < K) {
          float w = wv[u];
          if (p.renorm) w = __fdiv_rn(w, sum);
          if (p.scale != 1.0f) w = __fmul_rn(w, p.scale);
          p.w_out[token * K + k] = w;
          p.id_out[token * K + k] = id[u];
        }
      }
    }
    __syncwarp();
  }

  if (lane == 0 && *abort_flag) {
    // a wait ran out: record it, then let this warp's copy in flight land
    atomicExch(&g_router_error, 1);
    if (inflight) {
      for (uint32_t n = 0; n < sm100::kSpinLimit && !sm100::mbar_try_wait(full, static_cast<uint32_t>(i & 1));
           ++n) {
      }
    }
  }
}

}  // namespace router
}  // namespace mcpu
