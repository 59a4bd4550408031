// grouped_topk for fp32 logits, sigmoid scoring with a correction bias and 8
// groups of 16..32 experts (DeepSeek-V3's router): the coarse-key kernel
// (included by grouped_topk.cu after the quad kernel, whose helpers it uses).
//
// Same work split and buffering as the quad kernel: four lanes per token
// (lane q owns groups 2q and 2q + 1), 8 tokens per warp tile, one TMA buffer
// per warp handed back once the token's candidates are extracted.  What
// changes is the pass over every expert, which now runs two experts per
// instruction in f16x2:
//
//   coarse key c = f16(0.5 * tanh.approx.f16x2(0.5 * f16(x)) + f16(0.5 + b))
//
// is within delta of the fp32 fast key k = sigmoid_fast(x) + b (delta is a
// proven bound, below), and fp32 fast keys are then computed only for the
// experts the bound cannot rule out:
//
//   groups   coarse group scores (sum of the two best coarse keys) are
//            within 2 delta of the fast ones.  When the picked and the
//            unpicked groups are more than 4 delta apart the pick is the
//            fast keys' pick.  Otherwise a group above the (TG+1)-th coarse
//            score by more than 4 delta is surely picked, one below the
//            TG-th by more than 4 delta surely not, and only the groups in
//            between get fast scores: fast keys of the experts whose coarse
//            key is within 2 delta of the group's second best coarse key
//            (these include the two best fast keys).  The pick among them,
//            its 4 eps certification and the exact re-pick are the quad
//            kernel's, restricted to those groups.
//   experts  L0 = smallest lower bound of a picked group's second-best fast
//            key (its fast value, or coarse second best - delta); only keys
//            >= thr = L0 - 4 eps can be among the top k.  Quad lane q takes
//            the q-th picked group, marks the experts with coarse key >=
//            thr - delta, computes their fast keys and keeps those >= thr:
//            a superset of the quad kernel's candidates.  Ranking, the
//            k-th/k+1-th certification, the exact re-rank and the weights
//            are the quad kernel's.
//
// Every decision is therefore taken on fp32 fast (or exact) keys with the
// quad kernel's certificates: the result is the quad kernel's result.
#pragma once

#include <cuda_fp16.h>

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kCoarseThreads = 128;  // 4 warps per CTA

// |coarse key - fast key| <= delta for every expert when B = max |bias| is
// at most kCoarseMaxBias; the terms, with a 25 % margin on their sum:
//   logit rounded to f16       max_x |x| sigmoid'(x) 2^-11 < 0.2242 * 2^-11
//   tanh.approx.f16x2          kTanhF16AbsErr / 2 (largest error over every
//                              f16 input, measured on B200)
//   0.5 + bias rounded to f16  2^-11 (0.5 + B) + 2^-25
//   key rounded to f16         2^-11 (1 + B) + 2^-25  (|key| <= 1 + B)
//   fast key vs sigmoid + b    2^-21 + 2^-22 (1 + B)
// Beyond kCoarseMaxBias (or for a non-finite bias) delta is infinite: every
// expert is then evaluated in fp32, as in the quad kernel.
constexpr float kTanhF16AbsErr = 0x1p-10f;
constexpr float kCoarseMaxBias = 8.0f;

__host__ __device__ inline float coarse_delta(float max_abs_bias) {
  if (!(max_abs_bias <= kCoarseMaxBias)) return INFINITY;
  const float B = max_abs_bias;
  const float d = 0.2242f * 0x1p-11f + 0.5f * kTanhF16AbsErr + 0x1p-11f * (0.5f + B) + 0x1p-11f * (1.0f + B) +
                  0x1p-24f + 0x1p-21f + 0x1p-22f * (1.0f + B);
  return 1.25f * d;
}

struct CoarseLayout {
  int tile_bytes;    // one [8, E] fp32 tile
  int coarse_off;    // [8, E] f16 coarse keys; a token's candidate list reuses its row
  int sel_off, bar_off;
  int warp_bytes;
  int bias_off;      // fp32 bias [E]
  int biash_off;     // f16 (0.5 + bias) [E], then the CTA's delta
  int total;
};

__host__ __device__ inline CoarseLayout coarse_layout(int E, int K) {
  CoarseLayout L;
  L.tile_bytes = (kQuadTokens * E * 4 + 127) & ~127;
  int off = L.tile_bytes;
  L.coarse_off = off;
  off += (kQuadTokens * E * 2 + 127) & ~127;
  L.sel_off = off;
  off += kQuadTokens * (K + 1) * 8;
  L.bar_off = off;
  off += 16;
  L.warp_bytes = (off + 127) & ~127;
  L.bias_off = (kCoarseThreads / 32) * L.warp_bytes;
  L.biash_off = L.bias_off + ((E * 4 + 127) & ~127);
  L.total = L.biash_off + ((E * 2 + 127) & ~127) + 128 /*delta*/ + 128 /*alignment*/;
  return L;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two coarse keys: x2 = two logits in f16, bias2 = f16(0.5 + b) of both.
__device__ __forceinline__ __half2 coarse_key2(__half2 x2, uint32_t bias2) {
  const __half2 half = __float2half2_rn(0.5f);
  uint32_t t;
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(t) : "r"(h2_bits(__hmul2(x2, half))));
  return __hfma2(bits_h2(t), half, bits_h2(bias2));
}

// Experts of one group (GS coarse keys at p, 16-byte aligned) whose coarse
// key is >= thr2 (both halves the threshold): bit j of the result is expert
// 2j, bit 16 + j expert 2j + 1.
template <int GS_MAX>
__device__ __forceinline__ uint32_t coarse_members(const __half* p, int GS, __half2 thr2) {
  uint32_t m = 0;
#pragma unroll
  for (int c = 0; c < GS_MAX / 8; ++c) {
    if (c * 8 < GS) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + c * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int pr = c * 4 + u;  // pair index
        if (pr * 2 < GS) m |= (__hge2_mask(bits_h2(w[u]), thr2) << pr) & (0x00010001u << pr);
      }
    }
  }
  return m;
}

__device__ __forceinline__ int member_index(uint32_t bit) { return bit < 16 ? 2 * bit : 2 * (bit - 16) + 1; }

// The largest f16 not above v (v finite or -inf).
__device__ __forceinline__ __half2 half2_floor(float v) {
  const __half h = __float2half_rd(v);
  return __halves2half2(h, h);
}

template <int GS_MAX>
__global__ void __launch_bounds__(kCoarseThreads, 4) grouped_topk_coarse_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const long long wtiles) {
  constexpr int VE = 4;
  constexpr int NCH_MAX = GS_MAX / VE;
  static_assert(GS_MAX <= 32 && GS_MAX % 8 == 0, "bit masks are 32 bits, vectors of 8 halves");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((128 - (ra & 127)) & 127);
  const CoarseLayout L = coarse_layout(p.E, p.K);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* wb = base + warp * L.warp_bytes;
  float* tile = reinterpret_cast<float*>(wb);
  __half* coarse = reinterpret_cast<__half*>(wb + L.coarse_off);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(wb + L.sel_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(wb + L.bar_off);
  int* abort_flag = reinterpret_cast<int*>(wb + L.bar_off + 8);
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  __half* sbias_h = reinterpret_cast<__half*>(base + L.biash_off);
  float* sdelta = reinterpret_cast<float*>(base + L.biash_off + ((p.E * 2 + 127) & ~127));

  const int GS = p.GS, K = p.K, E = p.E, TG = p.TG;
  const int t = lane >> 2;  // token of the tile
  const int q = lane & 3;   // quad lane: groups 2q, 2q + 1
  const unsigned quadmask = 0xFu << (lane & ~3);
  const int tile_bytes = kQuadTokens * E * 4;
  const int nch = GS / VE;
  const int rot = lane % nch;  // chunk rotation: the lanes of a phase hit distinct banks
  const long long gw = static_cast<long long>(blockIdx.x) * (kCoarseThreads / 32) + warp;
  const long long nw = static_cast<long long>(gridDim.x) * (kCoarseThreads / 32);
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
  // bias in fp32 and as f16(0.5 + b); the CTA's delta from max |b|
  float bmax = 0.0f;
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    const float b = p.bias[i];
    sbias[i] = b;
    sbias_h[i] = __float2half_rn(__fadd_rn(0.5f, b));
    bmax = fmaxf(bmax, fabsf(b));
    if (b != b) bmax = INFINITY;  // a NaN bias disables the coarse bound
  }
  if (threadIdx.x == 0) *sdelta = 0.0f;
  __syncthreads();
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xFFFFFFFFu, bmax, off));
  if (lane == 0) atomicMax(reinterpret_cast<int*>(sdelta), __float_as_int(bmax));  // non-negative floats
  __syncthreads();  // bias staged, barriers initialised, max |b| known
  const float dlt = coarse_delta(*sdelta);
  const float four_d = 4.0f * dlt;

  long long i = 0;
  bool inflight = gw < wtiles;
  for (;; ++i) {
    const long long wt = gw + i * nw;
    if (wt >= wtiles) break;
    const bool ok = sm100::mbar_wait(full, static_cast<uint32_t>(i & 1), abort_flag);
    if (!__all_sync(0xFFFFFFFFu, ok)) break;
    inflight = false;

    const long long token = wt * kQuadTokens + t;
    const bool valid = token < p.T;
    const float* row = tile + t * E;
    __half* crow = coarse + t * E;
    const float* gx = gating + (valid ? token : 0) * static_cast<long long>(E);

    // ---- coarse keys (two experts per instruction), stored; two best per group
    float c1[2], c2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int gg = 2 * q + h;
      const float* gp = row + gg * GS;
      const uint2* bp = reinterpret_cast<const uint2*>(sbias_h + gg * GS);
      uint2* kp = reinterpret_cast<uint2*>(crow + gg * GS);
      const __half2 ninf = __float2half2_rn(-INFINITY);
      __half2 a1 = ninf, a2 = ninf;
#pragma unroll
      for (int c = 0; c < NCH_MAX; ++c) {
        if (c < nch) {
          int cc = c + rot;
          if (cc >= nch) cc -= nch;
          const float4 x4 = *reinterpret_cast<const float4*>(gp + cc * VE);
          const uint2 b2 = bp[cc];
          const __half2 k01 = coarse_key2(__floats2half2_rn(x4.x, x4.y), b2.x);
          const __half2 k23 = coarse_key2(__floats2half2_rn(x4.z, x4.w), b2.y);
          kp[cc] = make_uint2(h2_bits(k01), h2_bits(k23));
          a2 = __hmax2(a2, __hmin2(a1, k01));
          a1 = __hmax2(a1, k01);
          a2 = __hmax2(a2, __hmin2(a1, k23));
          a1 = __hmax2(a1, k23);
        }
      }
      const float l1 = __low2float(a1), h1 = __high2float(a1);
      const float l2 = __low2float(a2), h2 = __high2float(a2);
      c1[h] = fmaxf(l1, h1);
      c2[h] = fmaxf(fminf(l1, h1), fmaxf(l2, h2));
    }
    __syncwarp();  // every lane's coarse keys are stored

    // ---- group pick on coarse scores; if the margin is under 4 delta, on
    // fast (then exact) scores of the groups it leaves undecided
    float gs[2] = {c1[0] + c2[0], c1[1] + c2[1]};  // exact in fp32
    float m2v[2] = {c2[0] - dlt, c2[1] - dlt};      // lower bounds of the fast second bests
    bool amb[2] = {false, false};
    bool exact = false;
    bool gsel[2];
    float l0;
    bool coarse_round = true;
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
      if (coarse_round) {
        coarse_round = false;
        if (ghi == -INFINITY || (glo - ghi) > four_d) break;
        // undecided groups: fast scores from the experts within 2 delta of
        // the group's second-best coarse key; decided ones keep their side
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int gg = 2 * q + h;
          if (gs[h] > ghi + four_d) {
            gs[h] = INFINITY;
          } else if (gs[h] < glo - four_d) {
            gs[h] = -INFINITY;
          } else {
            amb[h] = true;
            uint32_t m = coarse_members<GS_MAX>(crow + gg * GS, GS, half2_floor(c2[h] - 2.0f * dlt));
            float e1 = -INFINITY, e2 = -INFINITY;
            for (; m; m &= m - 1) {
              const int e = gg * GS + member_index(__ffs(m) - 1);
              const float k = fast_key(row[e], sbias[e]);
              e2 = fmaxf(e2, fminf(e1, k));
              e1 = fmaxf(e1, k);
            }
            gs[h] = __fadd_rn(e1, e2);
            m2v[h] = e2;
          }
        }
        continue;
      }
      if (exact || ghi == -INFINITY || glo == INFINITY ||
          (glo - ghi) > 4.0f * key_eps(fmaxf(fabsf(glo), fabsf(ghi))))
        break;
      // exact two best of the undecided groups (the same members: delta
      // also bounds coarse against exact keys)
      exact = true;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!amb[h]) continue;
        const int gg = 2 * q + h;
        uint32_t m = coarse_members<GS_MAX>(crow + gg * GS, GS, half2_floor(c2[h] - 2.0f * dlt));
        float e1 = -INFINITY, e2 = -INFINITY;
        for (; m; m &= m - 1) {
          const float ke = quad_exact_key(gx, sbias, gg * GS + member_index(__ffs(m) - 1));
          e2 = fmaxf(e2, fminf(e1, ke));
          e1 = fmaxf(e1, ke);
        }
        gs[h] = __fadd_rn(e1, e2);
        m2v[h] = e2;
      }
    }
    const float thr = l0 - 4.0f * key_eps(fabsf(l0));

    // ---- candidates: fast keys >= thr among coarse keys >= thr - delta of
    // the picked groups; quad lane q scans the q-th (and q + 4-th)
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
    const __half2 cthr = half2_floor(thr - dlt);
    uint32_t cm[2] = {0u, 0u};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (cg[h] < 0) continue;
      for (uint32_t m = coarse_members<GS_MAX>(crow + cg[h] * GS, GS, cthr); m; m &= m - 1) {
        const int bit = __ffs(m) - 1;
        const int e = cg[h] * GS + member_index(bit);
        if (fast_key(row[e], sbias[e]) >= thr) cm[h] |= 1u << bit;
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
    // every lane is done with its token's coarse row: the candidate list
    // takes the row's place
    __syncwarp();
    unsigned long long* tc = reinterpret_cast<unsigned long long*>(crow);
    unsigned long long* ts = sel + t * (K + 1);
    const bool whole = C > kCap;
    if (!whole) {
      int pos = incl - cnt;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (cg[h] < 0) continue;
        for (uint32_t m = cm[h]; m; m &= m - 1) {
          const int e = cg[h] * GS + member_index(__ffs(m) - 1);
          const float v = exact ? quad_exact_key(gx, sbias, e) : fast_key(row[e], sbias[e]);
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

    // ---- weights (as the quad kernel)
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
