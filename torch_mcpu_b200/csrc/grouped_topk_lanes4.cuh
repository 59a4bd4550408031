// grouped_topk for fp32 logits [T, 256], sigmoid scoring with a correction
// bias, 8 groups of 32 experts, topk_group <= 4, topk == 8 (DeepSeek-V3's
// router): the four-lane kernel (included by grouped_topk.cu, after
// grouped_topk_pair.cuh, whose helpers it shares).
//
// Work split.  Four lanes serve one token: lane t + 8q (t < 8, q < 4) owns
// groups 2q and 2q + 1 of token t of the warp's tile, so a warp routes 8
// tokens.  Each warp owns one 8 KB shared-memory slot, filled by eight TMA
// boxes [8 tokens x 32 experts] (one per group, one 128-byte swizzle atom
// each); one CTA of NW warps per SM.  Against two lanes per token this
// halves each warp's serial work per tile and doubles the warps per SM,
// which is what the router's time depends on: each tile is a chain of
// dependent steps, and more warps hide more of it.  Waits are bounded;
// warps never wait for one another.
//
// Per token:
//   keys    every fast key sigmoid_fast(x) + bias (packed f32x2 arithmetic)
//           is computed once and written over its logit; each group's two
//           best keys stay in registers;
//   groups  every lane gathers the eight group scores (shuffles) and picks
//           topk_group groups, ties to the lower group;
//   experts thr = L0 - 4 eps as in the two-lane kernel; lane q scans the
//           q-th picked group into a 32-bit candidate mask; the lanes of a
//           pair (q, q ^ 1) swap masks, so both insert the candidates of
//           both groups into the same sorted list of nine packed keys; the
//           two pairs' lists are then merged in one bitonic step;
//   exactness the same two certificates (group margin, K-th / K+1-th bucket
//           edges).  After the tile the whole warp takes each uncertified
//           token: one exact key per lane and a bitonic sort when only the
//           expert boundary is open (l4_warp_rerank), else the exact pick
//           over all 256 experts (pair_warp_exact_pick);
//   weights lane q weighs picks 2q and 2q + 1; the sum over the four lanes
//           is taken in a fixed order.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kL4Tokens = 8;                        // tokens per warp tile
constexpr int kL4Tile = kL4Tokens * kPairE * 4;     // 8192 bytes
constexpr int kL4Box = kL4Tokens * kPairGS * 4;     // one group box, 1024 bytes

struct L4Layout {
  int bias_off, bar_off, total;
};

__host__ __device__ constexpr L4Layout l4_layout(int warps) {
  return L4Layout{warps * kL4Tile, warps * kL4Tile + kPairE * 4, 1024 + warps * kL4Tile + kPairE * 4 + warps * 16};
}

// Byte offset of expert (g, j) of the row at `rowoff` (swizzle x7).
__device__ __forceinline__ int l4_elem_off(int rowoff, int x7, int g, int j) {
  return g * kL4Box + rowoff + ((((j >> 2) << 4) ^ x7)) + ((j & 3) << 2);
}

// Position of the (n + 1)-th set bit of m (popc(m) > n).
__device__ __forceinline__ int nth_set_bit(uint32_t m, int n) {
  int pos = 0;
#pragma unroll
  for (int w = 16; w > 0; w >>= 1) {
    const uint32_t low = m & ((1u << w) - 1u);
    const int c = __popc(low);
    const bool up = n >= c;
    n = up ? n - c : n;
    m = up ? (m >> w) : low;
    pos += up ? w : 0;
  }
  return pos;
}

// A token whose group pick is certified but whose K-th / (K+1)-th boundary
// is not, re-ranked by the whole warp: lane l takes the l-th of its
// C <= 32 candidates (masks m[0..3] of the picked groups g[0..3], whose
// fast keys reach thr, so they hold the exact top K), evaluates its exact
// key (the reference's sigmoid of the logit, plus bias), and a bitonic sort
// of the 32 packed (key, inverted index) pairs leaves the exact top K in
// lanes 0 .. K - 1.  Writes the token's outputs.
__device__ __noinline__ void l4_warp_rerank(const float* gx, const float* sbias, const uint32_t (&m)[4],
                                            const int (&g)[4], int C, int renorm, float scale, float* w_out,
                                            int32_t* id_out, long long token, int lane) {
  unsigned long long key = 0ull;
  float sg = 0.0f;
  if (lane < C) {
    int n = lane, k = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int c = __popc(m[i]);
      if (k == i && n >= c) {
        n -= c;
        k = i + 1;
      }
    }
    const uint32_t mk = k == 0 ? m[0] : k == 1 ? m[1] : k == 2 ? m[2] : m[3];
    const int gk = k == 0 ? g[0] : k == 1 ? g[1] : k == 2 ? g[2] : g[3];
    const int e = gk * kPairGS + nth_set_bit(mk, n);
    sg = sigmoid_exact(__ldg(gx + e));
    key = pack_key(__fadd_rn(sg, sbias[e]), e);
  }
  // bitonic sort, descending over the lanes
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long ok = __shfl_xor_sync(0xFFFFFFFFu, key, j);
      const float osg = __shfl_xor_sync(0xFFFFFFFFu, sg, j);
      const bool desc = (lane & k) == 0;
      const bool low = (lane & j) == 0;
      const bool take = (low == desc) ? (ok > key) : (ok < key);
      key = take ? ok : key;
      sg = take ? osg : sg;
    }
  }
  float sum = 0.0f;
  for (int i = 0; i < kPairKMax; ++i) sum = __fadd_rn(sum, __shfl_sync(0xFFFFFFFFu, sg, i));
  if (lane < kPairKMax) {
    float w = sg;
    if (renorm) w = __fdiv_rn(w, sum);
    if (scale != 1.0f) w = __fmul_rn(w, scale);
    w_out[token * kPairKMax + lane] = w;
    id_out[token * kPairKMax + lane] = packed_index(key);
  }
}

template <int NW>
__global__ void __launch_bounds__(NW * 32, 1) grouped_topk_lanes4_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const long long wtiles, const int vec_out) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (ra & 1023)) & 1023);
  constexpr L4Layout L = l4_layout(NW);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  char* tb = reinterpret_cast<char*>(base + warp * kL4Tile);
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_off + warp * 16);
  int* abort_flag = reinterpret_cast<int*>(base + L.bar_off + warp * 16 + 8);

  const int TG = p.TG;
  const int t = lane & 7;         // token of the tile
  const int q = lane >> 3;        // quarter: groups 2q, 2q + 1
  const int rowoff = t * 128;     // the token's row in every group box
  const int x7 = t << 4;          // its 128-byte swizzle (row t of the atom)
  const long long gw = static_cast<long long>(blockIdx.x) * NW + warp;
  const long long nw = static_cast<long long>(gridDim.x) * NW;
  const float* gating = static_cast<const float*>(p.gating);

  auto issue = [&](long long wt) {
    if (lane == 0) sm100::mbar_arrive_expect_tx(full, kL4Tile);
    __syncwarp();
    if (lane < kPairG)
      sm100::tma_load_2d(tb + lane * kL4Box, &tm, full, lane * kPairGS, static_cast<int>(wt * kL4Tokens));
  };

  if (lane == 0) {
    sm100::mbar_init(full, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  __syncwarp();
  if (gw < wtiles) issue(gw);
  for (int i = threadIdx.x; i < kPairE; i += blockDim.x) sbias[i] = p.bias[i];
  __syncthreads();  // the only CTA-wide barrier: bias staged

  long long it = 0;
  bool inflight = gw < wtiles;
  for (;; ++it) {
    const long long wt = gw + it * nw;
    if (wt >= wtiles) break;
    const bool ok = sm100::mbar_wait(full, static_cast<uint32_t>(it & 1), abort_flag);
    if (!__all_sync(0xFFFFFFFFu, ok)) break;
    inflight = false;

    const long long token = wt * kL4Tokens + t;
    const bool valid = token < p.T;

    // ---- keys of this lane's two groups, written over the logits
    float gs2[2], m22[2];
    {
      char* qb = tb + 2 * q * kL4Box + rowoff;
      const float* bq = sbias + 2 * q * kPairGS;
      float m1[2] = {-INFINITY, -INFINITY};
      float m2v[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kPairGS / 4; ++c) {
#pragma unroll
        for (int gg = 0; gg < 2; ++gg) {
          float4* px = reinterpret_cast<float4*>(qb + gg * kL4Box + ((c << 4) ^ x7));
          const float4 x4 = *px;
          const float4 b4 = *reinterpret_cast<const float4*>(bq + gg * kPairGS + c * 4);
          float4 k4;
          fast_key2(x4.x, x4.y, b4.x, b4.y, k4.x, k4.y);
          fast_key2(x4.z, x4.w, b4.z, b4.w, k4.z, k4.w);
          *px = k4;
          top2_add4(m1[gg], m2v[gg], k4.x, k4.y, k4.z, k4.w);
        }
      }
#pragma unroll
      for (int gg = 0; gg < 2; ++gg) {
        m22[gg] = m2v[gg];
        gs2[gg] = __fadd_rn(m1[gg], m2v[gg]);
      }
    }
    // ---- all eight group scores (lane t + 8j holds groups 2j, 2j + 1);
    // group pick, ties to the lower group, certified by a margin over 4 eps
    float gs[kPairG], m2[kPairG];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        gs[2 * j + h] = __shfl_sync(0xFFFFFFFFu, gs2[h], t + 8 * j);
        m2[2 * j + h] = __shfl_sync(0xFFFFFFFFu, m22[h], t + 8 * j);
      }
    }
    uint32_t selbits = 0;
    float l0 = INFINITY, glo = INFINITY, ghi = -INFINITY;
#pragma unroll
    for (int g = 0; g < kPairG; ++g) {
      int r = 0;
#pragma unroll
      for (int j = 0; j < kPairG; ++j) {
        if (j == g) continue;
        r += (j < g) ? (gs[j] >= gs[g]) : (gs[j] > gs[g]);
      }
      if (r < TG) {
        selbits |= 1u << g;
        glo = fminf(glo, gs[g]);
        l0 = fminf(l0, m2[g]);
      } else {
        ghi = fmaxf(ghi, gs[g]);
      }
    }
    const bool gslow = !(ghi == -INFINITY || (glo - ghi) > 4.0f * key_eps(fmaxf(fabsf(glo), fabsf(ghi))));
    bool slow = gslow;
    const float thr = l0 - 4.0f * key_eps(fabsf(l0));

    // ---- candidates of the q-th picked group; the pair (q, q ^ 1) swaps masks
    uint32_t cm = 0u;
    int cg = 0;
    {
      uint32_t rest = selbits;
#pragma unroll
      for (int i = 0; i < 3; ++i)
        if (i < q) rest &= rest - 1;
      if (rest != 0u && q < TG) {  // (rest runs dry only on NaN scores)
        cg = __ffs(rest) - 1;
        const char* gp = tb + cg * kL4Box + rowoff;
#pragma unroll
        for (int c = 0; c < kPairGS / 4; ++c) {
          const float4 k4 = *reinterpret_cast<const float4*>(gp + ((c << 4) ^ x7));
          cm |= ((k4.x >= thr ? 1u : 0u) | (k4.y >= thr ? 2u : 0u) | (k4.z >= thr ? 4u : 0u) |
                 (k4.w >= thr ? 8u : 0u))
                << (4 * c);
        }
      }
    }
    const uint32_t ocm = __shfl_xor_sync(0xFFFFFFFFu, cm, 8);
    const int ocg = __shfl_xor_sync(0xFFFFFFFFu, cg, 8);
    const int pairc = __popc(cm) + __popc(ocm);
    const int C = pairc + __shfl_xor_sync(0xFFFFFFFFu, pairc, 16);

    // ---- the pair's sorted list of nine packed keys, then the two pairs'
    // lists merged in one bitonic step (lanes < 16 first, so every lane of
    // the token sees the same order)
    uint32_t lst[kPairList];
#pragma unroll
    for (int i = 0; i < kPairList; ++i) lst[i] = 0u;
    {
      unsigned long long mm = slow ? 0ull : (cm | (static_cast<unsigned long long>(ocm) << 32));
      while (mm) {
        const int i = __ffsll(mm) - 1;
        mm &= mm - 1;
        const int g = i < 32 ? cg : ocg;
        const int j = i & 31;
        const float key = *reinterpret_cast<const float*>(tb + l4_elem_off(rowoff, x7, g, j));
        list_insert(lst, (__float_as_uint(__fsub_rn(key, thr)) & ~255u) |
                             static_cast<uint32_t>(255 - (g * kPairGS + j)));
      }
    }
    uint32_t pk[kPairKMax];
    uint32_t lk, ln;
    {
      const bool lo = q < 2;
      uint32_t o[kPairList], c[kPairList];
#pragma unroll
      for (int i = 0; i < kPairList; ++i) o[i] = __shfl_xor_sync(0xFFFFFFFFu, lst[i], 16);
#pragma unroll
      for (int i = 0; i < kPairList; ++i)
        c[i] = max(lo ? lst[i] : o[i], lo ? o[kPairList - 1 - i] : lst[kPairList - 1 - i]);
      uint32_t mn = c[0];
#pragma unroll
      for (int i = 1; i < kPairList; ++i) mn = min(mn, c[i]);
      uint32_t sm = 0xFFFFFFFFu;
#pragma unroll
      for (int i = 0; i < kPairList; ++i) sm = min(sm, c[i] == mn ? 0xFFFFFFFFu : c[i]);
      ln = mn;
      lk = sm;
#pragma unroll
      for (int i = 0; i < kPairKMax; ++i) pk[i] = c[i] == mn ? c[kPairList - 1] : c[i];
    }
    if (!slow && C > kPairKMax) {
      bool cert = false;
      if ((lk >> 8) > (ln >> 8)) {
        const float lo = __uint_as_float(lk & ~255u), hi = __uint_as_float(ln | 255u);
        cert = (lo - hi) > 4.0f * key_eps(fabsf(thr) + lo) + 0x1p-22f * (lo + hi);
      }
      slow = !cert;
    }
    // this lane's picks 2q, 2q + 1 and their fast keys
    int pid[2];
    float pkv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t e8 = q == 0 ? pk[u] : q == 1 ? pk[2 + u] : q == 2 ? pk[4 + u] : pk[6 + u];
      pid[u] = 255 - static_cast<int>(e8 & 255u);
      pkv[u] = *reinterpret_cast<const float*>(tb + l4_elem_off(rowoff, x7, pid[u] >> 5, pid[u] & 31));
    }

    // ---- the slot is no longer needed: hand it to the next tile
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    {
      const long long nt = wt + nw;
      if (nt < wtiles) issue(nt);
      inflight = nt < wtiles;
    }

    // ---- weights; the sum over the four lanes in a fixed order
    const float* gx = gating + (valid ? token : 0) * static_cast<long long>(kPairE);
    float wv[2];
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float sg = __fsub_rn(pkv[u], sbias[pid[u]]);
      if (!slow && !(sg >= 0.0625f * fabsf(pkv[u]))) sg = quad_weight_sigmoid(__ldg(gx + pid[u]));
      wv[u] = sg;
      sum = __fadd_rn(sum, sg);
    }
    sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, 8));
    sum = __fadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, 16));
    if (valid && !slow) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float w = wv[u];
        if (p.renorm) w = __fdiv_rn(w, sum);
        if (p.scale != 1.0f) w = __fmul_rn(w, p.scale);
        wv[u] = w;
      }
      if (vec_out) {  // 8-byte aligned outputs: two weights and two ids per lane
        reinterpret_cast<float2*>(p.w_out + token * 8)[q] = make_float2(wv[0], wv[1]);
        reinterpret_cast<int2*>(p.id_out + token * 8)[q] = make_int2(pid[0], pid[1]);
      } else {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          p.w_out[token * 8 + 2 * q + u] = wv[u];
          p.id_out[token * 8 + 2 * q + u] = pid[u];
        }
      }
    }

    // ---- tokens without both certificates, by the whole warp: re-ranked on
    // exact keys of their candidates when only the K-th / (K+1)-th boundary
    // is open, else picked again on exact keys of all 256 experts
    unsigned pending = __ballot_sync(0xFFFFFFFFu, slow && valid && q == 0);
    while (pending) {
      const int src = __ffs(pending) - 1;
      pending &= pending - 1;
      const long long tok = wt * kL4Tokens + src;
      const bool whole = __shfl_sync(0xFFFFFFFFu, gslow, src) || __shfl_sync(0xFFFFFFFFu, C, src) > 32;
      if (whole) {
        pair_warp_exact_pick(gating + tok * kPairE, sbias, TG, kPairKMax, p.renorm, p.scale, p.w_out, p.id_out,
                             tok, lane);
      } else {
        uint32_t tm4[4];
        int tg4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          tm4[i] = __shfl_sync(0xFFFFFFFFu, cm, src + 8 * i);
          tg4[i] = __shfl_sync(0xFFFFFFFFu, cg, src + 8 * i);
        }
        l4_warp_rerank(gating + tok * kPairE, sbias, tm4, tg4, __shfl_sync(0xFFFFFFFFu, C, src), p.renorm,
                       p.scale, p.w_out, p.id_out, tok, lane);
      }
      if (lane == 0) atomicAdd(&g_exact_rows, 1ull);
    }
  }

  if (lane == 0 && *abort_flag) {
    // a wait ran out: record it, then let this warp's copy in flight land
    atomicExch(&g_router_error, 1);
    if (inflight) {
      for (uint32_t n = 0; n < sm100::kSpinLimit && !sm100::mbar_try_wait(full, static_cast<uint32_t>(it & 1));
           ++n) {
      }
    }
  }
}

}  // namespace router
}  // namespace mcpu
