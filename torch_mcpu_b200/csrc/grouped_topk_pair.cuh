// grouped_topk for fp32 logits [T, 256], sigmoid scoring with a correction
// bias, 8 groups of 32 experts, topk_group <= 4, topk <= 8 (DeepSeek-V3's
// router) on large batches: the pair kernel (included by grouped_topk.cu).
//
// Work split.  Two lanes serve one token: lane t (< 16) owns groups 0-3 and
// lane t + 16 groups 4-7 of token t of the warp's tile, so a warp routes 16
// tokens and all per-token work is per-lane register arithmetic plus a
// handful of shuffles between the two halves of the warp.  Each warp owns
// one 16 KB shared-memory slot, filled by eight TMA boxes [16 tokens x 32
// experts] (one per group) with the 128-byte swizzle, so a lane reads its
// row 16 bytes at a time with the eight lanes of each access phase on
// distinct banks.  One CTA of fourteen warps per SM (14 x 16 KB); the slot
// goes back to TMA as soon as the tile's candidates are extracted.  Waits
// are bounded; warps never wait for one another.
//
// Per token:
//   keys    every fast key sigmoid_fast(x) + bias (two at a time with the
//           packed f32x2 multiply and adds, bit-identical to the scalar
//           form) is computed once and written over its logit; each group's
//           two best keys stay in registers (3-input max);
//   groups  the two lanes swap their four group scores; each ranks all eight
//           (ties to the lower group index) and picks topk_group;
//   experts L0 = smallest second-best key of the picked groups; the picked
//           groups hold 2 * topk_group >= topk keys >= L0, so only keys >=
//           thr = L0 - 4 eps are candidates (about 11 per token).  Each lane
//           scans two of the picked groups and inserts its candidates into a
//           sorted register list of topk + 1 packed keys (bits(key - thr)
//           with the low 8 bits replaced by 255 - expert: ties go to the
//           lower expert); the lanes then merge their lists;
//   exactness fast keys are within eps = 2^-21 + 2^-22 |key| of the
//           reference's fp32 keys.  The group pick is certified by a margin
//           over 4 eps; the topk-th / (topk+1)-th boundary by the packed
//           list: the two entries must lie in different truncation buckets
//           whose edges are more than 4 eps (plus the rounding of key - thr)
//           apart.  A token that fails either test is picked again by the
//           whole warp on exact keys (the reference's sigmoid, correctly
//           rounded exp) of all 256 experts, eight per lane, after the tile;
//   weights the sigmoid of each pick is recovered from its fast key (key -
//           bias) or recomputed; renormalised and scaled.
#pragma once

#include "sm100.cuh"

namespace mcpu {
namespace router {

constexpr int kPairWarps = 14;   // one CTA per SM, 14 x 16 KB slots
constexpr int kPairTokens = 16;  // tokens per warp tile; lanes t and t + 16 share token t
constexpr int kPairE = 256, kPairGS = 32, kPairG = 8;
constexpr int kPairTile = kPairTokens * kPairE * 4;  // 16384 bytes
constexpr int kPairBox = kPairTokens * kPairGS * 4;  // one group box, 2048 bytes
constexpr int kPairTGMax = 4, kPairKMax = 8;
constexpr int kPairList = kPairKMax + 1;

struct PairLayout {
  int bias_off, bar_off, total;
};

// [slots: warps x 16 KB, 1024-byte aligned][bias 1 KB][per warp: mbarrier,
// abort flag]; `total` includes the alignment slack of the dynamic base.
__host__ __device__ constexpr PairLayout pair_layout(int warps) {
  return PairLayout{warps * kPairTile, warps * kPairTile + kPairE * 4,
                    1024 + warps * kPairTile + kPairE * 4 + warps * 16};
}

// Byte offset of expert (g, j) in the row at `rowoff` (swizzle x7): box g,
// 16-byte chunk j / 4 stored at chunk (j / 4) ^ (row % 8).
__device__ __forceinline__ int pair_elem_off(int rowoff, int x7, int g, int j) {
  return g * kPairBox + rowoff + ((((j >> 2) << 4) ^ x7)) + ((j & 3) << 2);
}

// Two fast keys: fl(rcp.approx(fl(1 + ex2.approx(fl(x * -log2 e)))) + b) for
// each half, with the multiply and the adds as packed f32x2 operations (one
// rounding each, as __fmul_rn / __fadd_rn).
__device__ __forceinline__ void fast_key2(float x0, float x1, float b0, float b1, float& k0, float& k1) {
  asm("{\n\t"
      ".reg .b64 v, c;\n\t"
      ".reg .f32 e0, e1;\n\t"
      "mov.b64 v, {%2, %3};\n\t"
      "mov.b64 c, {%6, %6};\n\t"
      "mul.rn.f32x2 v, v, c;\n\t"
      "mov.b64 {e0, e1}, v;\n\t"
      "ex2.approx.ftz.f32 e0, e0;\n\t"
      "ex2.approx.ftz.f32 e1, e1;\n\t"
      "mov.b64 v, {e0, e1};\n\t"
      "mov.b64 c, {%7, %7};\n\t"
      "add.rn.f32x2 v, v, c;\n\t"
      "mov.b64 {e0, e1}, v;\n\t"
      "rcp.approx.ftz.f32 e0, e0;\n\t"
      "rcp.approx.ftz.f32 e1, e1;\n\t"
      "mov.b64 v, {e0, e1};\n\t"
      "mov.b64 c, {%4, %5};\n\t"
      "add.rn.f32x2 v, v, c;\n\t"
      "mov.b64 {%0, %1}, v;\n\t"
      "}"
      : "=f"(k0), "=f"(k1)
      : "f"(x0), "f"(x1), "f"(b0), "f"(b1), "f"(-1.4426950408889634f), "f"(1.0f));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// (m1, m2) = the two largest of {m1, m2, k0..k3}, m1 >= m2.
__device__ __forceinline__ void top2_add4(float& m1, float& m2, float k0, float k1, float k2, float k3) {
  const float a = fmaxf(k0, k1), b = fminf(k0, k1), c = fmaxf(k2, k3), d = fminf(k2, k3);
  const float t1 = fmaxf(a, c), t2 = max3f(fminf(a, c), b, d);
  m2 = max3f(fminf(m1, t1), m2, t2);
  m1 = fmaxf(m1, t1);
}

// Inserts v into the descending list (the last entry drops out): slot i
// becomes max(L[i], min(L[i - 1], v)), every slot from the old list, so the
// update is two operations deep.
__device__ __forceinline__ void list_insert(uint32_t (&lst)[kPairList], uint32_t v) {
  uint32_t n[kPairList];
  n[0] = max(lst[0], v);
#pragma unroll
  for (int i = 1; i < kPairList; ++i) n[i] = max(lst[i], min(lst[i - 1], v));
#pragma unroll
  for (int i = 0; i < kPairList; ++i) lst[i] = n[i];
}

// 64-bit max across the warp (butterfly).
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, v, off);
    v = o > v ? o : v;
  }
  return v;
}

// The whole pick of one token on exact keys, by the whole warp: lane l
// evaluates experts 8l .. 8l + 7 (group l / 4) with the reference's sigmoid;
// group scores are the sums of each group's two best exact keys, ranked
// with ties to the lower group; then topk rounds of a warp arg-max over the
// picked groups' packed (key, inverted index) pairs.  Writes the token's
// outputs.
__device__ __noinline__ void pair_warp_exact_pick(const float* gx, const float* sbias, int TG, int K, int renorm,
                                                  float scale, float* w_out, int32_t* id_out, long long token,
                                                  int lane) {
  const float4 xa = __ldg(reinterpret_cast<const float4*>(gx) + 2 * lane);
  const float4 xb = __ldg(reinterpret_cast<const float4*>(gx) + 2 * lane + 1);
  const float x[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
  float sg[8], key[8];
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    sg[u] = sigmoid_exact(x[u]);
    key[u] = __fadd_rn(sg[u], sbias[8 * lane + u]);
    m2 = fmaxf(m2, fminf(m1, key[u]));
    m1 = fmaxf(m1, key[u]);
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    const float o1 = __shfl_xor_sync(0xFFFFFFFFu, m1, off);
    const float o2 = __shfl_xor_sync(0xFFFFFFFFu, m2, off);
    m2 = max3f(fminf(m1, o1), m2, o2);
    m1 = fmaxf(m1, o1);
  }
  const float gsc = __fadd_rn(m1, m2);
  const int g = lane >> 2;
  int r = 0;
#pragma unroll
  for (int j = 0; j < kPairG; ++j) {
    const float o = __shfl_sync(0xFFFFFFFFu, gsc, 4 * j);
    r += (o > gsc) || (o == gsc && j < g);
  }
  const bool sel = r < TG;
  unsigned long long pk[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) pk[u] = sel ? pack_key(key[u], 8 * lane + u) : 0ull;
  float myw = 0.0f;
  int myid = 0;
  for (int k = 0; k < K; ++k) {
    unsigned long long best = 0ull;
    float bsg = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (pk[u] > best) {
        best = pk[u];
        bsg = sg[u];
      }
    }
    const unsigned long long win = warp_max_u64(best);
    const int idx = packed_index(win);
    const float wsg = __shfl_sync(0xFFFFFFFFu, bsg, idx >> 3);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (pk[u] == win) pk[u] = 0ull;
    if (lane == k) {
      myw = wsg;
      myid = idx;
    }
  }
  float sum = 0.0f;
  for (int k = 0; k < K; ++k) sum = __fadd_rn(sum, __shfl_sync(0xFFFFFFFFu, myw, k));
  if (lane < K) {
    float w = myw;
    if (renorm) w = __fdiv_rn(w, sum);
    if (scale != 1.0f) w = __fmul_rn(w, scale);
    w_out[token * K + lane] = w;
    id_out[token * K + lane] = myid;
  }
}

template <int NW>
__global__ void __launch_bounds__(NW * 32, 1) grouped_topk_pair_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const long long wtiles, const int vec_out) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t ra = sm100::smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (ra & 1023)) & 1023);
  constexpr PairLayout L = pair_layout(NW);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  char* tb = reinterpret_cast<char*>(base + warp * kPairTile);
  float* sbias = reinterpret_cast<float*>(base + L.bias_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_off + warp * 16);
  int* abort_flag = reinterpret_cast<int*>(base + L.bar_off + warp * 16 + 8);

  const int TG = p.TG, K = p.K;
  const int t = lane & 15;          // token of the tile
  const int h = lane >> 4;          // half: groups 4h .. 4h + 3
  const int rowoff = t * 128;       // the token's row in every group box
  const int x7 = (t & 7) << 4;      // its 128-byte swizzle
  const long long gw = static_cast<long long>(blockIdx.x) * NW + warp;
  const long long nw = static_cast<long long>(gridDim.x) * NW;
  const float* gating = static_cast<const float*>(p.gating);

  // lane 0 arms the barrier, lanes 0..7 each load one group box
  auto issue = [&](long long wt) {
    if (lane == 0) sm100::mbar_arrive_expect_tx(full, kPairTile);
    __syncwarp();
    if (lane < kPairG)
      sm100::tma_load_2d(tb + lane * kPairBox, &tm, full, lane * kPairGS, static_cast<int>(wt * kPairTokens));
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

    const long long token = wt * kPairTokens + t;
    const bool valid = token < p.T;

    // ---- keys of this lane's four groups, written over the logits (chunk
    // by chunk across the four groups: four independent top-2 chains)
    float gsh[4], m2h[4];
    {
      char* hb = tb + h * 4 * kPairBox + rowoff;
      const float* bh = sbias + h * 4 * kPairGS;
      float m1[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      float m2v[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kPairGS / 4; ++c) {
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          float4* px = reinterpret_cast<float4*>(hb + gg * kPairBox + ((c << 4) ^ x7));
          const float4 x4 = *px;
          const float4 b4 = *reinterpret_cast<const float4*>(bh + gg * kPairGS + c * 4);
          float4 k4;
          fast_key2(x4.x, x4.y, b4.x, b4.y, k4.x, k4.y);
          fast_key2(x4.z, x4.w, b4.z, b4.w, k4.z, k4.w);
          *px = k4;
          top2_add4(m1[gg], m2v[gg], k4.x, k4.y, k4.z, k4.w);
        }
      }
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        m2h[gg] = m2v[gg];
        gsh[gg] = __fadd_rn(m1[gg], m2v[gg]);
      }
    }
    // ---- the two lanes swap their group scores; group pick (ties to the
    // lower group), certified by a margin over 4 eps
    float gs[kPairG], m2[kPairG];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float og = __shfl_xor_sync(0xFFFFFFFFu, gsh[i], 16);
      const float om = __shfl_xor_sync(0xFFFFFFFFu, m2h[i], 16);
      gs[i] = h ? og : gsh[i];
      gs[4 + i] = h ? gsh[i] : og;
      m2[i] = h ? om : m2h[i];
      m2[4 + i] = h ? m2h[i] : om;
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
    bool slow = !(ghi == -INFINITY || (glo - ghi) > 4.0f * key_eps(fmaxf(fabsf(glo), fabsf(ghi))));
    const float thr = l0 - 4.0f * key_eps(fabsf(l0));

    // ---- candidates of this lane's picked groups (the 2h-th and 2h+1-th)
    uint32_t cm[2] = {0u, 0u};
    int cg[2] = {0, 0};
    {
      uint32_t rest = selbits;
      if (h) {
        rest &= rest - 1;
        rest &= rest - 1;
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (rest != 0u && 2 * h + j < TG) {  // (rest runs dry only on NaN scores)
          const int g = __ffs(rest) - 1;
          rest &= rest - 1;
          cg[j] = g;
          const char* gp = tb + g * kPairBox + rowoff;
          uint32_t m = 0u;
#pragma unroll
          for (int c = 0; c < kPairGS / 4; ++c) {
            const float4 k4 = *reinterpret_cast<const float4*>(gp + ((c << 4) ^ x7));
            m |= ((k4.x >= thr ? 1u : 0u) | (k4.y >= thr ? 2u : 0u) | (k4.z >= thr ? 4u : 0u) |
                  (k4.w >= thr ? 8u : 0u))
                 << (4 * c);
          }
          cm[j] = m;
        }
      }
    }
    const int own = __popc(cm[0]) + __popc(cm[1]);
    const int C = own + __shfl_xor_sync(0xFFFFFFFFu, own, 16);

    // ---- sorted list of the K + 1 best packed keys: own candidates, then
    // the partner's list merged in
    uint32_t lst[kPairList];
#pragma unroll
    for (int i = 0; i < kPairList; ++i) lst[i] = 0u;
    {
      unsigned long long mm = slow ? 0ull : (cm[0] | (static_cast<unsigned long long>(cm[1]) << 32));
      while (mm) {
        const int i = __ffsll(mm) - 1;
        mm &= mm - 1;
        const int g = i < 32 ? cg[0] : cg[1];
        const int j = i & 31;
        const float key = *reinterpret_cast<const float*>(tb + pair_elem_off(rowoff, x7, g, j));
        list_insert(lst, (__float_as_uint(__fsub_rn(key, thr)) & ~255u) |
                             static_cast<uint32_t>(255 - (g * kPairGS + j)));
      }
    }
    // merge with the partner's list: the picks (K of them) in pk[0 .. K-1]
    // (any order), and the K-th / (K+1)-th best packed keys lk, ln
    uint32_t pk[kPairKMax];
    uint32_t lk, ln;
    {
      uint32_t o[kPairList];
#pragma unroll
      for (int i = 0; i < kPairList; ++i) o[i] = __shfl_xor_sync(0xFFFFFFFFu, lst[i], 16);
      if (K == kPairKMax) {
        // both lists descending: c[i] = max(A[i], B[8 - i]) is the best nine
        // of the union (in bitonic order); the ninth is its minimum, the
        // eighth the minimum of the rest
        // (both lanes orient it the same way, lane t's list first, so that
        // the two halves take their picks from the same order)
        uint32_t c[kPairList];
#pragma unroll
        for (int i = 0; i < kPairList; ++i)
          c[i] = max(h ? o[i] : lst[i], h ? lst[kPairList - 1 - i] : o[kPairList - 1 - i]);
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
      } else {
#pragma unroll
        for (int i = 0; i < kPairList; ++i) list_insert(lst, o[i]);
        lk = lst[0];
        ln = lst[0];
#pragma unroll
        for (int i = 0; i < kPairList; ++i) {
          if (i == K - 1) lk = lst[i];
          if (i == K) ln = lst[i];
        }
#pragma unroll
        for (int i = 0; i < kPairKMax; ++i) pk[i] = lst[i];
      }
    }
    // the K-th / (K+1)-th boundary, from the truncation buckets' edges in
    // key - thr space: every pick is >= lo, every other candidate <= hi
    if (!slow && C > K) {
      bool cert = false;
      if ((lk >> 8) > (ln >> 8)) {
        const float lo = __uint_as_float(lk & ~255u), hi = __uint_as_float(ln | 255u);
        cert = (lo - hi) > 4.0f * key_eps(fabsf(thr) + lo) + 0x1p-22f * (lo + hi);
      }
      slow = !cert;
    }
    // this lane's picks 4h .. 4h + 3, and their fast keys (read before the
    // slot is handed back)
    int pid[4];
    float pkv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t e8 = h ? pk[4 + u] : pk[u];
      pid[u] = 255 - static_cast<int>(e8 & 255u);
      pkv[u] = *reinterpret_cast<const float*>(tb + pair_elem_off(rowoff, x7, pid[u] >> 5, pid[u] & 31));
    }

    // ---- the slot is no longer needed: hand it to the next tile
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    {
      const long long nt = wt + nw;
      if (nt < wtiles) issue(nt);
      inflight = nt < wtiles;
    }

    // ---- weights: sigmoid = key - bias within 2^-20 relative while it is
    // at least |key| / 16, else recomputed from the logit
    const float* gx = gating + (valid ? token : 0) * static_cast<long long>(kPairE);
    float wv[4];
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      wv[u] = 0.0f;
      if (4 * h + u < K) {
        float sg = __fsub_rn(pkv[u], sbias[pid[u]]);
        if (!slow && !(sg >= 0.0625f * fabsf(pkv[u]))) sg = quad_weight_sigmoid(__ldg(gx + pid[u]));
        wv[u] = sg;
        sum = __fadd_rn(sum, sg);
      }
    }
    {
      const float other = __shfl_xor_sync(0xFFFFFFFFu, sum, 16);
      sum = h ? __fadd_rn(other, sum) : __fadd_rn(sum, other);
    }
    if (valid && !slow) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float w = wv[u];
        if (p.renorm) w = __fdiv_rn(w, sum);
        if (p.scale != 1.0f) w = __fmul_rn(w, p.scale);
        wv[u] = w;
      }
      if (vec_out) {  // K == 8, 16-byte aligned outputs: 4 weights and 4 ids per lane
        reinterpret_cast<float4*>(p.w_out + token * 8)[h] = make_float4(wv[0], wv[1], wv[2], wv[3]);
        reinterpret_cast<int4*>(p.id_out + token * 8)[h] = make_int4(pid[0], pid[1], pid[2], pid[3]);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (4 * h + u < K) {
            p.w_out[token * K + 4 * h + u] = wv[u];
            p.id_out[token * K + 4 * h + u] = pid[u];
          }
        }
      }
    }

    // ---- tokens without both certificates: picked again on exact keys by
    // the whole warp
    unsigned pending = __ballot_sync(0xFFFFFFFFu, slow && valid && h == 0);
    while (pending) {
      const int src = __ffs(pending) - 1;
      pending &= pending - 1;
      const long long tok = wt * kPairTokens + src;
      pair_warp_exact_pick(gating + tok * kPairE, sbias, TG, K, p.renorm, p.scale, p.w_out, p.id_out, tok, lane);
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
