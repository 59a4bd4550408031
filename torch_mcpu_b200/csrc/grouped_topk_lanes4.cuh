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
//
// Expert dispatch in the same launch (kDispatch): the outputs of vLLM's
// moe_align_block_size (vllm/_custom_ops.py:2247-2264) for the ids the
// launch writes, with every expert's run in ascending flat index.  Each CTA
// then routes one contiguous range of tiles, each warp a contiguous run of
// it (its slice of ids), and:
//   1. each warp, right after its last tile, counts its slice per expert in
//      the first 1 KB of its own slot (ids re-read from L2 and kept in
//      registers);
//   2. the CTA publishes its expert counts: one row of 16-bit counts, and a
//      red.add into the sum of its group of 16 CTAs;
//   3. one grid-wide barrier (cooperative launch; release-add arrival,
//      bounded acquire wait); meanwhile the CTA sorts its own entries by
//      expert into a staging buffer in shared memory: per-warp offsets plus
//      the ranks the counting pass's atomics returned (one token at a time,
//      so in index order);
//   4. expert totals from the group sums, the entries of earlier CTAs from
//      the earlier groups' sums and this group's earlier rows (at most
//      groups + 15 loads per expert pair); a scan of the padded totals gives
//      the run starts;
//   5. the grid writes the run padding, the tail and the block experts;
//      each CTA copies its sorted entries out, every expert's entries in
//      one contiguous run.
#pragma once

#include "peer.cuh"
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

// ---------------------------------------------------------------------------
// Expert dispatch fused into the router.
//
// Workspace, in 32-bit words:
//   [0]        generation, bumped once per launch (any start value); its
//              parity picks the arrival count and group sums of the launch
//   [1], [2]   arrival counts of even / odd generations
//   [32, ...)  group sums [2 parities][groups][256], one group per 16 CTAs
//   then       rows [CTAs][128]: each CTA's expert counts, two 16-bit
//              counts per word
// Everything before the rows is zero before the first launch; a launch
// clears the other parity's count and group sums for the next one.
constexpr int kDispatchHeaderWords = 32;
constexpr int kDispatchGroup = 16;  // CTAs per group sum

__host__ __device__ constexpr long long dispatch_groups(long long ctas) {
  return (ctas + kDispatchGroup - 1) / kDispatchGroup;
}
// First word of the rows, for a workspace laid out for `max_ctas` CTAs.
__host__ __device__ constexpr long long dispatch_rows_word(long long max_ctas) {
  return kDispatchHeaderWords + 2 * dispatch_groups(max_ctas) * kPairE;
}
__host__ __device__ constexpr long long dispatch_ws_words(long long max_ctas) {
  return dispatch_rows_word(max_ctas) + max_ctas * (kPairE / 2);
}

struct Dispatch {
  int32_t* sorted;      // sorted_token_ids
  long long sorted_cap;
  int32_t* expert_ids;
  long long eid_cap;
  int32_t* post_pad;    // num_tokens_post_pad (one int32)
  uint32_t* ws;
  int bs;               // block_size
  int max_ctas;         // CTAs the workspace is laid out for (>= the grid)
};

// Thread `first + k` loads word k * 16384 of [p, p + n) (one per 64 KB), so
// that the buffer's address translations are cached before it is written:
// the logits streamed while routing evict them.
__device__ __forceinline__ void l4_touch(const int32_t* p, long long n, int tid, int first) {
  const long long k = tid - first;
  if (k >= 0 && k < 64 && k * 16384 < n)
    asm volatile("{\n .reg .u32 t;\n ld.global.cg.u32 t, [%0];\n}" ::"l"(p + k * 16384) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Counts of the warp's slice of ids [sb, se) per expert into wh[0 .. 255]
// (the first 1 KB of the warp's own slot, free once its last tile is done),
// right after the warp's last tile.  The atomics go one token (8 lanes) at
// a time, so for a slice of at most 128 entries rk[] holds each entry's
// count of earlier entries of its expert in the slice (a token's experts
// are distinct); ev[] keeps the ids (-1 past the slice's end).
__device__ __forceinline__ void l4_slice_counts(int* wh, const int32_t* ids, long long sb, long long se, int lane,
                                                int (&ev)[4], int (&rk)[4]) {
#pragma unroll
  for (int i = 0; i < kPairE / 32; ++i) wh[i * 32 + lane] = 0;
  __syncwarp();  // also orders the warp's own id stores before the loads
  bool badid = false;
  for (long long b = sb; b < se; b += 128) {
    int v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long i = b + u * 32 + lane;
      v[u] = i < se ? __ldcg(ids + i) : -1;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const bool ok = static_cast<unsigned>(v[u]) < static_cast<unsigned>(kPairE);
      if (!ok && b + u * 32 + lane < se) badid = true;
      int r = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // token j of the batch: lanes 8j .. 8j + 7
        if ((lane >> 3) == j && ok) r = atomicAdd(&wh[v[u]], 1);
        __syncwarp();
      }
      ev[u] = v[u];
      rk[u] = r;
    }
  }
  if (badid) atomicOr(&g_router_error, 4);
}

// Staging buffer of the CTA's entries, sorted by expert, in the slots after
// the four scratch slots: the upper 7 KB of each (the first 1 KB holds the
// slot's warp's slice counts).
constexpr int kL4StagePerSlot = (kL4Tile - 1024) / 4;  // 1792 entries

__device__ __forceinline__ int* l4_stage_ptr(uint8_t* base, int j) {
  const int s = j / kL4StagePerSlot;
  return reinterpret_cast<int*>(base + (4 + s) * kL4Tile + 1024) + (j - s * kL4StagePerSlot);
}

// One warp's slice placed in index order, one token (8 entries, 8 lanes) a
// step: entry i of expert e goes to out(e, wh[e], i) and wh[e] advances
// (shared-memory atomic; a token's 8 experts are distinct, and where they
// are not the atomic still gives every entry its own place).  A batch of
// 32 entries holds 4 whole tokens (slices start on a tile).  `kept`: the
// slice's ids are ev[]; else they are re-read from L2.
template <typename Out>
__device__ __forceinline__ void l4_place_tokens(int* wh, const int32_t* ids, long long sb, long long se,
                                                bool kept, const int (&ev)[4], int lane, Out out) {
  const int tok = lane >> 3;
  for (long long b0 = sb; b0 < se; b0 += 128) {
    int v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long i = b0 + u * 32 + lane;
      v[u] = kept ? ev[u] : (i < se ? __ldcg(ids + i) : -1);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long b = b0 + u * 32;
      if (b >= se) break;
      const int e = v[u];
      const bool ok = b + lane < se && static_cast<unsigned>(e) < static_cast<unsigned>(kPairE);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (tok == j && ok) out(e, atomicAdd(&wh[e], 1), static_cast<int32_t>(b + lane));
        __syncwarp();
      }
    }
  }
}

// The CTA's part of the dispatch, after every warp's slice counts: publish
// the CTA's expert counts, sort the CTA's entries by expert in shared
// memory (each as index << 8 | expert) while the other CTAs arrive, wait for
// all CTAs (bounded), then copy the sorted entries to their places.  When
// the entries do not fit the staging buffer, or an index needs more than 24
// bits, each warp places its slice straight into the output instead.
// `bad` when one of the CTA's waits ran out: it then only takes part in
// the barrier.
template <int NW>
__device__ __forceinline__ void l4_dispatch(uint8_t* base, int* sflag, const Dispatch& d, const int32_t* ids,
                                            long long T, long long sb, long long se, const int (&ev)[4],
                                            const int (&rk)[4], const uint32_t* gen_smem, bool bad) {
  constexpr int E = kPairE;
  constexpr int NT = NW * 32;
  constexpr int Q = NT / 128;   // groups of 128 threads, each over two experts per thread
  constexpr int WPQ = NW / Q;   // warps per group
  constexpr int kStageCap = (NW - 4) * kL4StagePerSlot;
  static_assert(NT % 128 == 0 && NW % Q == 0 && NT >= E && NW > 4, "dispatch thread layout");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p2 = tid & 127, q = tid >> 7;  // experts 2 p2, 2 p2 + 1 of group q
  // scratch in the first four slots, after their first 1 KB (slice counts)
  int* psum = reinterpret_cast<int*>(base + 0 * kL4Tile + 1024);  // [Q][E]
  int* ptot = reinterpret_cast<int*>(base + 1 * kL4Tile + 1024);  // [Q][E]
  int* pbef = reinterpret_cast<int*>(base + 2 * kL4Tile + 1024);  // [Q][E]
  int* sstart = reinterpret_cast<int*>(base + 3 * kL4Tile + 1024);  // [E + 1] run starts
  int* stot = sstart + E + 1;   // [E] expert totals
  int* sfirst = stot + E;       // [E] this CTA's first slot per expert
  int* slstart = sfirst + E;    // [E] its first position in the staging buffer
  int* wsum = slstart + E;      // [E / 32] scan partials
  int* wsuml = wsum + E / 32;   // [E / 32] scan partials of the staging positions
  int* sblk = wsuml + E / 32;   // [E + 1] first block of each run, blocks of all runs
  uint32_t* ws = d.ws;
  const long long ngmax = dispatch_groups(d.max_ctas);
  uint32_t* rows = ws + dispatch_rows_word(d.max_ctas);
  const int c = blockIdx.x, gi = c / kDispatchGroup;
  const int ng = static_cast<int>(dispatch_groups(gridDim.x));

  __syncthreads();  // every warp's slice counts are in
  const uint32_t gen = *gen_smem;
  const int par = static_cast<int>(gen & 1u);
  uint32_t* gs_cur = ws + kDispatchHeaderWords + par * ngmax * E;
  uint32_t* gs_next = ws + kDispatchHeaderWords + (1 - par) * ngmax * E;

  // 1. the CTA's counts: partial sums over groups of WPQ warps
  if (!bad) {
    int2 acc = make_int2(0, 0);
#pragma unroll
    for (int j = 0; j < WPQ; ++j) {
      const int2 v = *reinterpret_cast<const int2*>(base + (q * WPQ + j) * kL4Tile + 8 * p2);
      acc.x += v.x;
      acc.y += v.y;
    }
    *reinterpret_cast<int2*>(psum + q * E + 2 * p2) = acc;
  }
  __syncthreads();
  int h = 0;
  if (!bad && tid < E) {
#pragma unroll
    for (int j = 0; j < Q; ++j) h += psum[j * E + tid];
  }
  // (the expert threads, warps 0 .. E/32 - 1, only: the other warps would
  // share their issue slots) staging positions: exclusive scan of h over
  // the experts; the CTA's row and group sum
  if (tid < E) {
    int hincl = h;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, hincl, o);
      if (lane >= o) hincl += v;
    }
    if (lane == 31) wsuml[warp] = hincl;
    slstart[tid] = hincl - h;  // within its group of 32 experts until the offsets below
    const uint32_t hn = __shfl_down_sync(0xFFFFFFFFu, static_cast<uint32_t>(h), 1);
    if ((tid & 1) == 0)
      rows[static_cast<long long>(c) * (E / 2) + (tid >> 1)] = static_cast<uint32_t>(h) | (hn << 16);
    if (h != 0) atomicAdd(gs_cur + static_cast<long long>(gi) * E + tid, static_cast<uint32_t>(h));
  }
  // 2. arrive (release: the CTA's row and group sum); while the other CTAs
  // arrive, the per-warp offsets within the CTA and the CTA's entries sorted
  // by expert into the staging buffer; then wait
  __syncthreads();
  if (tid == 0) red_release_gpu_add(ws + 1 + par, 1u);
  // the next launch's group sums and arrival count start at zero
  for (long long g = c; g < ngmax; g += gridDim.x)
    if (tid < E) gs_next[g * E + tid] = 0u;
  if (c == 0 && tid == 0) ws[1 + (1 - par)] = 0u;
  l4_touch(d.sorted, d.sorted_cap, tid, 0);
  l4_touch(d.expert_ids, d.eid_cap, tid, 64);
  int ncta = 0;  // the CTA's entries
#pragma unroll
  for (int w = 0; w < E / 32; ++w) ncta += wsuml[w];
  const bool staged = ncta <= kStageCap && T * kPairKMax <= (1LL << 24);
  if (!bad) {
    // per-warp offsets of experts 2 p2, 2 p2 + 1 within the CTA; staged,
    // plus the experts' first staging positions
    int2 run = make_int2(0, 0);
    for (int j = 0; j < q; ++j) {
      run.x += psum[j * E + 2 * p2];
      run.y += psum[j * E + 2 * p2 + 1];
    }
    if (staged) {
      int off = 0;
      for (int w = 0; w < (2 * p2) / 32; ++w) off += wsuml[w];
      run.x += off + slstart[2 * p2];  // (slstart is 4-byte aligned only)
      run.y += off + slstart[2 * p2 + 1];
    }
#pragma unroll
    for (int j = 0; j < WPQ; ++j) {
      int2* w = reinterpret_cast<int2*>(base + (q * WPQ + j) * kL4Tile + 8 * p2);
      const int2 v = *w;
      *w = run;
      run.x += v.x;
      run.y += v.y;
    }
  }
  __syncthreads();
  if (!bad && tid < E) {  // each expert's first staging position, for the copy-out
    int off = 0;
    for (int w = 0; w < warp; ++w) off += wsuml[w];
    slstart[tid] += off;
  }
  int* wh = reinterpret_cast<int*>(base + warp * kL4Tile);
  const bool kept = se - sb <= 128;
  if (!bad && staged) {  // wh[e]: this warp's first staging position of expert e
    if (kept) {  // positions from the counting pass's ranks, all at once
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long i = sb + u * 32 + lane;
        const int e = ev[u];
        if (i < se && static_cast<unsigned>(e) < static_cast<unsigned>(E))
          *l4_stage_ptr(base, wh[e] + rk[u]) =
              static_cast<int>((static_cast<uint32_t>(i) << 8) | static_cast<uint32_t>(e));
      }
    } else {
      l4_place_tokens(wh, ids, sb, se, kept, ev, lane, [&](int e, int pos, int32_t i) {
        *l4_stage_ptr(base, pos) = static_cast<int>((static_cast<uint32_t>(i) << 8) | e);
      });
    }
  }
  if (tid == 0) {
    bool ok = false;
    const unsigned long long t0 = peer::globaltimer();
    for (uint32_t i = 0; i < peer::kWaitPolls; ++i) {
      if (ld_acquire_gpu(ws + 1 + par) == gridDim.x) {
        ok = true;
        break;
      }
      if ((i & 31u) == 31u && peer::globaltimer() - t0 > peer::kWaitNs) break;
    }
    *sflag = ok ? 1 : 0;
  }
  __syncthreads();
  if (*sflag == 0) {
    if (tid == 0) atomicOr(&g_router_error, 2);
    return;
  }
  if (c == 0 && tid == 0) ws[0] = gen + 1u;  // every CTA read the generation before it arrived
  if (bad) return;

  // 3. expert totals (all group sums) and the entries of earlier CTAs (the
  // group sums of earlier groups, the rows of earlier CTAs of this group)
  {
    uint32_t tl = 0, th = 0, bl = 0, bh = 0;
#pragma unroll 2
    for (int g = q; g < ng; g += Q) {
      const uint2 v = __ldcg(reinterpret_cast<const uint2*>(gs_cur + static_cast<long long>(g) * E) + p2);
      tl += v.x;
      th += v.y;
      if (g < gi) {
        bl += v.x;
        bh += v.y;
      }
    }
    const int r0 = gi * kDispatchGroup;
#pragma unroll 3
    for (int r = r0 + q; r < c; r += Q) {
      const uint32_t v = __ldcg(rows + static_cast<long long>(r) * (E / 2) + p2);
      bl += v & 0xFFFFu;
      bh += v >> 16;
    }
    *reinterpret_cast<int2*>(ptot + q * E + 2 * p2) = make_int2(static_cast<int>(tl), static_cast<int>(th));
    *reinterpret_cast<int2*>(pbef + q * E + 2 * p2) = make_int2(static_cast<int>(bl), static_cast<int>(bh));
  }
  __syncthreads();
  int tot = 0, bef = 0;
  if (tid < E) {
#pragma unroll
    for (int j = 0; j < Q; ++j) {
      tot += ptot[j * E + tid];
      bef += pbef[j * E + tid];
    }
  }
  int nblk = 0, incl = 0;
  if (tid < E) {  // inclusive scan over the experts (warps 0 .. E/32 - 1), in blocks
    nblk = (tot + d.bs - 1) / d.bs;  // blocks of the expert's run
    incl = nblk;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
  }
  __syncthreads();
  if (tid < E) {
    int off = 0;
    for (int w = 0; w < warp; ++w) off += wsum[w];
    const int b0 = off + incl - nblk;
    const int start = b0 * d.bs;
    sblk[tid] = b0;
    sstart[tid] = start;
    stot[tid] = tot;
    sfirst[tid] = start + bef;
    if (tid == E - 1) {
      sblk[E] = off + incl;
      sstart[E] = (off + incl) * d.bs;
    }
  }
  __syncthreads();
  const int end = sstart[E];
  if (c == 0 && tid == 0) *d.post_pad = end;

  // 4. shared by the grid: run padding (expert e by CTA e % grid), the slots
  // after the last run and the expert of every block
  // (one warp per expert: with 148 CTAs only warps 0 and 1 have an expert,
  // and the others go straight on instead of sharing the issue slots)
  const int32_t numel = static_cast<int32_t>(T * kPairKMax);
  for (int e = c + warp * static_cast<int>(gridDim.x); e < E; e += NW * static_cast<int>(gridDim.x)) {
    const int from = sstart[e] + stot[e], to = sstart[e + 1];
    for (int j = from + lane; j < to; j += 32) d.sorted[j] = numel;
    const int b1 = sblk[e + 1];
    for (int b = sblk[e] + lane; b < b1; b += 32) d.expert_ids[b] = e;
  }
  const long long gtid = static_cast<long long>(c) * NT + tid;
  const long long gthreads = static_cast<long long>(gridDim.x) * NT;
  for (long long j = end + gtid; j < d.sorted_cap; j += gthreads) d.sorted[j] = numel;
  for (long long b = sblk[E] + gtid; b < d.eid_cap; b += gthreads) d.expert_ids[b] = -1;

  // 5. the CTA's entries to their places: staged entry j of expert e goes
  // to sfirst[e] + (j - slstart[e]), so each expert's entries land in one
  // contiguous run; or each warp's slice straight from its ids
  if (staged) {
    for (int j = tid; j < ncta; j += NT) {
      const uint32_t v = static_cast<uint32_t>(*l4_stage_ptr(base, j));
      const int e = static_cast<int>(v & 255u);
      d.sorted[sfirst[e] + (j - slstart[e])] = static_cast<int32_t>(v >> 8);
    }
  } else {
    l4_place_tokens(wh, ids, sb, se, kept, ev, lane,
                    [&](int e, int pos, int32_t i) { d.sorted[sfirst[e] + pos] = i; });
  }
}

template <int NW, bool kDispatch>
__global__ void __launch_bounds__(NW * 32, 1) grouped_topk_lanes4_kernel(
    const __grid_constant__ CUtensorMap tm, const Params p, const long long wtiles, const int vec_out,
    const Dispatch d) {
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
  // tiles tfirst, tfirst + tstep, ... below tend: round-robin over every
  // warp of the grid -- with at most one tile per warp, consecutive tiles on
  // different CTAs (a small batch spreads over as many SMs as it has tiles),
  // else consecutive tiles on one CTA's warps -- or (dispatch) a contiguous
  // run of the CTA's contiguous range [c0, c1)
  long long tfirst, tstep, tend;
  if constexpr (kDispatch) {
    const long long c0 = static_cast<long long>(blockIdx.x) * wtiles / gridDim.x;
    const long long c1 = static_cast<long long>(blockIdx.x + 1) * wtiles / gridDim.x;
    const long long tpw = (c1 - c0 + NW - 1) / NW;
    tfirst = c0 + warp * tpw;
    tstep = 1;
    tend = tfirst + tpw < c1 ? tfirst + tpw : c1;
  } else {
    tstep = static_cast<long long>(gridDim.x) * NW;
    tfirst = wtiles <= tstep ? static_cast<long long>(warp) * gridDim.x + blockIdx.x
                             : static_cast<long long>(blockIdx.x) * NW + warp;
    tend = wtiles;
  }
  const float* gating = static_cast<const float*>(p.gating);

  // the logits are read once: first out of L2, so that they do not evict
  // the outputs, the workspace and this kernel's instructions
  const uint64_t stream_policy = sm100::l2_evict_first_policy();
  auto issue = [&](long long wt) {
    if (lane == 0) sm100::mbar_arrive_expect_tx(full, kL4Tile);
    __syncwarp();
    if (lane < kPairG)
      sm100::tma_load_2d_hint(tb + lane * kL4Box, &tm, full, lane * kPairGS, static_cast<int>(wt * kL4Tokens),
                              stream_policy);
  };

  if (lane == 0) {
    sm100::mbar_init(full, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  if constexpr (kDispatch) {
    // the dispatch's generation, fixed until every CTA of this launch has
    // arrived at its barrier: kept in the spare word of warp 1's barrier slot
    if (threadIdx.x == 0)
      *reinterpret_cast<uint32_t*>(base + L.bar_off + 16 + 12) = *reinterpret_cast<volatile uint32_t*>(d.ws);
  }
  __syncwarp();
  if (tfirst < tend) issue(tfirst);
  for (int i = threadIdx.x; i < kPairE; i += blockDim.x) sbias[i] = p.bias[i];
  __syncthreads();  // the only CTA-wide barrier of the routing loop: bias staged

  long long it = 0;
  bool inflight = tfirst < tend;
  for (;; ++it) {
    const long long wt = tfirst + it * tstep;
    if (wt >= tend) break;
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
      const long long nt = wt + tstep;
      if (nt < tend) issue(nt);
      inflight = nt < tend;
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
  if constexpr (kDispatch) {
    // the warp's slice of ids: its tokens [tfirst * 8, min(tend * 8, T))
    const long long sb = tfirst * (kL4Tokens * kPairKMax);
    long long se = tend * (kL4Tokens * kPairKMax);
    if (se > p.T * kPairKMax) se = p.T * kPairKMax;
    if (se < sb) se = sb;
    const bool wbad = __shfl_sync(0xFFFFFFFFu, lane == 0 ? *abort_flag : 0, 0) != 0;
    if (lane == 0) l4_touch(reinterpret_cast<const int32_t*>(d.ws), dispatch_ws_words(d.max_ctas), 0, 0);
    int ev[4] = {-1, -1, -1, -1}, rk[4] = {0, 0, 0, 0};
    if (!wbad) l4_slice_counts(reinterpret_cast<int*>(tb), p.id_out, sb, se, lane, ev, rk);
    const bool bad = __syncthreads_or(wbad) != 0;
    int* sync_flag = reinterpret_cast<int*>(base + L.bar_off + 12);  // spare word of warp 0's barrier slot
    l4_dispatch<NW>(base, sync_flag, d, p.id_out, p.T, sb, se, ev, rk,
                    reinterpret_cast<const uint32_t*>(base + L.bar_off + 16 + 12), bad);
  }
}

}  // namespace router
}  // namespace mcpu
