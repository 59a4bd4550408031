// vLLM sampler kernels the reference registers on the mcpu device
// (csrc/aten/vllm_kernels/min_p.cpp, logprob.cpp), which run after the model
// on the decode path:
//   vllm_min_p_kernel             logits below max + log(min_p) -> -inf, in
//                                 place, per token's request (min_p.cpp:13-58)
//   vllm_topk_log_softmax_kernel  logits[ids] - logsumexp(row)
//                                 (logprob.cpp:15-69)
//   vllm_ranks_kernel             number of logits >= the sampled token's
//                                 (logprob.cpp:123-149)
//   vllm_penalties_kernel         repetition / frequency / presence penalties
//                                 in place (penalties.cpp:14-84)
//   vllm_bincount_kernel          prompt bit mask and output token counts
//                                 (penalties.cpp:187-246)
//   vllm_bias_kernel              allowed-token mask, logit bias, min-length
//                                 stop tokens (logit_bias.cpp:15-96)
//   vllm_bad_words_kernel         -inf on the last id of each bad word whose
//                                 prefix ends the sequence (bad_words.cpp:13-82)
// In the first three, each row is split over a cluster of 8 CTAs (256
// threads each): every CTA
// streams its eighth of the row (16-byte loads, four in flight per thread,
// where the row start allows), the CTAs combine their partial maxima, sums
// or counts through distributed shared memory in rank order, and each then
// runs the op's pass over its eighth again (from L2).  Logits are fp32,
// fp16 or bf16, compared as fp32 like the reference; the log-sum-exp sums
// exp(x - max) in fp64 as the reference does, each term from the fp32 exp.
#include <cooperative_groups.h>
#include <math.h>

#include "common.cuh"

namespace mcpu {
namespace sampler {

namespace cg = cooperative_groups;

constexpr int kThreads = 256;  // per CTA
constexpr int kCluster = 8;    // CTAs per row

__device__ int g_sampler_error = 0;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T neg_inf();
template <>
__device__ __forceinline__ float neg_inf<float>() { return -INFINITY; }
template <>
__device__ __forceinline__ __half neg_inf<__half>() { return __ushort_as_half(0xFC00); }
template <>
__device__ __forceinline__ __nv_bfloat16 neg_inf<__nv_bfloat16>() { return __ushort_as_bfloat16(0xFF80); }

// Calls f(i, value) for every element of this CTA's part of the row: with a
// 16-byte-aligned row start, the row's 16-byte vectors are split evenly over
// the cluster (the last CTA also takes the scalar tail); otherwise the
// elements are.
template <typename T, typename F>
__device__ __forceinline__ void for_part(const T* row, long long n, int part, F&& f) {
  constexpr int V = 16 / sizeof(T);
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const long long nv = n / V;
    const long long v0 = nv * part / kCluster, v1 = nv * (part + 1) / kCluster;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    long long j = v0 + threadIdx.x;
    for (; j + 3 * kThreads < v1; j += 4 * kThreads) {  // four 16-byte loads in flight per thread
      uint4 u[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) u[r] = __ldg(rv + j + r * kThreads);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const T* t = reinterpret_cast<const T*>(&u[r]);
#pragma unroll
        for (int k = 0; k < V; ++k) f((j + r * kThreads) * V + k, to_f(t[k]));
      }
    }
    for (; j < v1; j += kThreads) {
      const uint4 u = __ldg(rv + j);
      const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < V; ++k) f(j * V + k, to_f(t[k]));
    }
    if (part == kCluster - 1)
      for (long long i = nv * V + threadIdx.x; i < n; i += kThreads) f(i, to_f(row[i]));
  } else {
    const long long e0 = n * part / kCluster, e1 = n * (part + 1) / kCluster;
    for (long long i = e0 + threadIdx.x; i < e1; i += kThreads) f(i, to_f(row[i]));
  }
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < kThreads / 32 ? red[l] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

template <typename A>
__device__ __forceinline__ A block_sum(A v, A* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < kThreads / 32 ? red[l] : A(0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Combines one value per CTA of the cluster, in rank order, on every CTA.
// `slot` is this CTA's shared variable holding its value.
template <typename A, typename Op>
__device__ __forceinline__ A cluster_combine(A* slot, A init, Op op) {
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every CTA's slot is written
  A v = init;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) v = op(v, *cluster.map_shared_rank(slot, r));
  cluster.sync();  // every CTA has read every slot before any reuses or leaves
  return v;
}

// The row maximum as the reference takes it: a running `v > max` from -inf,
// so NaN never becomes the maximum.
template <typename T>
__device__ __forceinline__ float row_max(const T* row, long long n, int part, float* red, float* slot) {
  float m = -INFINITY;
  for_part(row, n, part, [&](long long, float v) { m = v > m ? v : m; });
  m = block_max(m, red);
  if (threadIdx.x == 0) *slot = m;
  return cluster_combine(slot, -INFINITY, [](float a, float b) { return fmaxf(a, b); });
}

template <typename T>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    min_p_kernel(T* logits, long long stride, const int32_t* idx, const float* min_p, long long vocab) {
  __shared__ float red[kThreads / 32];
  __shared__ float slot;
  const long long r = blockIdx.x / kCluster;
  const int part = blockIdx.x % kCluster;
  T* row = logits + r * stride;
  const float mp = min_p[idx[r]];
  if (mp == 0.0f) return;  // the same for every CTA of the cluster
  // log(p) rounded once from fp64: the fp32 logarithm to within rounding
  const float thr = row_max(row, vocab, part, red, &slot) + static_cast<float>(log(static_cast<double>(mp)));
  // the compare pass, one 16-byte store per vector that changes
  constexpr int V = 16 / sizeof(T);
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const long long nv = vocab / V;
    const long long v0 = nv * part / kCluster, v1 = nv * (part + 1) / kCluster;
    uint4* rv = reinterpret_cast<uint4*>(row);
    for (long long j = v0 + threadIdx.x; j < v1; j += kThreads) {
      uint4 u = __ldg(rv + j);
      T* t = reinterpret_cast<T*>(&u);
      bool any = false;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        if (to_f(t[k]) < thr) {
          t[k] = neg_inf<T>();
          any = true;
        }
      }
      if (any) rv[j] = u;
    }
    if (part == kCluster - 1)
      for (long long i = nv * V + threadIdx.x; i < vocab; i += kThreads)
        if (to_f(row[i]) < thr) row[i] = neg_inf<T>();
  } else {
    for_part(static_cast<const T*>(row), vocab, part, [&](long long i, float v) {
      if (v < thr) row[i] = neg_inf<T>();
    });
  }
}

template <typename T>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    topk_log_softmax_kernel(float* out, const T* logits, long long stride, const int64_t* ids, long long ids_stride,
                            int topk, long long vocab) {
  __shared__ float red[kThreads / 32];
  __shared__ double redd[kThreads / 32];
  __shared__ float slot;
  __shared__ double dslot;
  const long long r = blockIdx.x / kCluster;
  const int part = blockIdx.x % kCluster;
  const T* row = logits + r * stride;
  const float m = row_max(row, vocab, part, red, &slot);
  double s = 0.0;
  // exp in fp32 (within about one ulp of the fp64 exp the reference takes),
  // summed in fp64 like the reference
  for_part(row, vocab, part, [&](long long, float v) { s += static_cast<double>(expf(v - m)); });
  s = block_sum(s, redd);
  if (threadIdx.x == 0) dslot = s;
  s = cluster_combine(&dslot, 0.0, [](double a, double b) { return a + b; });
  if (part != 0) return;
  const float lse = m + static_cast<float>(log(s));
  for (int k = threadIdx.x; k < topk; k += kThreads) {
    long long id = ids[r * ids_stride + k];
    if (id < 0) id = 0;
    if (id >= vocab) id = vocab - 1;
    out[r * static_cast<long long>(topk) + k] = to_f(row[id]) - lse;
  }
}

template <typename T>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    ranks_kernel(int64_t* out, const T* logits, long long stride, const int64_t* ids, long long vocab) {
  __shared__ long long redl[kThreads / 32];
  __shared__ long long slot;
  const long long r = blockIdx.x / kCluster;
  const int part = blockIdx.x % kCluster;
  const T* row = logits + r * stride;
  const long long id = ids[r];
  if (id < 0 || id >= vocab) {  // the same for every CTA of the cluster
    if (part == 0 && threadIdx.x == 0) {
      out[r] = 0;
      atomicOr(&g_sampler_error, 1);
    }
    return;
  }
  const float x = to_f(row[id]);
  long long c = 0;
  for_part(row, vocab, part, [&](long long, float v) { c += v >= x ? 1 : 0; });
  c = block_sum(c, redl);
  if (threadIdx.x == 0) slot = c;
  c = cluster_combine(&slot, 0LL, [](long long a, long long b) { return a + b; });
  if (part == 0 && threadIdx.x == 0) out[r] = c;
}

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Repetition / frequency / presence penalties in place
// (csrc/aten/vllm_kernels/penalties.cpp:14-84).  One CTA per (row, 2048
// logits); every thread holds 8 logits and their output counts, adds the
// row's draft tokens (token_ids[tok - pos + 1 .. tok], staged in shared
// memory 256 at a time) to the counts, and writes each logit back once.  The
// arithmetic is the reference's, one rounding per operation (no contraction):
// l / rep or l * rep where the token is in the prompt or the output, then
// l - freq * count, then l - pres * [count > 0].
constexpr int kPenElems = 8;
constexpr int kPenChunk = kThreads * kPenElems;

template <typename T>
struct PenVec;  // four logits in one load
template <>
struct PenVec<float> { using type = float4; };
template <>
struct PenVec<__half> { using type = uint2; };
template <>
struct PenVec<__nv_bfloat16> { using type = uint2; };

template <typename T>
__global__ void __launch_bounds__(kThreads)
    penalties_kernel(T* logits, long long stride, long long vocab, const int32_t* idx, const int32_t* tids,
                     const int32_t* lpos, const float* rep, const float* freq, const float* pres,
                     long long num_reqs, const int32_t* pbm, long long pbm_stride, const int32_t* obc,
                     long long obc_stride, long long max_spec_len) {
  __shared__ int32_t drafts[kThreads];
  const long long tok = blockIdx.x;
  const int32_t req = idx[tok];
  if (req < 0 || req >= num_reqs) {  // the same for every CTA of the row
    if (blockIdx.y == 0 && threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    return;
  }
  const float rp = rep[req], fp = freq[req], pp = pres[req];
  if (rp == 1.0f && fp == 0.0f && pp == 0.0f) return;
  const int32_t pos = lpos[tok];
  const bool use_drafts = pos > 0 && max_spec_len > 0;
  const long long d0 = tok - pos + 1;  // first draft; the last is token tok
  if (use_drafts && d0 < 0) {
    if (blockIdx.y == 0 && threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    return;
  }
  T* row = logits + tok * stride;
  const int32_t* orow = obc + req * obc_stride;
  const int32_t* prow = pbm + req * pbm_stride;
  const long long base = static_cast<long long>(blockIdx.y) * kPenChunk;
  // With 16-byte-aligned logits and count rows, thread i takes the 4-element
  // vectors i and i + 256 of the chunk (one 16-byte count load and one 16- or
  // 8-byte logit load each); otherwise the elements i + 256 s, s < 8.
  const bool vec = ((reinterpret_cast<uintptr_t>(row) | reinterpret_cast<uintptr_t>(orow)) & 15) == 0;
  long long e[kPenElems];
#pragma unroll
  for (int s = 0; s < kPenElems; ++s)
    e[s] = vec ? base + (static_cast<long long>((s / 4) * kThreads + threadIdx.x) << 2) + (s % 4)
               : base + threadIdx.x + s * kThreads;
  using Vec = typename PenVec<T>::type;
  int cnt[kPenElems];
  float x[kPenElems];
#pragma unroll
  for (int j = 0; j < kPenElems / 4; ++j) {
    const long long e0 = e[j * 4];
    if (vec && e0 + 3 < vocab) {
      const int4 c = *reinterpret_cast<const int4*>(orow + e0);
      const Vec u = *reinterpret_cast<const Vec*>(row + e0);
      const T* t = reinterpret_cast<const T*>(&u);
      cnt[j * 4] = c.x, cnt[j * 4 + 1] = c.y, cnt[j * 4 + 2] = c.z, cnt[j * 4 + 3] = c.w;
#pragma unroll
      for (int k = 0; k < 4; ++k) x[j * 4 + k] = to_f(t[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const long long v = e[j * 4 + k];
        cnt[j * 4 + k] = v < vocab ? orow[v] : 0;
        x[j * 4 + k] = v < vocab ? to_f(row[v]) : 0.0f;
      }
    }
  }
  if (use_drafts) {
    for (int b0 = 0; b0 < pos; b0 += kThreads) {
      const int nd = min(kThreads, pos - b0);
      __syncthreads();
      if (static_cast<int>(threadIdx.x) < nd) drafts[threadIdx.x] = tids[d0 + b0 + threadIdx.x];
      __syncthreads();
      for (int d = 0; d < nd; ++d) {
        const long long t = drafts[d];
#pragma unroll
        for (int s = 0; s < kPenElems; ++s) cnt[s] += t == e[s] ? 1 : 0;
      }
    }
  }
  alignas(16) T y[kPenElems];  // stored as whole vectors below
#pragma unroll
  for (int s = 0; s < kPenElems; ++s) {
    const long long v = e[s];
    float l = x[s];
    const bool in_out = cnt[s] > 0;
    if (rp != 1.0f && v < vocab) {
      const bool in_prompt = (static_cast<uint32_t>(prow[v >> 5]) >> (v & 31)) & 1u;
      if (in_prompt || in_out) l = l > 0.0f ? __fdiv_rn(l, rp) : __fmul_rn(l, rp);
    }
    l = __fsub_rn(l, __fmul_rn(fp, __int2float_rn(cnt[s])));
    l = __fsub_rn(l, __fmul_rn(pp, in_out ? 1.0f : 0.0f));
    y[s] = from_f<T>(l);
  }
#pragma unroll
  for (int j = 0; j < kPenElems / 4; ++j) {
    const long long e0 = e[j * 4];
    if (vec && e0 + 3 < vocab) {
      *reinterpret_cast<Vec*>(row + e0) = *reinterpret_cast<const Vec*>(&y[j * 4]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (e[j * 4 + k] < vocab) row[e[j * 4 + k]] = y[j * 4 + k];
    }
  }
}

// Prompt bit mask and output counts of each listed request
// (penalties.cpp:187-246): one CTA per entry of expanded_idx_mapping; the
// prompt tokens set bits with atomicOr, the tokens generated since prefill
// (positions prompt_len .. prefill_len) add to the counts with atomicAdd,
// so the integer results do not depend on the order.  Tokens outside the
// vocabulary are skipped, as in the reference; a request index or length
// outside its tensor sets the error flag.
__global__ void __launch_bounds__(kThreads)
    bincount_kernel(const int32_t* idx, const int32_t* tids, long long tids_stride, long long max_seq,
                    const int32_t* plen, const int32_t* flen, long long num_reqs, int32_t* pbm,
                    long long packed_cols, long long pbm_stride, int32_t* obc, long long vocab,
                    long long obc_stride) {
  const int32_t req = idx[blockIdx.x];
  if (req < 0 || req >= num_reqs) {
    if (threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    return;
  }
  long long p = plen[req], f = flen[req];
  if (p < 0 || f > max_seq) {
    if (threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    p = max(p, 0LL);
    f = min(f, max_seq);
  }
  const int32_t* trow = tids + req * tids_stride;
  int32_t* prow = pbm + req * pbm_stride;
  int32_t* orow = obc + req * obc_stride;
  for (long long i = threadIdx.x; i < min(p, max_seq); i += kThreads) {
    const int32_t t = trow[i];
    if (t >= 0 && t / 32 < packed_cols) atomicOr(&prow[t / 32], static_cast<int32_t>(1u << (t % 32)));
  }
  for (long long i = p + threadIdx.x; i < f; i += kThreads) {
    const int32_t t = trow[i];
    if (t >= 0 && t < vocab) atomicAdd(&orow[t], 1);
  }
}

// Allowed-token masks, logit bias and min-length stop tokens
// (logit_bias.cpp:15-96), one CTA per token row, in the reference's order
// with a block barrier between the steps: (1) the first min(n, 512) allowed
// ids (clamped into the vocabulary) keep their values, staged in shared
// memory, and the rest of the row becomes -inf; (2) one thread adds the
// biases in list order, rounding to the logits dtype after each add, so
// repeated ids give the reference's sums; (3) while pos < min_len the stop
// ids become -inf.  A count above its list's width is clamped and sets the
// error flag (the reference reads past the row).
constexpr int kMaxAllowed = 512;

template <typename T>
__global__ void __launch_bounds__(kThreads)
    bias_kernel(T* logits, long long stride, long long vocab, const int32_t* idx, long long num_reqs,
                const int32_t* n_allowed, const int32_t* allowed, long long allowed_stride, long long allowed_cols,
                const int32_t* n_bias, const int32_t* bias_ids, long long bias_ids_stride, const float* bias,
                long long bias_stride, long long bias_cols, const int64_t* pos, const int32_t* min_lens,
                const int32_t* n_stop, const int32_t* stop, long long stop_stride, long long stop_cols) {
  __shared__ __align__(4) unsigned char saved_raw[kMaxAllowed * sizeof(T)];  // the values, bit for bit
  __shared__ int32_t saved_ids[kMaxAllowed];
  T* saved = reinterpret_cast<T*>(saved_raw);
  const long long tok = blockIdx.x;
  const int32_t req = idx[tok];
  if (req < 0 || req >= num_reqs) {
    if (threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    return;
  }
  T* row = logits + tok * stride;
  const int32_t na = n_allowed[req];
  if (na > 0) {
    if (na > allowed_cols && threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    const int ns = static_cast<int>(min(min(static_cast<long long>(na), static_cast<long long>(kMaxAllowed)),
                                        allowed_cols));
    const int32_t* arow = allowed + req * allowed_stride;
    for (int k = threadIdx.x; k < ns; k += kThreads) {
      const int32_t id = min(max(arow[k], 0), static_cast<int32_t>(vocab - 1));
      saved_ids[k] = id;
      saved[k] = row[id];
    }
    __syncthreads();
    for (long long i = threadIdx.x; i < vocab; i += kThreads) row[i] = neg_inf<T>();
    __syncthreads();
    // repeated ids saved the same value, so the order of these stores does not matter
    for (int k = threadIdx.x; k < ns; k += kThreads) row[saved_ids[k]] = saved[k];
  }
  __syncthreads();
  const int32_t nb = n_bias[req];
  if (nb > 0 && threadIdx.x == 0) {
    if (nb > bias_cols) atomicOr(&g_sampler_error, 1);
    const long long n = min(static_cast<long long>(nb), bias_cols);
    const int32_t* brow = bias_ids + req * bias_ids_stride;
    const float* vrow = bias + req * bias_stride;
    for (long long k = 0; k < n; ++k) {
      const int32_t id = brow[k];
      if (id < 0 || id >= vocab) continue;
      row[id] = from_f<T>(__fadd_rn(to_f(row[id]), vrow[k]));
    }
  }
  __syncthreads();
  const int32_t nst = n_stop[req];
  if (nst > 0 && pos[tok] < min_lens[req]) {
    if (nst > stop_cols && threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    const long long n = min(static_cast<long long>(nst), stop_cols);
    const int32_t* srow = stop + req * stop_stride;
    for (long long k = threadIdx.x; k < n; k += kThreads) {
      const int32_t id = srow[k];
      if (id >= 0 && id < vocab) row[id] = neg_inf<T>();
    }
  }
}

// Bad words (bad_words.cpp:13-82): one CTA per token row, one thread per
// bad word of the row's request.  A bad word is ids[off[w] .. off[w+1]);
// when its prefix (all but the last id) equals the last tokens of the row's
// sequence — the request's output tokens all_token_ids[q, prompt_len ..
// total_len) followed by the row's drafts input_ids[t-pos .. t) — its last
// id becomes -inf.  Threads that ban the same id store the same value.
// Indexes that would leave their tensors set the error flag and skip the
// word (or the row), where the reference reads out of bounds.
constexpr int kBadWordThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kBadWordThreads)
    bad_words_kernel(T* logits, long long stride, long long vocab, const int32_t* idx, long long num_reqs,
                     const int32_t* bw_ids, long long bw_ids_stride, long long bw_ids_cols, const int32_t* bw_off,
                     long long bw_off_stride, long long bw_off_cols, const int32_t* n_bw, const int32_t* atids,
                     long long atids_stride, long long max_seq, const int32_t* plen, const int32_t* tlen,
                     const int32_t* input_ids, const int32_t* local_pos) {
  const long long tok = blockIdx.x;
  const int32_t req = idx[tok];
  bool bad = req < 0 || req >= num_reqs;
  const int32_t nw = bad ? 0 : n_bw[req];
  if (!bad && nw <= 0) return;
  const int32_t pos = local_pos[tok];
  const long long first = tok - pos;  // the request's first row in this batch
  const int32_t pl = bad ? 0 : plen[req], tl = bad ? 0 : tlen[req];
  bad = bad || pos < 0 || first < 0 || pl < 0 || tl < pl || tl > max_seq || nw + 1 > bw_off_cols;
  if (bad) {
    if (threadIdx.x == 0) atomicOr(&g_sampler_error, 1);
    return;
  }
  const int32_t out_len = tl - pl;
  const int32_t eff_len = out_len + pos;
  const int32_t* off = bw_off + req * bw_off_stride;
  const int32_t* ids = bw_ids + req * bw_ids_stride;
  const int32_t* out = atids + req * atids_stride + pl;
  T* row = logits + tok * stride;
  for (int w = threadIdx.x; w < nw; w += kBadWordThreads) {
    const int32_t start = off[w], end = off[w + 1];
    const int32_t prefix = end - start - 1;
    if (prefix > eff_len) continue;
    if (end - 1 < 0 || end - 1 >= bw_ids_cols || (prefix > 0 && start < 0)) {
      atomicOr(&g_sampler_error, 1);
      continue;
    }
    bool match = true;
    for (int32_t i = 0; i < prefix && match; ++i) {
      const int32_t p = eff_len - prefix + i;  // position in output tokens + drafts
      const int32_t actual = p >= out_len ? input_ids[first + (p - out_len)] : out[p];
      match = ids[start + i] == actual;
    }
    const int32_t last = ids[end - 1];
    if (match && last >= 0 && last < vocab) row[last] = neg_inf<T>();
  }
}

orError_t check_float(int dtype, const char* op) {
  MCPU_ARG_CHECK(dtype == MCPU_FLOAT32 || dtype == MCPU_FLOAT16 || dtype == MCPU_BFLOAT16,
                 "%s: logits must be float32, float16 or bfloat16 (dtype code %d)", op, dtype);
  return orSuccess;
}

}  // namespace sampler

orError_t sampler_read_error(int* flag, bool reset) {
  MCPU_CUDA_TRY(cudaMemcpyFromSymbol(flag, sampler::g_sampler_error, sizeof(int)), "sampler error flag");
  if (reset) {
    const int zero = 0;
    MCPU_CUDA_TRY(cudaMemcpyToSymbol(sampler::g_sampler_error, &zero, sizeof(int)), "sampler error flag reset");
  }
  return orSuccess;
}

}  // namespace mcpu

using namespace mcpu;

extern "C" orError_t mcpu_vllm_min_p(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                     const int32_t* expanded_idx_mapping, const float* min_p, int64_t vocab_size,
                                     orStream_t stream) {
  orError_t e = sampler::check_float(dtype, "vllm_min_p_kernel");
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(num_tokens >= 0 && num_tokens < (1LL << 31), "vllm_min_p_kernel: bad num_tokens");
  MCPU_ARG_CHECK(vocab_size > 0 && vocab_size <= logits_stride, "vllm_min_p_kernel: vocab_size %lld out of range",
                 static_cast<long long>(vocab_size));
  if (num_tokens == 0) return orSuccess;
  MCPU_ARG_CHECK(logits && expanded_idx_mapping && min_p, "vllm_min_p_kernel: NULL pointer");
  MCPU_ARG_CHECK(num_tokens <= (1LL << 31) / sampler::kCluster - 1, "vllm_min_p_kernel: too many rows");
  const dim3 grid(static_cast<unsigned>(num_tokens * sampler::kCluster));
  cudaStream_t st = as_cuda(stream);
  if (dtype == MCPU_FLOAT32)
    sampler::min_p_kernel<float><<<grid, sampler::kThreads, 0, st>>>(static_cast<float*>(logits), logits_stride,
                                                                       expanded_idx_mapping, min_p, vocab_size);
  else if (dtype == MCPU_FLOAT16)
    sampler::min_p_kernel<__half><<<grid, sampler::kThreads, 0, st>>>(static_cast<__half*>(logits), logits_stride,
                                                                        expanded_idx_mapping, min_p, vocab_size);
  else
    sampler::min_p_kernel<__nv_bfloat16><<<grid, sampler::kThreads, 0, st>>>(
        static_cast<__nv_bfloat16*>(logits), logits_stride, expanded_idx_mapping, min_p, vocab_size);
  return from_cuda(cudaGetLastError(), "vllm_min_p_kernel launch");
}

extern "C" orError_t mcpu_vllm_topk_log_softmax(float* output, const void* logits, int dtype, int64_t batch,
                                                int64_t logits_stride, const int64_t* topk_ids,
                                                int64_t topk_ids_stride, int64_t topk, int64_t vocab_size,
                                                orStream_t stream) {
  orError_t e = sampler::check_float(dtype, "vllm_topk_log_softmax_kernel");
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(batch >= 0 && batch < (1LL << 31) && topk >= 0 && topk < (1LL << 31),
                 "vllm_topk_log_softmax_kernel: bad batch or topk");
  MCPU_ARG_CHECK(vocab_size > 0 && vocab_size <= logits_stride,
                 "vllm_topk_log_softmax_kernel: vocab_size %lld out of range", static_cast<long long>(vocab_size));
  if (batch == 0 || topk == 0) return orSuccess;
  MCPU_ARG_CHECK(output && logits && topk_ids, "vllm_topk_log_softmax_kernel: NULL pointer");
  MCPU_ARG_CHECK(batch <= (1LL << 31) / sampler::kCluster - 1, "vllm_topk_log_softmax_kernel: too many rows");
  const dim3 grid(static_cast<unsigned>(batch * sampler::kCluster));
  cudaStream_t st = as_cuda(stream);
  if (dtype == MCPU_FLOAT32)
    sampler::topk_log_softmax_kernel<float><<<grid, sampler::kThreads, 0, st>>>(
        output, static_cast<const float*>(logits), logits_stride, topk_ids, topk_ids_stride, static_cast<int>(topk),
        vocab_size);
  else if (dtype == MCPU_FLOAT16)
    sampler::topk_log_softmax_kernel<__half><<<grid, sampler::kThreads, 0, st>>>(
        output, static_cast<const __half*>(logits), logits_stride, topk_ids, topk_ids_stride, static_cast<int>(topk),
        vocab_size);
  else
    sampler::topk_log_softmax_kernel<__nv_bfloat16><<<grid, sampler::kThreads, 0, st>>>(
        output, static_cast<const __nv_bfloat16*>(logits), logits_stride, topk_ids, topk_ids_stride,
        static_cast<int>(topk), vocab_size);
  return from_cuda(cudaGetLastError(), "vllm_topk_log_softmax_kernel launch");
}

extern "C" orError_t mcpu_vllm_ranks(int64_t* output, const void* logits, int dtype, int64_t batch,
                                     int64_t logits_stride, const int64_t* token_ids, int64_t vocab_size,
                                     orStream_t stream) {
  orError_t e = sampler::check_float(dtype, "vllm_ranks_kernel");
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(batch >= 0 && batch < (1LL << 31), "vllm_ranks_kernel: bad batch");
  MCPU_ARG_CHECK(vocab_size > 0 && vocab_size <= logits_stride, "vllm_ranks_kernel: vocab_size %lld out of range",
                 static_cast<long long>(vocab_size));
  if (batch == 0) return orSuccess;
  MCPU_ARG_CHECK(output && logits && token_ids, "vllm_ranks_kernel: NULL pointer");
  MCPU_ARG_CHECK(batch <= (1LL << 31) / sampler::kCluster - 1, "vllm_ranks_kernel: too many rows");
  const dim3 grid(static_cast<unsigned>(batch * sampler::kCluster));
  cudaStream_t st = as_cuda(stream);
  if (dtype == MCPU_FLOAT32)
    sampler::ranks_kernel<float><<<grid, sampler::kThreads, 0, st>>>(output, static_cast<const float*>(logits),
                                                                       logits_stride, token_ids, vocab_size);
  else if (dtype == MCPU_FLOAT16)
    sampler::ranks_kernel<__half><<<grid, sampler::kThreads, 0, st>>>(output, static_cast<const __half*>(logits),
                                                                        logits_stride, token_ids, vocab_size);
  else
    sampler::ranks_kernel<__nv_bfloat16><<<grid, sampler::kThreads, 0, st>>>(
        output, static_cast<const __nv_bfloat16*>(logits), logits_stride, token_ids, vocab_size);
  return from_cuda(cudaGetLastError(), "vllm_ranks_kernel launch");
}

extern "C" orError_t mcpu_vllm_penalties(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                         const int32_t* expanded_idx_mapping, const int32_t* token_ids,
                                         const int32_t* expanded_local_pos, const float* repetition_penalty,
                                         const float* frequency_penalty, const float* presence_penalty,
                                         int64_t max_num_reqs, const int32_t* prompt_bin_mask, int64_t pbm_stride,
                                         const int32_t* output_bin_counts, int64_t obc_stride, int64_t vocab_size,
                                         int64_t max_spec_len, orStream_t stream) {
  orError_t e = sampler::check_float(dtype, "vllm_penalties_kernel");
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(num_tokens >= 0 && num_tokens < (1LL << 31), "vllm_penalties_kernel: bad num_tokens");
  MCPU_ARG_CHECK(vocab_size > 0 && vocab_size <= logits_stride && vocab_size <= obc_stride &&
                     vocab_size <= pbm_stride * 32 && vocab_size < (1LL << 31),
                 "vllm_penalties_kernel: vocab_size %lld out of range", static_cast<long long>(vocab_size));
  MCPU_ARG_CHECK(max_num_reqs > 0, "vllm_penalties_kernel: no requests");
  if (num_tokens == 0) return orSuccess;
  MCPU_ARG_CHECK(logits && expanded_idx_mapping && token_ids && expanded_local_pos && repetition_penalty &&
                     frequency_penalty && presence_penalty && prompt_bin_mask && output_bin_counts,
                 "vllm_penalties_kernel: NULL pointer");
  const int64_t chunks = (vocab_size + sampler::kPenChunk - 1) / sampler::kPenChunk;
  MCPU_ARG_CHECK(chunks <= 65535, "vllm_penalties_kernel: vocab_size too large");
  const dim3 grid(static_cast<unsigned>(num_tokens), static_cast<unsigned>(chunks));
  cudaStream_t st = as_cuda(stream);
#define MCPU_PENALTIES(T)                                                                                      \
  sampler::penalties_kernel<T><<<grid, sampler::kThreads, 0, st>>>(                                            \
      static_cast<T*>(logits), logits_stride, vocab_size, expanded_idx_mapping, token_ids, expanded_local_pos, \
      repetition_penalty, frequency_penalty, presence_penalty, max_num_reqs, prompt_bin_mask, pbm_stride,      \
      output_bin_counts, obc_stride, max_spec_len)
  if (dtype == MCPU_FLOAT32)
    MCPU_PENALTIES(float);
  else if (dtype == MCPU_FLOAT16)
    MCPU_PENALTIES(__half);
  else
    MCPU_PENALTIES(__nv_bfloat16);
#undef MCPU_PENALTIES
  return from_cuda(cudaGetLastError(), "vllm_penalties_kernel launch");
}

extern "C" orError_t mcpu_vllm_bincount(const int32_t* expanded_idx_mapping, int64_t num_reqs,
                                        const int32_t* all_token_ids, int64_t tids_stride, int64_t max_seq_len,
                                        const int32_t* prompt_len, const int32_t* prefill_len, int64_t max_num_reqs,
                                        int32_t* prompt_bin_mask, int64_t packed_cols, int64_t pbm_stride,
                                        int32_t* output_bin_counts, int64_t vocab_size, int64_t obc_stride,
                                        orStream_t stream) {
  MCPU_ARG_CHECK(num_reqs >= 0 && num_reqs < (1LL << 31), "vllm_bincount_kernel: bad num_reqs");
  MCPU_ARG_CHECK(max_seq_len >= 0 && max_seq_len <= tids_stride && packed_cols >= 0 && packed_cols <= pbm_stride &&
                     vocab_size >= 0 && vocab_size <= obc_stride,
                 "vllm_bincount_kernel: sizes exceed their strides");
  if (num_reqs == 0) return orSuccess;
  MCPU_ARG_CHECK(max_num_reqs > 0, "vllm_bincount_kernel: no requests");
  MCPU_ARG_CHECK(expanded_idx_mapping && all_token_ids && prompt_len && prefill_len && prompt_bin_mask &&
                     output_bin_counts,
                 "vllm_bincount_kernel: NULL pointer");
  sampler::bincount_kernel<<<static_cast<unsigned>(num_reqs), sampler::kThreads, 0, as_cuda(stream)>>>(
      expanded_idx_mapping, all_token_ids, tids_stride, max_seq_len, prompt_len, prefill_len, max_num_reqs,
      prompt_bin_mask, packed_cols, pbm_stride, output_bin_counts, vocab_size, obc_stride);
  return from_cuda(cudaGetLastError(), "vllm_bincount_kernel launch");
}

extern "C" orError_t mcpu_vllm_bias(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                    int64_t vocab_size, const int32_t* expanded_idx_mapping, int64_t max_num_reqs,
                                    const int32_t* num_allowed, const int32_t* allowed, int64_t allowed_stride,
                                    int64_t allowed_cols, const int32_t* num_bias, const int32_t* bias_ids,
                                    int64_t bias_ids_stride, const float* bias, int64_t bias_stride,
                                    int64_t bias_cols, const int64_t* pos, const int32_t* min_lens,
                                    const int32_t* num_stop, const int32_t* stop_ids, int64_t stop_stride,
                                    int64_t stop_cols, orStream_t stream) {
  orError_t e = sampler::check_float(dtype, "vllm_bias_kernel");
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(num_tokens >= 0 && num_tokens < (1LL << 31), "vllm_bias_kernel: bad num_tokens");
  MCPU_ARG_CHECK(vocab_size > 0 && vocab_size <= logits_stride && vocab_size < (1LL << 31),
                 "vllm_bias_kernel: vocab_size %lld out of range", static_cast<long long>(vocab_size));
  MCPU_ARG_CHECK(allowed_cols >= 0 && allowed_cols <= allowed_stride && bias_cols >= 0 &&
                     bias_cols <= bias_ids_stride && bias_cols <= bias_stride && stop_cols >= 0 &&
                     stop_cols <= stop_stride,
                 "vllm_bias_kernel: list widths exceed their strides");
  if (num_tokens == 0) return orSuccess;
  MCPU_ARG_CHECK(max_num_reqs > 0, "vllm_bias_kernel: no requests");
  MCPU_ARG_CHECK(logits && expanded_idx_mapping && num_allowed && allowed && num_bias && bias_ids && bias && pos &&
                     min_lens && num_stop && stop_ids,
                 "vllm_bias_kernel: NULL pointer");
  const dim3 grid(static_cast<unsigned>(num_tokens));
  cudaStream_t st = as_cuda(stream);
#define MCPU_BIAS(T)                                                                                               \
  sampler::bias_kernel<T><<<grid, sampler::kThreads, 0, st>>>(                                                     \
      static_cast<T*>(logits), logits_stride, vocab_size, expanded_idx_mapping, max_num_reqs, num_allowed, allowed, \
      allowed_stride, allowed_cols, num_bias, bias_ids, bias_ids_stride, bias, bias_stride, bias_cols, pos,         \
      min_lens, num_stop, stop_ids, stop_stride, stop_cols)
  if (dtype == MCPU_FLOAT32)
    MCPU_BIAS(float);
  else if (dtype == MCPU_FLOAT16)
    MCPU_BIAS(__half);
  else
    MCPU_BIAS(__nv_bfloat16);
#undef MCPU_BIAS
  return from_cuda(cudaGetLastError(), "vllm_bias_kernel launch");
}

extern "C" orError_t mcpu_vllm_bad_words(void* logits, int dtype, int64_t num_tokens, int64_t logits_stride,
                                         int64_t vocab_size, const int32_t* expanded_idx_mapping,
                                         int64_t max_num_reqs, const int32_t* bad_word_token_ids,
                                         int64_t bw_ids_stride, int64_t bw_ids_cols,
                                         const int32_t* bad_word_offsets, int64_t bw_off_stride,
                                         int64_t bw_off_cols, const int32_t* num_bad_words,
                                         const int32_t* all_token_ids, int64_t token_ids_stride,
                                         int64_t max_seq_len, const int32_t* prompt_len, const int32_t* total_len,
                                         const int32_t* input_ids, const int32_t* expanded_local_pos,
                                         orStream_t stream) {
  orError_t e = sampler::check_float(dtype, "vllm_bad_words_kernel");
  if (e != orSuccess) return e;
  MCPU_ARG_CHECK(num_tokens >= 0 && num_tokens < (1LL << 31), "vllm_bad_words_kernel: bad num_tokens");
  MCPU_ARG_CHECK(vocab_size > 0 && vocab_size <= logits_stride && vocab_size < (1LL << 31),
                 "vllm_bad_words_kernel: vocab_size %lld out of range", static_cast<long long>(vocab_size));
  MCPU_ARG_CHECK(bw_ids_cols >= 0 && bw_ids_cols <= bw_ids_stride && bw_off_cols >= 0 &&
                     bw_off_cols <= bw_off_stride && max_seq_len >= 0 && max_seq_len <= token_ids_stride,
                 "vllm_bad_words_kernel: widths exceed their strides");
  if (num_tokens == 0) return orSuccess;
  MCPU_ARG_CHECK(max_num_reqs > 0, "vllm_bad_words_kernel: no requests");
  MCPU_ARG_CHECK(logits && expanded_idx_mapping && bad_word_token_ids && bad_word_offsets && num_bad_words &&
                     all_token_ids && prompt_len && total_len && input_ids && expanded_local_pos,
                 "vllm_bad_words_kernel: NULL pointer");
  const dim3 grid(static_cast<unsigned>(num_tokens));
  cudaStream_t st = as_cuda(stream);
#define MCPU_BAD_WORDS(T)                                                                                        \
  sampler::bad_words_kernel<T><<<grid, sampler::kBadWordThreads, 0, st>>>(                                       \
      static_cast<T*>(logits), logits_stride, vocab_size, expanded_idx_mapping, max_num_reqs, bad_word_token_ids, \
      bw_ids_stride, bw_ids_cols, bad_word_offsets, bw_off_stride, bw_off_cols, num_bad_words, all_token_ids,     \
      token_ids_stride, max_seq_len, prompt_len, total_len, input_ids, expanded_local_pos)
  if (dtype == MCPU_FLOAT32)
    MCPU_BAD_WORDS(float);
  else if (dtype == MCPU_FLOAT16)
    MCPU_BAD_WORDS(__half);
  else
    MCPU_BAD_WORDS(__nv_bfloat16);
#undef MCPU_BAD_WORDS
  return from_cuda(cudaGetLastError(), "vllm_bad_words_kernel launch");
}
