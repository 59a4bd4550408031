/*
 * CPU oracle for the torch_mcpu device hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke
 * check in __graft_entry__.py and the CPU legs of bench.py (cpu_baseline and
 * --impl reference) call it.  Nothing in the product package links or calls
 * it; the product path is the CUDA library in torch_mcpu_b200/csrc.
 *
 * It restates, in plain C, the arithmetic the reference performs on its
 * simulated "mcpu" device (every citation is a path inside the reference
 * project kzwrime/torch_mcpu):
 *
 *   grouped_topk  tests/test_grouped_topk_compile.py:15-66, the reference's
 *                 copy of vLLM's grouped-top-k router, executed on mcpu as a
 *                 chain of aten ops (sigmoid/softmax, add, topk, sum/max,
 *                 scatter mask, masked_fill, topk, gather, div, mul).
 *   sigmoid       csrc/aten/ops/unary_out.cpp:46-49, the raw scalar loop
 *                 1.0f / (1.0f + std::exp(-x)) in fp32 (glibc expf).
 *   silu          csrc/aten/ops/unary_out.cpp:50-51, x / (1.0f + std::exp(-x)).
 *   mul           csrc/aten/ops/binary_out.cpp:544-560 -> at::mul_out (CPU):
 *                 bf16 operands widened to fp32, product rounded to bf16.
 *   rms_norm      vLLM 0.22 vllm/ir/ops/layernorm.py:10-21 (third party),
 *                 evaluated on mcpu as pow -> mean
 *                 (csrc/aten/ops/reduction_scatter.cpp:248-285) -> add ->
 *                 rsqrt -> mul -> to(bf16) -> mul(weight).
 *
 * Exponential modes.  The reference's sigmoid/silu call glibc expf, which is
 * not correctly rounded on about 7.6e-5 of fp32 inputs.  ORACLE_EXP_GLIBC
 * reproduces the reference exactly on this host; ORACLE_EXP_CR uses the
 * correctly rounded value (float)exp((double)x), which is the definition the
 * CUDA kernels implement on their exact path.  Tests run both and report the
 * rows on which the two differ.
 *
 * Selection semantics (grouped_topk).  ATen's CPU topk does not break ties
 * toward the lower index and its sorted=False order is an implementation
 * artefact, so this oracle defines: rank by key descending, ties to the lower
 * index; emit the top-k in that order.  The key is the biased score
 * (score + bias) when a bias is given (reference lines 37-42, 55-57) and the
 * raw logit otherwise (softmax and sigmoid are monotone, so the selected set
 * equals the reference's except where the reference's rounded scores tie,
 * which the tie flag reports).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORACLE_EXP_GLIBC = 0, ORACLE_EXP_CR = 1 };
enum { ORACLE_F32 = 0, ORACLE_BF16 = 1 };
enum { ORACLE_SOFTMAX = 0, ORACLE_SIGMOID = 1 };

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round-to-nearest-even fp32 -> bf16 (c10::BFloat16's conversion for finite
 * values; NaN is kept quiet). */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

static inline float oracle_expf(float x, int mode) {
  if (mode == ORACLE_EXP_CR) return (float)exp((double)x);
  return expf(x);
}

/* csrc/aten/ops/unary_out.cpp:46-49 */
static inline float sigmoid_f(float x, int mode) {
  return 1.0f / (1.0f + oracle_expf(-x, mode));
}

/* csrc/aten/ops/unary_out.cpp:50-51 */
static inline float silu_f(float x, int mode) {
  return x / (1.0f + oracle_expf(-x, mode));
}

static inline int better(float a, int ia, float b, int ib) {
  /* a ranks before b: larger key first, equal keys -> lower index first */
  return (a > b) || (a == b && ia < ib);
}

static float rel_gap(float a, float b) {
  if (isinf(b) && b < 0) return INFINITY;
  float m = fmaxf(fabsf(a), fabsf(b));
  if (m < 1e-30f) m = 1e-30f;
  return (a - b) / m;
}

/*
 * grouped_topk for one row.  Returns 1 when an exact tie sits on a selection
 * boundary (group pick or expert pick), 0 otherwise; *gap gets the smallest
 * relative gap across those boundaries.
 */
static int grouped_topk_row(const float* x, int E, int G, int TG, int K,
                            int renorm, float scale, const float* bias,
                            int scoring, int in_bf16, int exp_mode,
                            float* w_out, int32_t* id_out, float* gap,
                            float* scores, float* keys) {
  const int GS = E / G;
  /* scores: tests/test_grouped_topk_compile.py:28-33 */
  if (scoring == ORACLE_SIGMOID) {
    for (int e = 0; e < E; ++e) {
      float s = sigmoid_f(x[e], exp_mode);
      scores[e] = in_bf16 ? round_bf16(s) : s;
    }
  } else {
    float m = -INFINITY;
    for (int e = 0; e < E; ++e) m = fmaxf(m, x[e]);
    float sum = 0.0f;
    for (int e = 0; e < E; ++e) {
      scores[e] = oracle_expf(x[e] - m, exp_mode);
      sum += scores[e];
    }
    for (int e = 0; e < E; ++e) {
      float s = scores[e] / sum;
      scores[e] = in_bf16 ? round_bf16(s) : s;
    }
  }
  /* ranking keys: lines 36-45 (biased scores) or the monotone logit */
  float gs[1024];
  if (bias) {
    for (int e = 0; e < E; ++e) keys[e] = scores[e] + bias[e];
    for (int g = 0; g < G; ++g) {
      float m1 = -INFINITY, m2 = -INFINITY;
      for (int j = 0; j < GS; ++j) {
        float v = keys[g * GS + j];
        if (v > m1) {
          m2 = m1;
          m1 = v;
        } else if (v > m2) {
          m2 = v;
        }
      }
      gs[g] = m1 + m2; /* topk(2)[0].sum(-1) */
    }
  } else {
    for (int e = 0; e < E; ++e) keys[e] = x[e];
    for (int g = 0; g < G; ++g) {
      float m1 = -INFINITY;
      for (int j = 0; j < GS; ++j) m1 = fmaxf(m1, keys[g * GS + j]);
      gs[g] = m1; /* max(dim=-1).values */
    }
  }
  int tie = 0;
  float min_gap = INFINITY;
  /* group pick: topk(group_scores, k=topk_group), lines 47-55 */
  int gorder[1024];
  for (int g = 0; g < G; ++g) gorder[g] = g;
  for (int i = 1; i < G; ++i) { /* insertion sort, G is small */
    int v = gorder[i], j = i - 1;
    while (j >= 0 && better(gs[v], v, gs[gorder[j]], gorder[j])) {
      gorder[j + 1] = gorder[j];
      --j;
    }
    gorder[j + 1] = v;
  }
  unsigned char gsel[1024];
  memset(gsel, 0, (size_t)G);
  for (int i = 0; i < TG; ++i) gsel[gorder[i]] = 1;
  if (TG < G) {
    float a = gs[gorder[TG - 1]], b = gs[gorder[TG]];
    if (a == b) tie = 1;
    float r = rel_gap(a, b);
    if (r < min_gap) min_gap = r;
  }
  /* expert pick among unmasked experts: lines 56-60 */
  int best[64];
  int nb = 0;
  for (int e = 0; e < E; ++e) {
    if (!gsel[e / GS]) continue;
    /* keep the best K+1 (the extra one measures the boundary gap) */
    int cap = K + 1;
    if (nb < cap) {
      int j = nb++;
      while (j > 0 && better(keys[e], e, keys[best[j - 1]], best[j - 1])) {
        best[j] = best[j - 1];
        --j;
      }
      best[j] = e;
    } else if (better(keys[e], e, keys[best[cap - 1]], best[cap - 1])) {
      int j = cap - 1;
      while (j > 0 && better(keys[e], e, keys[best[j - 1]], best[j - 1])) {
        best[j] = best[j - 1];
        --j;
      }
      best[j] = e;
    }
  }
  if (nb > K) {
    float a = keys[best[K - 1]], b = keys[best[K]];
    if (a == b) tie = 1;
    float r = rel_gap(a, b);
    if (r < min_gap) min_gap = r;
  }
  /* weights: gather of unbiased scores (line 58) or the top-k values of the
   * softmax/sigmoid scores (line 60); renormalise (62-63); scale (65-66) */
  float w[64];
  for (int k = 0; k < K; ++k) w[k] = scores[best[k]];
  if (renorm) {
    float sum = 0.0f;
    for (int k = 0; k < K; ++k) sum += w[k];
    if (in_bf16) sum = round_bf16(sum);
    for (int k = 0; k < K; ++k) {
      float q = w[k] / sum;
      w[k] = in_bf16 ? round_bf16(q) : q;
    }
  }
  if (scale != 1.0f) {
    for (int k = 0; k < K; ++k) {
      float q = w[k] * scale;
      w[k] = in_bf16 ? round_bf16(q) : q;
    }
  }
  for (int k = 0; k < K; ++k) {
    w_out[k] = w[k];
    id_out[k] = best[k];
  }
  if (gap) *gap = min_gap;
  return tie;
}

/*
 * Returns 0 on success, a negative code on bad arguments.
 * gating: [T, E] fp32 or bf16 (row-major); bias: [E] fp32 or NULL.
 * tie_rows (optional): 1 where an exact tie sits on a selection boundary.
 * gaps (optional): smallest relative gap at a selection boundary per row.
 */
int oracle_grouped_topk(const void* gating, int in_dtype, int64_t T, int E,
                        int G, int TG, int K, int renorm, float scale,
                        const float* bias, int scoring, int exp_mode,
                        float* w_out, int32_t* id_out, uint8_t* tie_rows,
                        float* gaps, int nthreads) {
  if (E <= 0 || E > 1024 || G <= 0 || E % G != 0 || TG <= 0 || TG > G ||
      K <= 0 || K > 63 || K > TG * (E / G))
    return -1;
  if (bias && E / G < 2) return -2;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
  {
    float xr[1024], scores[1024], keys[1024];
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int64_t t = 0; t < T; ++t) {
      if (in_dtype == ORACLE_BF16) {
        const uint16_t* row = (const uint16_t*)gating + t * (int64_t)E;
        for (int e = 0; e < E; ++e) xr[e] = bf16_to_f32(row[e]);
      } else {
        memcpy(xr, (const float*)gating + t * (int64_t)E, sizeof(float) * (size_t)E);
      }
      float gap = 0.0f;
      int tie = grouped_topk_row(xr, E, G, TG, K, renorm, scale, bias, scoring,
                                 in_dtype == ORACLE_BF16, exp_mode,
                                 w_out + t * K, id_out + t * K, &gap, scores,
                                 keys);
      if (tie_rows) tie_rows[t] = (uint8_t)tie;
      if (gaps) gaps[t] = gap;
    }
  }
  return 0;
}

/* silu_and_mul on bf16: out[t, j] = bf16(bf16(silu(a)) * b) with
 * a = x[t, j], b = x[t, d + j]  (vLLM SiluAndMul.forward_native,
 * activation.py:135-139, run on mcpu as raw silu then aten mul). */
int oracle_silu_and_mul_bf16(const uint16_t* x, int64_t T, int64_t d,
                             uint16_t* out, int exp_mode, int nthreads) {
  if (T < 0 || d < 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* row = x + t * 2 * d;
    for (int64_t j = 0; j < d; ++j) {
      float a = bf16_to_f32(row[j]);
      float b = bf16_to_f32(row[d + j]);
      float s = round_bf16(silu_f(a, exp_mode));
      out[t * d + j] = f32_to_bf16(s * b);
    }
  }
  return 0;
}

/* rms_norm on bf16 (vllm/ir/ops/layernorm.py:14-21):
 *   xf = float(x); var = mean(xf*xf); y = bf16(xf * (1/sqrt(var + eps)));
 *   out = bf16(float(y) * float(w)).
 * The mean is accumulated in double and rounded once (the reference's
 * vectorised fp32 sum differs only in summation order). */
int oracle_rms_norm_bf16(const uint16_t* x, const uint16_t* w, int64_t T,
                         int64_t H, float eps, uint16_t* out, int nthreads) {
  if (T < 0 || H <= 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (int64_t t = 0; t < T; ++t) {
    const uint16_t* row = x + t * H;
    double acc = 0.0;
    for (int64_t j = 0; j < H; ++j) {
      float v = bf16_to_f32(row[j]);
      acc += (double)(v * v);
    }
    float var = (float)(acc / (double)H);
    float r = 1.0f / sqrtf(var + eps);
    for (int64_t j = 0; j < H; ++j) {
      float y = round_bf16(bf16_to_f32(row[j]) * r);
      out[t * H + j] = f32_to_bf16(y * bf16_to_f32(w[j]));
    }
  }
  return 0;
}

/* Elementwise sigmoid, exposed so tests can compare exponential modes. */
void oracle_sigmoid_f32(const float* x, int64_t n, float* out, int exp_mode) {
  for (int64_t i = 0; i < n; ++i) out[i] = sigmoid_f(x[i], exp_mode);
}

/* The reference's raw silu loop on bf16 (csrc/aten/ops/unary_out.cpp:46-51,
 * raw_unary_value<Silu>): one thread, element by element, fp32 arithmetic,
 * rounded to bf16.  `rows` rows of `d` values at row pitch `pitch`
 * (elements) in, dense [rows, d] out. */
void oracle_silu_raw_bf16(const uint16_t* x, int64_t rows, int64_t d, int64_t pitch, uint16_t* out,
                          int exp_mode) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < d; ++j)
      out[r * d + j] = f32_to_bf16(silu_f(bf16_to_f32(x[r * pitch + j]), exp_mode));
}
