/*
 * moe_oracle.c — CPU oracle for the INT4 weight-only MoE expert-FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * legs may load the shared library built from it.  The CUDA library under
 * llm-on-cpu_b200/ never links or calls it.
 *
 * It restates, in plain scalar C, the arithmetic of appolloqin/llm-on-cpu for
 * this path, in the same operation order as the reference's AVX2/FMA build so
 * that the fp32 results are bitwise identical to it:
 *
 *   fp16/bf16 decode ........ src/hal/cpu_ops.h:15-49
 *   INT4 AWQ-sym GEMV ....... src/hal/int4_ops.cpp:54-80 (dot), :204-299 (rows)
 *   INT4 GPTQ-asym GEMV ..... src/hal/int4_ops.cpp:82-108 (dot), :301-320 (rows)
 *   INT4 batch GEMM ......... src/hal/int4_ops.cpp:621-638 (same per-row math)
 *   INT4 dequant row ........ src/hal/int4_ops.cpp:640-668
 *   BF16 router GEMV ........ src/hal/cpu_ops.cpp:57-95 (gemm_bias_free)
 *   SiLU * up ............... src/hal/cpu_ops.cpp:228-251
 *   softmax/top-k/renorm .... src/model/qwen3_6_moe_int4_model.cpp:386-402
 *   expert FFN + combine .... src/model/qwen3_6_moe_int4_model.cpp:184-232
 *   shared expert ........... src/model/qwen3_6_moe_int4_model.cpp:352-374
 *   AWQ-sym quantizer ....... tools/quantize_int4.py:115-124, :150-166
 *   GPTQ-asym quantizer ..... tools/quantize_int4.py:127-147
 *
 * The AVX2 kernels keep 32 fp32 FMA chains per dot product (4 ymm registers
 * x 8 lanes; chain j covers k = k0 + j (mod 32)) and fold them with a fixed
 * tree: a[i] = (c[i]+c[8+i]) + (c[16+i]+c[24+i]); b[i] = a[i]+a[4+i];
 * r = (b0+b1) + (b2+b3) (hsum256, int4_ops.cpp:27-36).  Outside the explicit
 * intrinsics, GCC (-O3 -mfma, GNU mode => -ffp-contract=fast) contracts
 * `acc += a * b` into one fused multiply-add; this file writes those as fmaf()
 * and is compiled with -ffp-contract=off so that only the explicit fmaf() calls
 * fuse.  The bit-exact agreement is pinned by tests against fixtures produced
 * by the reference's own compiled sources.
 *
 * Parts with no counterpart in the reference (restated from the path's
 * specification, parity pinned only by this file and its tests):
 *   - sigmoid + per-expert-bias router with routed scaling;
 *   - canonical token->expert permutation (stable by expert, token, slot);
 *   - top-k on logits with ties broken by the smaller expert id (the
 *     reference's std::partial_sort leaves tie order unspecified).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

enum { ORC_SCHEME_GPTQ_ASYM = 1, ORC_SCHEME_AWQ_SYM = 2 };
enum { ORC_ROUTER_SOFTMAX = 0, ORC_ROUTER_SIGMOID_BIAS = 1 };

/* ------------------------------------------------------------------ */
/* scalar conversions (cpu_ops.h:15-49)                                */
/* ------------------------------------------------------------------ */

ORC_API float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1u;
  const uint32_t ex = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  uint32_t out;
  if (ex == 0) {
    if (man == 0) {
      out = sign << 31;
    } else {
      float f = ldexpf((float)man, -24);
      return sign ? -f : f;
    }
  } else if (ex == 31) {
    out = (sign << 31) | 0x7F800000u | (man << 13);
  } else {
    out = (sign << 31) | ((ex + (127 - 15)) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &out, sizeof f);
  return f;
}

ORC_API float orc_bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* round-to-nearest-even, no NaN special case (cpu_ops.h:44-49) */
ORC_API uint16_t orc_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* IEEE binary16 round-to-nearest-even (numpy astype(np.float16), the
 * conversion tools/quantize_int4.py:42-43 relies on). */
ORC_API uint16_t orc_f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, sizeof x);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
  if (ax < 0x38800000u) {                                    /* f16 subnormal / zero */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* < 2^-25: rounds to 0 */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e; /* 14..24 */
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (r & 1u))) r += 1u;
    return (uint16_t)(sign | r);
  }
  uint32_t r = ((ax >> 13) - (112u << 10)); /* rebias exponent 127 -> 15 */
  const uint32_t rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1u;
  return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------ */
/* 32-chain dot products (int4_ops.cpp:27-108, cpu_ops.cpp:65-86)       */
/* ------------------------------------------------------------------ */

static inline float orc_fold32(const float c[32]) {
  float a[8], b[4];
  for (int i = 0; i < 8; ++i) a[i] = (c[i] + c[8 + i]) + (c[16 + i] + c[24 + i]);
  for (int i = 0; i < 4; ++i) b[i] = a[i] + a[4 + i];
  return (b[0] + b[1]) + (b[2] + b[3]);
}

static inline int orc_nib(const uint8_t* qrow, int k) {
  const uint8_t b = qrow[k >> 1];
  return (k & 1) ? ((b >> 4) & 0xF) : (b & 0xF);
}

/* dot_awq_noscale (int4_ops.cpp:54-80): sum_k x[k] * (q[k] - zp) */
static float orc_dot_awq_noscale(const float* x, const uint8_t* qrow, int k0, int k1, float zp) {
  float c[32];
  for (int j = 0; j < 32; ++j) c[j] = 0.f;
  int k = k0;
  for (; k + 32 <= k1; k += 32)
    for (int j = 0; j < 32; ++j) c[j] = fmaf(x[k + j], (float)orc_nib(qrow, k + j) - zp, c[j]);
  float acc = orc_fold32(c);
  for (; k < k1; ++k) acc = fmaf(x[k], (float)orc_nib(qrow, k) - zp, acc);
  return acc;
}

/* dot_gptq_avx2 (int4_ops.cpp:82-108): sum_k x[k] * (q[k]*scale + zero) */
static float orc_dot_gptq(const float* x, const uint8_t* qrow, int k0, int k1, float scale,
                          float zero) {
  float c[32];
  for (int j = 0; j < 32; ++j) c[j] = 0.f;
  int k = k0;
  for (; k + 32 <= k1; k += 32)
    for (int j = 0; j < 32; ++j)
      c[j] = fmaf(x[k + j], fmaf((float)orc_nib(qrow, k + j), scale, zero), c[j]);
  float acc = orc_fold32(c);
  for (; k < k1; ++k) acc = fmaf(x[k], fmaf((float)orc_nib(qrow, k), scale, zero), acc);
  return acc;
}

/* ------------------------------------------------------------------ */
/* INT4 view and GEMV / GEMM / dequant                                  */
/* ------------------------------------------------------------------ */

/* Mirrors qlwc::Int4View (src/weights/qlwc_store.h:17-27). */
typedef struct {
  const uint8_t* qweight;  /* [M, ceil(K/2)] low nibble = even k */
  const uint16_t* scales;  /* [M, ng] fp16 bits */
  const uint16_t* zeros;   /* [M, ng] fp16 bits (GPTQ) or NULL */
  int M, K, group_size;
  int scheme;              /* ORC_SCHEME_* */
  int awq_zp;              /* <= 0 -> 7 */
} orc_int4_view;

static inline int orc_ng(const orc_int4_view* W) {
  return (W->K + W->group_size - 1) / W->group_size;
}

/* One output row.  `single` selects the arithmetic of the reference's
 * single-row code path (finish_1, int4_ops.cpp:230-239, and the single-row
 * loops of the batch kernel, :507-519, :552-563): there the compiled
 * reference keeps the per-group `acc += dot * scale` as a multiply then an
 * add, while the 2- and 4-row paths (:240-257, :262-289) fuse it into one
 * FMA.  GPTQ rows add the group dot without a multiply, so both agree. */
static float orc_row(const float* x, const orc_int4_view* W, int m, int single) {
  const int K = W->K, gs = W->group_size, ng = orc_ng(W);
  const size_t rb = (size_t)((K + 1) / 2);
  const uint8_t* qrow = W->qweight + (size_t)m * rb;
  float acc = 0.f;
  if (W->scheme == ORC_SCHEME_AWQ_SYM) {
    const float zp = (float)(W->awq_zp > 0 ? W->awq_zp : 7);
    for (int g = 0; g < ng; ++g) {
      const int k0 = g * gs;
      const int k1 = (K < k0 + gs) ? K : k0 + gs;
      const float s = orc_f16_to_f32(W->scales[(size_t)m * ng + g]);
      const float p = orc_dot_awq_noscale(x, qrow, k0, k1, zp);
      if (single) {
        const float ps = p * s;
        acc = acc + ps;
      } else {
        acc = fmaf(p, s, acc); /* int4_ops.cpp:228 */
      }
    }
  } else {
    for (int g = 0; g < ng; ++g) {
      const int k0 = g * gs;
      const int k1 = (K < k0 + gs) ? K : k0 + gs;
      const float s = orc_f16_to_f32(W->scales[(size_t)m * ng + g]);
      const float z = W->zeros ? orc_f16_to_f32(W->zeros[(size_t)m * ng + g]) : 0.f;
      acc += orc_dot_gptq(x, qrow, k0, k1, s, z); /* int4_ops.cpp:316 */
    }
  }
  return isfinite(acc) ? acc : 0.f;
}

/* Whether the reference computes row m on its single-row path.  AWQ GEMV
 * (int4_ops.cpp:259-298): M >= 4096 walks rows in fours and hands a 2- or
 * 3-row remainder to finish_2, a 1-row remainder to finish_1; smaller M
 * walks pairs with an odd last row on finish_1.  The batch kernel
 * (:475-566) walks fours with remainder rows one by one for M >= 4096, pairs
 * otherwise.  Reference defect, not reproduced: for M >= 4096 with
 * M = 3 (mod 4) its GEMV never writes row M-1 (finish_2 covers two of the
 * three remainder rows); the oracle computes that row on the single path. */
static int orc_is_single_row(int M, int m, int batch) {
  if (M >= 4096) {
    const int rem = M % 4;
    if (m < M - rem) return 0;
    if (batch || rem == 1) return 1;
    return rem == 3 && m == M - 1;
  }
  return (M & 1) && m == M - 1;
}

/* hal::gemm_int4 (int4_ops.cpp:422-443): y[M] = W[M,K] . x[K] */
ORC_API void orc_gemm_int4(const float* x, const orc_int4_view* W, float* y) {
  for (int m = 0; m < W->M; ++m) y[m] = orc_row(x, W, m, orc_is_single_row(W->M, m, 0));
}

/* Row value of hal::gemm_int4_argmax (int4_ops.cpp:344-381).  AWQ: per group
 * dot_awq_noscale(x, q, zp) x scale accumulated in fp32 (:365-369); GPTQ: the
 * scalar row gemm_row_scalar (:323-342), w = q * s + z in fp32 and the sum of
 * x[k] * w in double.  awq_fma / w_fma / acc_fma: whether those multiply-adds
 * are fused.  Against the compiled reference: the AWQ group sum is a multiply
 * then an add (the fused form differed in 3 of 12 cases); for GPTQ the four
 * forms gave the reference's result in all of 400 cases (the double sum hides
 * the difference), and the unfused one is used. */
static float orc_argmax_row(const float* x, const orc_int4_view* W, int m, int awq_fma, int w_fma, int acc_fma) {
  const int K = W->K, gs = W->group_size, ng = orc_ng(W);
  const size_t rb = (size_t)((K + 1) / 2);
  const uint8_t* qrow = W->qweight + (size_t)m * rb;
  if (W->scheme == ORC_SCHEME_AWQ_SYM) {
    const float zp = (float)(W->awq_zp > 0 ? W->awq_zp : 7);
    float acc = 0.f;
    for (int g = 0; g < ng; ++g) {
      const int k0 = g * gs;
      const int k1 = (K < k0 + gs) ? K : k0 + gs;
      const float s = orc_f16_to_f32(W->scales[(size_t)m * ng + g]);
      const float p = orc_dot_awq_noscale(x, qrow, k0, k1, zp);
      if (awq_fma) {
        acc = fmaf(p, s, acc);
      } else {
        const float ps = p * s;
        acc = acc + ps;
      }
    }
    return acc;
  }
  double acc = 0.0;
  for (int g = 0; g < ng; ++g) {
    const int k0 = g * gs;
    const int k1 = (K < k0 + gs) ? K : k0 + gs;
    const float s = orc_f16_to_f32(W->scales[(size_t)m * ng + g]);
    const float z = W->zeros ? orc_f16_to_f32(W->zeros[(size_t)m * ng + g]) : 0.f;
    for (int k = k0; k < k1; ++k) {
      const uint8_t b = qrow[k / 2];
      const int qi = (k & 1) ? ((b >> 4) & 0xF) : (b & 0xF);
      float w;
      if (w_fma) {
        w = fmaf((float)qi, s, z);
      } else {
        const float qs = (float)qi * s;
        w = qs + z;
      }
      if (acc_fma) {
        acc = fma((double)x[k], (double)w, acc);
      } else {
        const double xw = (double)x[k] * (double)w;
        acc = acc + xw;
      }
    }
  }
  return (float)acc;
}

static void orc_argmax_v(const float* x, const orc_int4_view* W, int32_t* index, float* value, int awq_fma,
                         int w_fma, int acc_fma) {
  int32_t bi = 0;
  float bv = -1e30f;
  for (int m = 0; m < W->M; ++m) {
    float v = orc_argmax_row(x, W, m, awq_fma, w_fma, acc_fma);
    if (!isfinite(v)) v = -1e30f; /* :376 */
    if (v > bv) {                 /* first maximum in row order (:424-431) */
      bv = v;
      bi = m;
    }
  }
  *index = bi;
  *value = bv;
}

/* hal::gemm_int4_argmax (int4_ops.cpp:344-446), the serial rule: the first
 * maximum in row order (the reference's OpenMP branch for M >= 4096 breaks
 * ties between threads by timing; with one thread it is this rule). */
ORC_API void orc_gemm_int4_argmax(const float* x, const orc_int4_view* W, int32_t* index, float* value) {
  orc_argmax_v(x, W, index, value, 0, 0, 0);
}

/* hal::gemm_int4_batch (int4_ops.cpp:621-638): Y[n,M] = X[n,K] . W^T.  The
 * token-tiled AVX2 kernels compute each (t, m) with the same chains as the
 * single-token kernel; only the row grouping differs (orc_is_single_row). */
ORC_API void orc_gemm_int4_batch(const float* X, int n, const orc_int4_view* W, float* Y) {
  if (n == 1) {
    orc_gemm_int4(X, W, Y);
    return;
  }
#pragma omp parallel for schedule(static) if (n * (long)W->M * W->K > (1L << 22))
  for (int t = 0; t < n; ++t)
    for (int m = 0; m < W->M; ++m)
      Y[(size_t)t * W->M + m] =
          orc_row(X + (size_t)t * W->K, W, m, orc_is_single_row(W->M, m, 1));
}

/* hal::dequant_int4_row (int4_ops.cpp:640-662).  Returns 0, or -1 for a bad row. */
ORC_API int orc_dequant_int4_row(const orc_int4_view* W, int row, float* out) {
  if (row < 0 || row >= W->M) return -1;
  const int K = W->K, gs = W->group_size, ng = orc_ng(W);
  const int awq = W->scheme == ORC_SCHEME_AWQ_SYM;
  const float zp = (float)(W->awq_zp > 0 ? W->awq_zp : 7);
  const uint8_t* qrow = W->qweight + (size_t)row * (size_t)((K + 1) / 2);
  for (int g = 0; g < ng; ++g) {
    const int k0 = g * gs;
    const int k1 = (K < k0 + gs) ? K : k0 + gs;
    const float s = orc_f16_to_f32(W->scales[(size_t)row * ng + g]);
    const float z = (!awq && W->zeros) ? orc_f16_to_f32(W->zeros[(size_t)row * ng + g]) : 0.f;
    for (int k = k0; k < k1; ++k) {
      const int q = orc_nib(qrow, k);
      /* q*s is exact in fp32 (4-bit x 11-bit), so fma and mul+add agree */
      out[k] = awq ? ((float)q - zp) * s : fmaf((float)q, s, z);
    }
  }
  return 0;
}

ORC_API int orc_dequant_int4_matrix(const orc_int4_view* W, float* out) {
  if (!out || !W->qweight || W->M <= 0 || W->K <= 0) return -1;
  for (int r = 0; r < W->M; ++r) orc_dequant_int4_row(W, r, out + (size_t)r * W->K);
  return 0;
}

/* hal::gemm_bias_free, AVX2 branch (cpu_ops.cpp:57-86): y[M] = W16[M,K] . x.
 * w_is_f16 selects fp16 weights, else bf16. */
ORC_API void orc_gemm_bias_free(const float* x, const uint16_t* W, float* y, int M, int K,
                                int w_is_f16) {
  for (int m = 0; m < M; ++m) {
    const uint16_t* row = W + (size_t)m * K;
    float c[32];
    for (int j = 0; j < 32; ++j) c[j] = 0.f;
    int k = 0;
    for (; k + 32 <= K; k += 32)
      for (int j = 0; j < 32; ++j) {
        const float w = w_is_f16 ? orc_f16_to_f32(row[k + j]) : orc_bf16_to_f32(row[k + j]);
        c[j] = fmaf(x[k + j], w, c[j]);
      }
    float acc = orc_fold32(c);
    for (; k < K; ++k) {
      const float w = w_is_f16 ? orc_f16_to_f32(row[k]) : orc_bf16_to_f32(row[k]);
      const float xw = x[k] * w; /* this tail stays unfused in the reference build */
      acc = acc + xw;
    }
    y[m] = isfinite(acc) ? acc : 0.f;
  }
}

/* hal::silu_and_mul (cpu_ops.cpp:228-251) */
ORC_API void orc_silu_and_mul(const float* gate, const float* up, float* out, int n) {
  for (int i = 0; i < n; ++i) {
    const float g = gate[i];
    out[i] = (g / (1.f + expf(-g))) * up[i];
  }
}

/* ------------------------------------------------------------------ */
/* routing                                                              */
/* ------------------------------------------------------------------ */

/* Descending by key, ties by the smaller expert id.  Selection sort over the
 * first k positions (E <= a few hundred, k <= 64). */
static void orc_topk_desc(const float* key, int E, int k, int* ids) {
  unsigned char* used = (unsigned char*)calloc((size_t)E, 1);
  for (int j = 0; j < k; ++j) {
    int best = -1;
    for (int e = 0; e < E; ++e) {
      if (used[e]) continue;
      if (best < 0 || key[e] > key[best]) best = e;
    }
    used[best] = 1;
    ids[j] = best;
  }
  free(used);
}

/* Softmax router (qwen3_6_moe_int4_model.cpp:386-402, weights at :192/:287).
 * logits[E] in; ids[k], weights[k] out; probs[E] (optional) receives the
 * float probabilities the reference sorts on.  Selection is on logits (softmax
 * is monotone), ties to the smaller id.  Returns 1 when the k-th and (k+1)-th
 * probabilities are equal (the reference's order is then unspecified), else 0. */
ORC_API int orc_route_softmax(const float* logits_in, int E, int k, int* ids, float* weights,
                              float* probs_out) {
  float* p = (float*)malloc(sizeof(float) * (size_t)E);
  float m = logits_in[0];
  for (int e = 1; e < E; ++e)
    if (logits_in[e] > m) m = logits_in[e];
  double s = 0.0;
  for (int e = 0; e < E; ++e) {
    p[e] = expf(logits_in[e] - m);
    s += p[e];
  }
  for (int e = 0; e < E; ++e) p[e] = (float)(p[e] / s);
  orc_topk_desc(logits_in, E, k, ids);
  double wsum = 0.0;
  for (int j = 0; j < k; ++j) wsum += p[ids[j]];
  if (wsum < 1e-12) wsum = 1.0;
  for (int j = 0; j < k; ++j) weights[j] = (float)(p[ids[j]] / wsum);
  int tie = 0;
  if (k < E) {
    /* largest prob among the unselected vs the smallest selected */
    float kth = p[ids[k - 1]];
    for (int e = 0; e < E; ++e) {
      int sel = 0;
      for (int j = 0; j < k; ++j) sel |= (ids[j] == e);
      if (!sel && p[e] == kth) tie = 1;
    }
  }
  if (probs_out) memcpy(probs_out, p, sizeof(float) * (size_t)E);
  free(p);
  return tie;
}

/* sigmoid in double, rounded once to float: the CUDA path computes the same
 * expression, so both sides agree except where the double result sits within
 * one double ulp of a float rounding boundary. */
static inline float orc_sigmoid_f(float l) { return (float)(1.0 / (1.0 + exp(-(double)l))); }

/* Sigmoid + bias router (no counterpart in the reference; specified for the
 * GLM-4.5-Air / Kimi-K2 shapes).  s_e = sigmoid(l_e); experts chosen by
 * s_e + b_e (bias only for selection, ties to the smaller id); weights are
 * s_j / sum_sel s (double sum in selection order) times routed_scaling. */
ORC_API void orc_route_sigmoid_bias(const float* logits, const float* bias, int E, int k,
                                    float routed_scaling, int* ids, float* weights) {
  float* s = (float*)malloc(sizeof(float) * (size_t)E);
  float* sel = (float*)malloc(sizeof(float) * (size_t)E);
  for (int e = 0; e < E; ++e) {
    s[e] = orc_sigmoid_f(logits[e]);
    sel[e] = s[e] + bias[e];
  }
  orc_topk_desc(sel, E, k, ids);
  double wsum = 0.0;
  for (int j = 0; j < k; ++j) wsum += s[ids[j]];
  if (wsum < 1e-20) wsum = 1.0;
  for (int j = 0; j < k; ++j) weights[j] = (float)((double)s[ids[j]] / wsum) * routed_scaling;
  free(s);
  free(sel);
}

/* Canonical token->expert permutation: the (token t, slot j) pairs sorted
 * stably by expert id, then t, then j.  ids[T*kk] (kk slots per token, expert
 * ids in [0, n_exp)).  offsets[n_exp+1]; sorted[T*kk] holds t*kk+j;
 * inverse[t*kk+j] = position in sorted. */
ORC_API void orc_permute(const int* ids, int T, int kk, int n_exp, int* offsets, int* sorted,
                         int* inverse) {
  for (int e = 0; e <= n_exp; ++e) offsets[e] = 0;
  for (int p = 0; p < T * kk; ++p) offsets[ids[p] + 1] += 1;
  for (int e = 0; e < n_exp; ++e) offsets[e + 1] += offsets[e];
  int* cur = (int*)malloc(sizeof(int) * (size_t)(n_exp > 0 ? n_exp : 1));
  for (int e = 0; e < n_exp; ++e) cur[e] = offsets[e];
  for (int p = 0; p < T * kk; ++p) { /* p = t*kk + j is already (t, j) order */
    const int pos = cur[ids[p]]++;
    sorted[pos] = p;
    inverse[p] = pos;
  }
  free(cur);
}

/* ------------------------------------------------------------------ */
/* the MoE layer                                                        */
/* ------------------------------------------------------------------ */

typedef struct {
  orc_int4_view gate, up, down;
} orc_expert;

typedef struct {
  int H, I, E, topk;
  int router;              /* ORC_ROUTER_* */
  const uint16_t* router_w; /* [E, H] bf16 */
  const float* bias;       /* [E] (sigmoid router) */
  float routed_scaling;    /* sigmoid router */
  const orc_expert* experts; /* [E] */
  const orc_expert* shared;  /* NULL or one expert with the same (I, H) */
  float shared_scale;
  /* NULL, or the shared expert's gate row (bf16 [H]): the shared expert's
   * weight is then per token, sigmoid(gate . x) with the router's dot order
   * and the reference's float sigmoid (qwen3_6_moe_int4_model.cpp:29, :365-371) */
  const uint16_t* shared_gate_w;
} orc_layer;

/* One expert's SwiGLU FFN on one token: d[H] = down(silu(gate x) * up x)
 * (qwen3_6_moe_int4_model.cpp:195-199). */
static void orc_expert_ffn(const orc_expert* ex, const float* x, float* g, float* u, float* mid,
                           float* d) {
  orc_gemm_int4(x, &ex->gate, g);
  orc_gemm_int4(x, &ex->up, u);
  orc_silu_and_mul(g, u, mid, ex->gate.M);
  orc_gemm_int4(mid, &ex->down, d);
}

/* Per-token MoE FFN (moe_ffn_token, qwen3_6_moe_int4_model.cpp:377-404 with
 * the expert loop of :184-232 run on one thread and the shared expert of
 * :352-374).  X[T,H] fp32 in, Y[T,H] fp32 out (overwritten).  ids/weights
 * [T, topk] receive the routing; ties[T] (optional) flags softmax ties. */
ORC_API void orc_moe_layer_forward(const orc_layer* L, const float* X, int T, float* Y, int* ids,
                                   float* weights, int* ties) {
  const int H = L->H, I = L->I, E = L->E, K = L->topk;
#pragma omp parallel
  {
    float* logits = (float*)malloc(sizeof(float) * (size_t)E);
    float* g = (float*)malloc(sizeof(float) * (size_t)I);
    float* u = (float*)malloc(sizeof(float) * (size_t)I);
    float* mid = (float*)malloc(sizeof(float) * (size_t)I);
    float* d = (float*)malloc(sizeof(float) * (size_t)H);
#pragma omp for schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
      const float* x = X + (size_t)t * H;
      float* y = Y + (size_t)t * H;
      int* id = ids + (size_t)t * K;
      float* w = weights + (size_t)t * K;
      orc_gemm_bias_free(x, L->router_w, logits, E, H, 0);
      int tie = 0;
      if (L->router == ORC_ROUTER_SOFTMAX)
        tie = orc_route_softmax(logits, E, K, id, w, NULL);
      else
        orc_route_sigmoid_bias(logits, L->bias, E, K, L->routed_scaling, id, w);
      if (ties) ties[t] = tie;
      for (int h = 0; h < H; ++h) y[h] = 0.f;
      for (int j = 0; j < K; ++j) {
        orc_expert_ffn(&L->experts[id[j]], x, g, u, mid, d);
        for (int h = 0; h < H; ++h) y[h] = fmaf(w[j], d[h], y[h]);
      }
      if (L->shared) {
        float ss = L->shared_scale;
        if (L->shared_gate_w) {
          float gl;
          orc_gemm_bias_free(x, L->shared_gate_w, &gl, 1, H, 0);
          ss = 1.f / (1.f + expf(-gl));
        }
        orc_expert_ffn(L->shared, x, g, u, mid, d);
        for (int h = 0; h < H; ++h) y[h] = fmaf(ss, d[h], y[h]);
      }
    }
    free(logits);
    free(g);
    free(u);
    free(mid);
    free(d);
  }
}

/* The routing part of orc_moe_layer_forward for every token (router GEMV in
 * the reference's order, then its softmax or the sigmoid + bias selection):
 * logits[T,E], ids/weights[T,topk].  Tokens run in parallel (checker for
 * large batches; no expert weights are read). */
ORC_API void orc_moe_route(const orc_layer* L, const float* X, int T, float* logits, int* ids,
                           float* weights) {
  const int H = L->H, E = L->E, K = L->topk;
#pragma omp parallel for schedule(dynamic, 16)
  for (int t = 0; t < T; ++t) {
    float* lg = logits + (size_t)t * E;
    orc_gemm_bias_free(X + (size_t)t * H, L->router_w, lg, E, H, 0);
    if (L->router == ORC_ROUTER_SOFTMAX)
      orc_route_softmax(lg, E, K, ids + (size_t)t * K, weights + (size_t)t * K, NULL);
    else
      orc_route_sigmoid_bias(lg, L->bias, E, K, L->routed_scaling, ids + (size_t)t * K, weights + (size_t)t * K);
  }
}

/* Expert FFN with the routing given (the contract of hal::cuda::try_moe_ffn_int4,
 * src/hal/cuda_backend.cpp:5217-5317): y = sum_j w_j * ffn_j(x) in the given
 * order, experts with |w| < 1e-12 skipped, then the shared expert. */
ORC_API void orc_moe_ffn_routed(const float* x, int H, int I, const orc_expert* experts,
                                const float* w, int n, const orc_expert* shared,
                                float shared_scale, float* y) {
  float* g = (float*)malloc(sizeof(float) * (size_t)I);
  float* u = (float*)malloc(sizeof(float) * (size_t)I);
  float* mid = (float*)malloc(sizeof(float) * (size_t)I);
  float* d = (float*)malloc(sizeof(float) * (size_t)H);
  for (int h = 0; h < H; ++h) y[h] = 0.f;
  for (int j = 0; j < n; ++j) {
    if (fabsf(w[j]) < 1e-12f) continue;
    orc_expert_ffn(&experts[j], x, g, u, mid, d);
    for (int h = 0; h < H; ++h) y[h] = fmaf(w[j], d[h], y[h]);
  }
  if (shared && fabsf(shared_scale) > 0.f) {
    orc_expert_ffn(shared, x, g, u, mid, d);
    for (int h = 0; h < H; ++h) y[h] = fmaf(shared_scale, d[h], y[h]);
  }
  free(g);
  free(u);
  free(mid);
  free(d);
}

/* ------------------------------------------------------------------ */
/* quantizers (tools/quantize_int4.py)                                  */
/* ------------------------------------------------------------------ */

/* pack_int4 (:115-124): low nibble = even k. q[M,K] values 0..15. */
ORC_API void orc_pack_int4(const uint8_t* q, int M, int K, uint8_t* packed) {
  const int rb = (K + 1) / 2;
  for (int m = 0; m < M; ++m)
    for (int b = 0; b < rb; ++b) {
      const uint8_t lo = q[(size_t)m * K + 2 * b];
      const uint8_t hi = (2 * b + 1 < K) ? q[(size_t)m * K + 2 * b + 1] : 0;
      packed[(size_t)m * rb + b] = (uint8_t)(lo | (hi << 4));
    }
}

/* quant_awq_sym (:150-166): scale = max(absmax/7, 1e-8) (fp32),
 * q = clip(rint(W/scale) + 7, 0, 15), scales stored as fp16 (RNE).
 * bf16_scale != 0 first rounds the scale to bf16 (the BASELINE's "bf16 scale
 * per group", exactly representable in the fp16 slot) and quantizes with it. */
ORC_API void orc_quant_awq_sym(const float* W, int M, int K, int gs, int bf16_scale,
                               uint8_t* packed, uint16_t* scales_f16) {
  const int ng = K / gs, rb = K / 2;
  for (int m = 0; m < M; ++m) {
    const float* row = W + (size_t)m * K;
    uint8_t* prow = packed + (size_t)m * rb;
    for (int g = 0; g < ng; ++g) {
      float amax = 0.f;
      for (int k = g * gs; k < (g + 1) * gs; ++k) {
        const float a = fabsf(row[k]);
        if (a > amax) amax = a;
      }
      float s = amax / 7.0f;
      if (!(s > 1e-8f)) s = 1e-8f;
      if (bf16_scale) s = orc_bf16_to_f32(orc_f32_to_bf16(s));
      scales_f16[(size_t)m * ng + g] = orc_f32_to_f16_rne(s);
      for (int k = g * gs; k < (g + 1) * gs; k += 2) {
        float q0 = rintf(row[k] / s) + 7.0f, q1 = rintf(row[k + 1] / s) + 7.0f;
        q0 = q0 < 0.f ? 0.f : (q0 > 15.f ? 15.f : q0);
        q1 = q1 < 0.f ? 0.f : (q1 > 15.f ? 15.f : q1);
        prow[k / 2] = (uint8_t)((uint8_t)q0 | ((uint8_t)q1 << 4));
      }
    }
  }
}

/* quant_gptq_asym (:127-147): scale = max((max-min)/15, 1e-8), zero = min,
 * q = clip(rint((W - zero)/scale), 0, 15); scales and zeros as fp16 (RNE). */
ORC_API void orc_quant_gptq_asym(const float* W, int M, int K, int gs, uint8_t* packed,
                                 uint16_t* scales_f16, uint16_t* zeros_f16) {
  const int ng = K / gs, rb = K / 2;
  for (int m = 0; m < M; ++m) {
    const float* row = W + (size_t)m * K;
    uint8_t* prow = packed + (size_t)m * rb;
    for (int g = 0; g < ng; ++g) {
      float mn = row[g * gs], mx = row[g * gs];
      for (int k = g * gs; k < (g + 1) * gs; ++k) {
        if (row[k] < mn) mn = row[k];
        if (row[k] > mx) mx = row[k];
      }
      float s = (mx - mn) / 15.0f;
      if (!(s > 1e-8f)) s = 1e-8f;
      scales_f16[(size_t)m * ng + g] = orc_f32_to_f16_rne(s);
      zeros_f16[(size_t)m * ng + g] = orc_f32_to_f16_rne(mn);
      for (int k = g * gs; k < (g + 1) * gs; k += 2) {
        float q0 = rintf((row[k] - mn) / s), q1 = rintf((row[k + 1] - mn) / s);
        q0 = q0 < 0.f ? 0.f : (q0 > 15.f ? 15.f : q0);
        q1 = q1 < 0.f ? 0.f : (q1 > 15.f ? 15.f : q1);
        prow[k / 2] = (uint8_t)((uint8_t)q0 | ((uint8_t)q1 << 4));
      }
    }
  }
}
