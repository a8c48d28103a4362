// route_dev.cuh — device code shared by the routing kernels (route.cu) and
// the fused single-token decode kernel (int4_gemm.cu): the router's dot
// product in the reference's FMA-chain order and the per-token top-k.
#pragma once
#include <cfloat>

#include "kernels.cuh"

namespace llmoc {

// One (token, expert) router logit by one warp, from bf16 rows: lane c runs
// the reference's FMA chain c (k = c mod 32, ascending; fp32 of the bf16
// values; src/hal/cpu_ops.cpp:57-86), and the chains are folded with shuffles
// in its tree order: a[i] = (c[i]+c[8+i]) + (c[16+i]+c[24+i]);
// b[i] = a[i] + a[4+i]; r = (b0+b1) + (b2+b3).  Requires H % 32 == 0 (no
// unfused tail).  Every lane returns r, non-finite -> 0.
__device__ __forceinline__ float router_dot_warp(const uint16_t* wrow, const uint16_t* xrow, int H, int lane) {
  float c = 0.f;
  for (int k = lane; k < H; k += 32) c = __fmaf_rn(bf16_bits_to_f32(xrow[k]), bf16_bits_to_f32(wrow[k]), c);
  const float c8 = __shfl_down_sync(0xffffffffu, c, 8), c16 = __shfl_down_sync(0xffffffffu, c, 16),
              c24 = __shfl_down_sync(0xffffffffu, c, 24);
  const float av = (c + c8) + (c16 + c24);                       // a[lane], lanes 0..7
  const float bv = av + __shfl_down_sync(0xffffffffu, av, 4);    // b[lane], lanes 0..3
  const float b1 = __shfl_down_sync(0xffffffffu, bv, 1), b2 = __shfl_down_sync(0xffffffffu, bv, 2),
              b3 = __shfl_down_sync(0xffffffffu, bv, 3);
  const float r = __shfl_sync(0xffffffffu, (bv + b1) + (b2 + b3), 0);
  return isfinite(r) ? r : 0.f;
}

// The sigmoid+bias router's score of a logit: 1 / (1 + exp(-l)) in double,
// rounded to fp32 (this router has no reference counterpart; the oracle
// specifies it so), part of the selection key.
__device__ __forceinline__ float sigmoid_ref(float l) { return (float)(1.0 / (1.0 + exp(-(double)l))); }

// Order-preserving map of a non-NaN float key to uint32 (larger key ->
// larger code; -0 is folded into +0 first, so equal keys get equal codes).
__device__ __forceinline__ uint32_t key_code(float v) {
  const uint32_t u = __float_as_uint(v + 0.f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Top-k of one token by one warp (E <= 32 * kTopkSlots).  Lane l holds the
// keys and values of experts l, l + 32, ... in registers; a round takes the
// warp's largest key (smaller id on ties) with two warp reductions, and the
// chosen ids and values stay in registers until the weights are written.
constexpr int kTopkSlots = 16;  // E <= 512
// KIND: 0 softmax router, 1 sigmoid+bias router, 2 the same with the scores
// precomputed in a.sig (a compile-time choice: the executed path carries no
// branches around the other kinds' code, whose fetch would cost a round trip
// each in a kernel whose code is not in cache).
template <int Q, int KIND>  // slots per lane: E <= 32 * Q
__device__ __forceinline__ void topk_token_q(const TopkArgs& a, int t, int lane) {
  const float* lg = a.logits + (size_t)t * (a.ld > 0 ? a.ld : a.E);
  float key[Q], val[Q];
  // every logit (and bias) of the lane first, so the loads are in flight
  // together rather than one round trip each behind the arithmetic
  float lv[Q], bv[Q];
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int e = lane + 32 * q;
    // sigmoid router with precomputed values: those instead of the logits
    lv[q] = e < a.E ? (KIND == 2 ? a.sig[(size_t)t * (a.ld > 0 ? a.ld : a.E) + e] : lg[e]) : 0.f;
    bv[q] = KIND != 0 && e < a.E ? a.bias[e] : 0.f;
  }
  if constexpr (KIND == 0) {
    // keys = logits; probabilities exp(l - max) (their rounding only reaches
    // the weights, which are compared with a tolerance, never the ids)
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int e = lane + 32 * q;
      key[q] = e < a.E ? lv[q] : -INFINITY;
      m = fmaxf(m, key[q]);
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
#pragma unroll
    for (int q = 0; q < Q; ++q) val[q] = lane + 32 * q < a.E ? expf(key[q] - m) : 0.f;
  } else {
    // s = sigmoid(l) in double rounded to fp32 (part of the selection key)
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int e = lane + 32 * q;
      if (e < a.E) {
        const float sg = KIND == 2 ? lv[q] : sigmoid_ref(lv[q]);
        val[q] = sg;
        const float kv = sg + bv[q];
        key[q] = kv == kv ? kv : -FLT_MAX;  // a NaN bias must still leave a valid id
      } else {
        val[q] = 0.f;
        key[q] = -INFINITY;
      }
    }
  }

  // k rounds of argmax over keys (ties -> smaller id); selected keys -> -inf.
  // Padding slots (e >= E) hold -inf with ids above every real id, so a tie at
  // -inf still resolves to a real expert.
  int my_id = 0;
  float my_val = 0.f;
  for (int j = 0; j < a.k; ++j) {
    uint32_t bc = key_code(key[0]);
    int bq = 0;
#pragma unroll
    for (int q = 1; q < Q; ++q) {
      const uint32_t c = key_code(key[q]);
      if (c > bc) {
        bc = c;
        bq = q;
      }
    }
    const uint32_t mc = __reduce_max_sync(0xffffffffu, bc);
    const int bi = (int)__reduce_min_sync(0xffffffffu, bc == mc ? (uint32_t)(lane + 32 * bq) : 0x7fffffffu);
    const int oq = bi >> 5, ol = bi & 31;
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < Q; ++q)
      if (q == oq) {
        v = val[q];
        if (lane == ol) key[q] = -INFINITY;
      }
    v = __shfl_sync(0xffffffffu, v, ol);
    if (lane == (j & 31)) {
      if (j < 32) {
        my_id = bi;
        my_val = v;
      }
    }
    if (j >= 32 && lane == (j & 31)) {  // k > 32: slots 32..63 go out now
      a.ids[(size_t)t * a.kk + j] = bi;
      if (a.ep_key) a.ep_key[(size_t)t * a.kk + j] = (bi % a.ep_world) * a.ep_e_loc + bi / a.ep_world;
      a.weights[(size_t)t * a.kk + j] = v;  // finished below
    }
  }

  // weights: lane l computes w[j] for j = l, l+32 (k <= 64); sums are warp
  // reductions in double (the reference sums sequentially in double; the two
  // agree except for double roundings far below fp32 resolution); the
  // divisions are fp32 by the sums rounded to fp32 (the reference divides in
  // double, then rounds: within about 3 fp32 roundings of it, where a double
  // division costs far more here)
  int* ids = a.ids + (size_t)t * a.kk;
  float* w = a.weights + (size_t)t * a.kk;
  float sel[2];
  sel[0] = my_val;
  sel[1] = lane + 32 < a.k ? w[lane + 32] : 0.f;
  __syncwarp();
  if (lane < a.k) {
    ids[lane] = my_id;
    if (a.ep_key) a.ep_key[(size_t)t * a.kk + lane] = (my_id % a.ep_world) * a.ep_e_loc + my_id / a.ep_world;
  }
  if constexpr (KIND == 0) {
    double s = 0.0;
#pragma unroll
    for (int q = 0; q < Q; ++q) s += (double)val[q];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float sf = (float)s;
    float p[2];
    double ws = 0.0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = lane + 32 * h;
      p[h] = j < a.k ? __fdiv_rn(sel[h], sf) : 0.f;  // the reference's fp32 prob
      ws += (double)p[h];
    }
    for (int o = 16; o; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
    if (ws < 1e-12) ws = 1.0;
    const float wsf = (float)ws;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (lane + 32 * h < a.k) w[lane + 32 * h] = __fdiv_rn(p[h], wsf);
  } else {
    double sv[2], ws = 0.0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = lane + 32 * h;
      sv[h] = j < a.k ? (double)sel[h] : 0.0;
      ws += sv[h];
    }
    for (int o = 16; o; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
    if (ws < 1e-20) ws = 1.0;
    const float wsf = (float)ws;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (lane + 32 * h < a.k) w[lane + 32 * h] = __fmul_rn(__fdiv_rn(sel[h], wsf), a.routed_scaling);
  }
  if (lane == 0 && (a.has_shared || a.shared_w)) {
    // the shared expert's weight: constant, or the reference's float sigmoid of
    // its gate row's logit (qwen3_6_moe_int4_model.cpp:29, :365-371)
    const float sw = a.shared_gate ? 1.f / (1.f + expf(-lg[a.E])) : a.shared_scale;
    if (a.has_shared) {
      ids[a.k] = a.E;
      w[a.k] = sw;
    }
    if (a.shared_w) a.shared_w[t] = sw;
  }
}

template <int KIND>
__device__ __forceinline__ void topk_token_k(const TopkArgs& a, int t, int lane) {
  if (a.E <= 128) topk_token_q<4, KIND>(a, t, lane);
  else if (a.E <= 256) topk_token_q<8, KIND>(a, t, lane);
  else if (a.E <= 384) topk_token_q<12, KIND>(a, t, lane);
  else topk_token_q<16, KIND>(a, t, lane);
}
__device__ __forceinline__ void topk_token(const TopkArgs& a, int t, int lane) {
  if (a.router == 0) topk_token_k<0>(a, t, lane);
  else if (a.sig) topk_token_k<2>(a, t, lane);
  else topk_token_k<1>(a, t, lane);
}

}  // namespace llmoc
