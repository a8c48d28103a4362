// route.cu — router GEMV, top-k selection and token->expert permutation.
//
// Router GEMV: logits[t,e] = W_r[e,:] . x[t,:] in exactly the fp32 order of
// the reference's AVX2 hal::gemm_bias_free (src/hal/cpu_ops.cpp:57-86): 32
// independent FMA chains, chain c covering k = c (mod 32) in increasing k,
// folded as a[i] = (c[i]+c[8+i]) + (c[16+i]+c[24+i]); b[i] = a[i]+a[4+i];
// r = (b0+b1) + (b2+b3); a K % 32 tail is added unfused; non-finite -> 0.
// Products of bf16 weights with bf16/fp32 activations are formed by fmaf,
// so the logits are bitwise equal to the reference's and the top-k ids are
// too.  Layout: 8 lanes own the 32 chains of one (token, expert) dot (4
// chains per lane, fed by 8-byte/16-byte vector loads); a warp holds 4 such
// groups; register blocking over TW tokens x EW experts per group.
//
// Top-k: one warp per token, k rounds of a warp argmax (largest key, ties
// to the smaller expert id).  Softmax weights follow
// src/model/qwen3_6_moe_int4_model.cpp:388-402 (exp of l - max rounded to
// fp32, probabilities normalised by a double sum in index order, weights
// renormalised by a double sum in selection order).  Sigmoid+bias: s =
// 1/(1+exp(-l)) in double rounded to fp32, selection on s + bias,
// weights s / sum(s_sel) * routed_scaling.
//
// Permutation: one CTA, deterministic: pairs p = t*kk + j sorted stably by
// expert (canonical order: expert, then t, then j), with per-expert offsets,
// the inverse map, and the list of work items (<= 32 pairs of one expert).
#include <cfloat>
#include <cstdlib>
#include <cstring>

#include <algorithm>

#include "kernels.cuh"
#include "route_dev.cuh"

namespace llmoc {

// ------------------------------------------------------------ router GEMV

template <typename XT>
struct XLoad4;
template <>
struct XLoad4<__nv_bfloat16> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float v[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xFFFF0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xFFFF0000u);
  }
};
template <>
struct XLoad4<float> {
  __device__ __forceinline__ static void load(const float* p, float v[4]) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    v[0] = u.x;
    v[1] = u.y;
    v[2] = u.z;
    v[3] = u.w;
  }
};

// grid.x covers groups of (TW tokens x EW experts); 8 lanes per group.
template <typename XT, int TW, int EW>
__global__ void __launch_bounds__(256) k_router_logits(const XT* __restrict__ X,
                                                       const uint16_t* __restrict__ Wr, int T,
                                                       int E, int H, float* __restrict__ logits) {
  grid_dep_wait();
  grid_dep_release();
  const int lane = threadIdx.x & 31;
  const int sub = lane & 7;  // owns chains 4*sub .. 4*sub+3
  const int group = (blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  const int n_et = (E + EW - 1) / EW;
  const int et = group % n_et;
  const int tt = group / n_et;
  const int t0 = tt * TW, e0 = et * EW;
  const bool live = t0 < T;  // whole 8-lane group agrees

  float acc[TW][EW][4];
#pragma unroll
  for (int a = 0; a < TW; ++a)
#pragma unroll
    for (int b = 0; b < EW; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  const XT* xr[TW];
  const uint16_t* wr[EW];
#pragma unroll
  for (int a = 0; a < TW; ++a) xr[a] = X + (size_t)min(t0 + a, T - 1) * H;
#pragma unroll
  for (int b = 0; b < EW; ++b) wr[b] = Wr + (size_t)min(e0 + b, E - 1) * H;

  const int K32 = live ? (H & ~31) : 0;
#pragma unroll 4
  for (int k = 4 * sub; k < K32; k += 32) {
    float xv[TW][4];
#pragma unroll
    for (int a = 0; a < TW; ++a) XLoad4<XT>::load(xr[a] + k, xv[a]);
#pragma unroll
    for (int b = 0; b < EW; ++b) {
      const uint2 u = *reinterpret_cast<const uint2*>(wr[b] + k);
      float wv[4];
      wv[0] = __uint_as_float(u.x << 16);
      wv[1] = __uint_as_float(u.x & 0xFFFF0000u);
      wv[2] = __uint_as_float(u.y << 16);
      wv[3] = __uint_as_float(u.y & 0xFFFF0000u);
#pragma unroll
      for (int a = 0; a < TW; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] = __fmaf_rn(xv[a][c], wv[c], acc[a][b][c]);
    }
  }

  // Fold: chain index ch = 4*sub + c.  a[i] = (c[i]+c[8+i]) + (c[16+i]+c[24+i])
  // chain i lives in lane sub = i/4 register i%4; chain 8+i in sub+2; 16+i in
  // sub+4; 24+i in sub+6.
#pragma unroll
  for (int a = 0; a < TW; ++a)
#pragma unroll
    for (int b = 0; b < EW; ++b) {
      float v[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float c8 = __shfl_down_sync(0xffffffffu, acc[a][b][c], 2, 8);
        const float c16 = __shfl_down_sync(0xffffffffu, acc[a][b][c], 4, 8);
        const float c24 = __shfl_down_sync(0xffffffffu, acc[a][b][c], 6, 8);
        v[c] = (acc[a][b][c] + c8) + (c16 + c24);  // valid in sub 0,1: a[4*sub + c]
      }
      // b[i] = a[i] + a[4+i]: a[i] in sub 0 reg i, a[4+i] in sub 1 reg i
      float bb[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) bb[c] = v[c] + __shfl_down_sync(0xffffffffu, v[c], 1, 8);
      float r = (bb[0] + bb[1]) + (bb[2] + bb[3]);
      if (sub == 0 && live && t0 + a < T && e0 + b < E) {
        const int t = t0 + a, e = e0 + b;
        for (int kk = K32; kk < H; ++kk) {
          const float prod =
              __fmul_rn(to_f32(X[(size_t)t * H + kk]), bf16_bits_to_f32(Wr[(size_t)e * H + kk]));
          r = __fadd_rn(r, prod);  // the reference leaves this tail unfused
        }
        logits[(size_t)t * E + e] = isfinite(r) ? r : 0.f;
      }
    }
}

// ----------------------------------------------- router GEMV, tiled (bf16 X)
//
// The same arithmetic as k_router_logits, laid out as an SGEMM whose 32 lanes
// are the 32 chains: lane c of a warp accumulates chain c (k = c mod 32, k
// ascending) of TT tokens x EE experts in registers, one fmaf per k and
// output, from fp32 copies of X and W_r staged through shared memory in
// 256-wide K chunks (double-buffered; the next chunk's global loads are in
// flight while the current one is multiplied).  After the K loop every lane
// writes its chain values to shared memory and each thread folds whole
// outputs in the reference's tree order.  A CTA of WT x WE warps covers
// TT*WT tokens x EE*WE experts.  Requires H % 256 == 0.
constexpr int kRouterKC = 256;

template <int TT, int EE, int WT, int WE>
struct RouterTile {
  static constexpr int kThreads = 32 * WT * WE;
  static constexpr int kRowsX = TT * WT, kRowsW = EE * WE, kRows = kRowsX + kRowsW;
  static constexpr int kChunks = kRows * (kRouterKC / 8);            // 8-element pieces per stage
  static constexpr int kPer = (kChunks + kThreads - 1) / kThreads;   // per thread
  static constexpr int kStage = kRows * kRouterKC;                   // floats per stage
  static constexpr int kOut = kRowsX * kRowsW;
  static constexpr size_t kSmem =
      (size_t)4 * (2 * kStage > kOut * 33 ? 2 * kStage : kOut * 33);  // stages, reused for the fold
};

// With xo.xh, the CTAs of the first expert tile also make their tokens' fp16
// rows for the decode gate/up GEMM (prep_xh_row's format): each warp first
// reads its token rows' largest exponent, then converts every staged chunk.
template <int TT, int EE, int WT, int WE>
__global__ void __launch_bounds__(RouterTile<TT, EE, WT, WE>::kThreads, 1)
    k_router_tiled(const __nv_bfloat16* __restrict__ X, const uint16_t* __restrict__ Wr, int T, int E, int H,
                   float* __restrict__ logits, XhOut xo) {
  using RT = RouterTile<TT, EE, WT, WE>;
  constexpr int kWarpsR = RT::kThreads / 32;
  constexpr int kXRowsPerWarp = (RT::kRowsX + kWarpsR - 1) / kWarpsR;
  extern __shared__ float rsm[];
  grid_dep_wait();
  grid_dep_release();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tg = warp % WT, eg = warp / WT;
  const int t0 = blockIdx.y * RT::kRowsX, e0 = blockIdx.x * RT::kRowsW;
  // fp16 rows: warp w owns token rows w, w + kWarpsR, ... of the tile
  const bool xh = xo.xh != nullptr && blockIdx.x == 0;
  float xdown[kXRowsPerWarp];
  if (xh) {
#pragma unroll
    for (int j = 0; j < kXRowsPerWarp; ++j) {
      const int row = warp + j * kWarpsR, t = t0 + row;
      uint32_t mexp = 0;
      if (row < RT::kRowsX && t < T) {
        const uint4* src = reinterpret_cast<const uint4*>(X + (size_t)t * H);
        for (int i0 = 0; i0 < H / 8; i0 += 8 * 32) {
          uint4 v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int i = i0 + lane + 32 * q;
            v[q] = i < H / 8 ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            mexp = bf16x2_max_exp(v[q].x, mexp);
            mexp = bf16x2_max_exp(v[q].y, mexp);
            mexp = bf16x2_max_exp(v[q].z, mexp);
            mexp = bf16x2_max_exp(v[q].w, mexp);
          }
        }
      }
      mexp = __reduce_max_sync(0xffffffffu, mexp);
      const int e = mexp == 0 ? 0 : max(-100, (int)mexp - 141);
      xdown[j] = __int_as_float((127 - e) << 23);
      if (lane == 0 && row < RT::kRowsX && t < T) xo.xscale[t] = __int_as_float((127 + e) << 23);
    }
  }
  // convert a parked stage's token rows (fp32 copies of the bf16 values): lane
  // L takes 8 consecutive values of each of the warp's rows
  auto emit_xh = [&](int s, int kc) {
#pragma unroll
    for (int j = 0; j < kXRowsPerWarp; ++j) {
      const int row = warp + j * kWarpsR, t = t0 + row;
      if (row >= RT::kRowsX) continue;  // uniform over the warp
      const float* xs = rsm + (size_t)s * RT::kStage + (size_t)row * kRouterKC + 8 * lane;
      uint32_t o[4];
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 h2 = __floats2half2_rn(xs[2 * q] * xdown[j], xs[2 * q + 1] * xdown[j]);
        const float2 f2 = __half22float2(h2);
        sum += f2.x;
        sum += f2.y;
        o[q] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      const int lpg = xo.gs / 8;
      for (int off = 1; off < lpg; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (t < T) {
        reinterpret_cast<uint4*>(xo.xh)[((size_t)t * H + kc + 8 * lane) / 8] = make_uint4(o[0], o[1], o[2], o[3]);
        if (lane % lpg == 0) xo.xsum[(size_t)t * (H / xo.gs) + (kc + 8 * lane) / xo.gs] = sum;
      }
    }
  };

  // staging piece q: row q / 32 (X rows first, then W_r rows), k offset 8 (q % 32)
  const uint4* src[RT::kPer];
  bool live[RT::kPer];
#pragma unroll
  for (int p = 0; p < RT::kPer; ++p) {
    const int q = threadIdx.x + p * RT::kThreads;
    live[p] = q < RT::kChunks;
    const int row = live[p] ? q / 32 : 0, k8 = q % 32;
    const uint16_t* base = row < RT::kRowsX
                               ? reinterpret_cast<const uint16_t*>(X) + (size_t)min(t0 + row, T - 1) * H
                               : Wr + (size_t)min(e0 + row - RT::kRowsX, E - 1) * H;
    src[p] = reinterpret_cast<const uint4*>(base + 8 * k8);
  }
  uint4 stg[RT::kPer];
  auto fetch = [&](int kc) {
#pragma unroll
    for (int p = 0; p < RT::kPer; ++p)
      if (live[p]) stg[p] = __ldg(src[p] + kc / 8);
  };
  auto park = [&](int s) {  // staged bf16 -> fp32 in stage s
#pragma unroll
    for (int p = 0; p < RT::kPer; ++p) {
      if (!live[p]) continue;
      const int q = threadIdx.x + p * RT::kThreads;
      float4* d = reinterpret_cast<float4*>(rsm + (size_t)s * RT::kStage + (q / 32) * kRouterKC + 8 * (q % 32));
      const uint4 u = stg[p];
      d[0] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                         __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
      d[1] = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xFFFF0000u),
                         __uint_as_float(u.w << 16), __uint_as_float(u.w & 0xFFFF0000u));
    }
  };

  float acc[TT][EE];
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < EE; ++b) acc[a][b] = 0.f;

  fetch(0);
  park(0);
  __syncthreads();
  const int nk = H / kRouterKC;
  for (int c = 0; c < nk; ++c) {
    const int s = c & 1;
    if (c + 1 < nk) fetch((c + 1) * kRouterKC);
    if (xh) emit_xh(s, c * kRouterKC);
    const float* xs = rsm + (size_t)s * RT::kStage + (tg * TT) * kRouterKC + lane;
    const float* ws = rsm + (size_t)s * RT::kStage + (RT::kRowsX + eg * EE) * kRouterKC + lane;
#pragma unroll 2
    for (int i = 0; i < kRouterKC / 32; ++i) {
      float xv[TT], wv[EE];
#pragma unroll
      for (int a = 0; a < TT; ++a) xv[a] = xs[a * kRouterKC + 32 * i];
#pragma unroll
      for (int b = 0; b < EE; ++b) wv[b] = ws[b * kRouterKC + 32 * i];
#pragma unroll
      for (int a = 0; a < TT; ++a)
#pragma unroll
        for (int b = 0; b < EE; ++b) acc[a][b] = __fmaf_rn(xv[a], wv[b], acc[a][b]);
    }
    if (c + 1 < nk) park(s ^ 1);
    __syncthreads();
  }

  // chain values -> shared memory [output][chain] (33-float rows), then fold
  // one output per thread: a[i] = (c[i]+c[8+i]) + (c[16+i]+c[24+i]);
  // b[i] = a[i] + a[4+i]; r = (b0+b1) + (b2+b3)
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < EE; ++b) {
      const int o = (tg * TT + a) * RT::kRowsW + eg * EE + b;
      rsm[o * 33 + lane] = acc[a][b];
    }
  __syncthreads();
  for (int o = threadIdx.x; o < RT::kOut; o += RT::kThreads) {
    const int t = t0 + o / RT::kRowsW, e = e0 + o % RT::kRowsW;
    if (t >= T || e >= E) continue;
    const float* ch = rsm + o * 33;
    float av[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) av[i] = (ch[i] + ch[8 + i]) + (ch[16 + i] + ch[24 + i]);
    float bv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) bv[i] = av[i] + av[4 + i];
    const float r = (bv[0] + bv[1]) + (bv[2] + bv[3]);
    logits[(size_t)t * E + e] = isfinite(r) ? r : 0.f;
  }
}

// ------------------------------------------- router GEMV, decode (T <= 8)
//
// Decode batches read the whole router matrix for a handful of tokens, so the
// work is one pass over W_r spread over as many SMs as possible.  A CTA takes
// EPC expert rows and every token: it copies those rows and the T token rows
// (bf16) into shared memory with one 16-byte load per thread and piece, then
// each (token, expert) dot is one warp whose lane c runs the reference's FMA
// chain c (k = c mod 32, ascending; fp32 of the bf16 values), and the chains
// are folded with shuffles in the reference's tree order:
// a[i] = (c[i]+c[8+i]) + (c[16+i]+c[24+i]); b[i] = a[i] + a[4+i];
// r = (b0+b1) + (b2+b3).  Requires H % 256 == 0 (no unfused tail).
constexpr int kRouterSmallThreads = 256;
// With xo.xh, CTA t < T also makes token t's fp16 row from its shared copy.
template <int EPC>
__global__ void __launch_bounds__(kRouterSmallThreads) k_router_small(const __nv_bfloat16* __restrict__ X,
                                                                      const uint16_t* __restrict__ Wr, int T,
                                                                      int E, int H, float* __restrict__ logits,
                                                                      XhOut xo) {
  extern __shared__ __align__(16) uint16_t rsm16[];  // [EPC + T][H] bf16
  grid_dep_wait();
  grid_dep_release();
  const int e0 = blockIdx.x * EPC;
  const int nw = min(EPC, E - e0);
  const int n8 = H / 8;
  // W_r rows e0 .. e0 + nw - 1, then the T token rows: eight 16-byte pieces
  // per thread requested at once
  const int total = (nw + T) * n8;
  for (int q0 = 0; q0 < total; q0 += 8 * kRouterSmallThreads) {
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int q = q0 + threadIdx.x + j * kRouterSmallThreads;
      if (q < total) {
        const int row = q / n8, c = q % n8;
        const uint16_t* src = row < nw ? Wr + (size_t)(e0 + row) * H
                                       : reinterpret_cast<const uint16_t*>(X) + (size_t)(row - nw) * H;
        v[j] = __ldg(reinterpret_cast<const uint4*>(src) + c);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int q = q0 + threadIdx.x + j * kRouterSmallThreads;
      if (q < total) reinterpret_cast<uint4*>(rsm16)[q] = v[j];
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int pr = warp; pr < nw * T; pr += kRouterSmallThreads / 32) {
    const int e = pr % nw, t = pr / nw;
    const float r = router_dot_warp(rsm16 + (size_t)e * H, rsm16 + (size_t)(nw + t) * H, H, lane);
    if (lane == 0) logits[(size_t)t * E + e0 + e] = r;
  }
  if (xo.xh && (int)blockIdx.x < T && warp == kRouterSmallThreads / 32 - 1)
    prep_xh_row<4, false>(reinterpret_cast<const uint4*>(rsm16 + (size_t)(nw + blockIdx.x) * H), blockIdx.x, H,
                          xo.gs, static_cast<uint4*>(xo.xh), xo.xsum, xo.xscale, lane);
}

template <int EPC>
static cudaError_t launch_router_small(const __nv_bfloat16* X, const uint16_t* Wr, int T, int E, int H, float* logits,
                                       cudaStream_t st, const XhOut& xo) {
  const size_t smem = (size_t)(EPC + T) * H * 2;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(k_router_small<EPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  if ((E + EPC - 1) / EPC < T && xo.xh) return cudaErrorInvalidValue;  // a CTA per token row
  return launch_pdl(k_router_small<EPC>, dim3((E + EPC - 1) / EPC), dim3(kRouterSmallThreads), smem, st, X, Wr, T,
                    E, H, logits, xo);
}

static long router_sm_count() {
  static long n[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

template <int TT, int EE, int WT, int WE>
static cudaError_t launch_router_tiled(const __nv_bfloat16* X, const uint16_t* Wr, int T, int E, int H,
                                       float* logits, cudaStream_t st, const XhOut& xo = XhOut{}) {
  using RT = RouterTile<TT, EE, WT, WE>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_router_tiled<TT, EE, WT, WE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)RT::kSmem);
    attr = true;
  }
  const dim3 grid((E + RT::kRowsW - 1) / RT::kRowsW, (T + RT::kRowsX - 1) / RT::kRowsX);
  return launch_pdl(k_router_tiled<TT, EE, WT, WE>, grid, dim3(RT::kThreads), RT::kSmem, st, X, Wr, T, E, H, logits,
                    xo);
}

// --------------------------------------------------------------- top-k


// (key_code, topk_token_q and topk_token: route_dev.cuh)


// One warp per token.
__global__ void __launch_bounds__(256) k_topk(TopkArgs a) {
  grid_dep_wait();
  grid_dep_release();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= a.T) return;
  topk_token(a, t, lane);
  if (a.xh)
    prep_xh_row<16, true>(static_cast<const uint4*>(a.x) + (size_t)t * (a.H / 8), t, a.H, a.gs,
                          static_cast<uint4*>(a.xh), a.xsum, a.xscale, lane);
}

// ----------------------------------------------------------- permutation

// One CTA of kPermThreads threads.  The pairs are counted and placed in NW
// ranges, one per warp 0..NW-1 (NW <= kPermWarps: fewer ranges make the
// per-expert loops and the counters NW long, which pays when there are few
// pairs; the result is the same, pairs of an expert in ascending order).
// cnt: NW x n_exp ints of shared memory (counts, then running positions).
template <int NW>
__device__ __forceinline__ void permute_block(const PermArgs& a, int* cnt) {
  static_assert(NW >= 1 && NW <= kPermWarps, "counting ranges");
  flag_wait_block(a.wait);  // the transport's sources (their counts and rows) first
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < NW * a.n_exp; i += kPermThreads) cnt[i] = 0;
  // Index space walked: 0..nv-1.  Plain input: the slots themselves.
  // Segmented input: the occupied slots of each segment, segment after
  // segment (slot order), v -> slot via the segments' exclusive offsets.
  __shared__ int seg_off[kEpMaxWorld + 1];
  const bool segd = a.seg_len > 0;
  if (segd && threadIdx.x == 0) {
    int o = 0;
    for (int s = 0; s < a.n_seg; ++s) {
      seg_off[s] = o;
      o += min(max(a.seg_count[(size_t)s * a.seg_stride], 0), a.seg_len);
    }
    seg_off[a.n_seg] = o;
  }
  __syncthreads();
  const int nv = segd ? seg_off[a.n_seg] : a.n;
  auto slot_of = [&](int v) {
    if (!segd) return v;
    int s = 0;
    while (v >= seg_off[s + 1]) ++s;
    return s * a.seg_len + (v - seg_off[s]);
  };

  const int per = (nv + NW - 1) / NW;
  const int lo = min(nv, warp * per), hi = min(nv, lo + per);  // empty for warps >= NW
  // ids outside [0, n_exp) are empty slots (the padded receive layout of the
  // NVLink expert-parallel transport): not counted, not placed, inverse -1
  for (int v = lo + lane; v < hi; v += 32) {
    const int ex = a.ids[slot_of(v)];
    if ((unsigned)ex < (unsigned)a.n_exp) atomicAdd(&cnt[warp * a.n_exp + ex], 1);
  }
  __syncthreads();

  // per expert totals -> exclusive scans (pairs and work chunks); thread e
  // handles expert e (n_exp <= 512 < 1024 threads).
  const int e = threadIdx.x;
  int tot = 0;
  if (e < a.n_exp)
    for (int w = 0; w < NW; ++w) tot += cnt[w * a.n_exp + e];
  const int chunks = (tot + a.chunk - 1) / a.chunk;
  // block exclusive scan of (tot, chunks, active) packed: do two scans
  int v1 = tot, v2 = chunks, v3 = tot > 0;
  for (int o = 1; o < 32; o <<= 1) {
    const int a1 = __shfl_up_sync(0xffffffffu, v1, o);
    const int a2 = __shfl_up_sync(0xffffffffu, v2, o);
    const int a3 = __shfl_up_sync(0xffffffffu, v3, o);
    if (lane >= o) {
      v1 += a1;
      v2 += a2;
      v3 += a3;
    }
  }
  __shared__ int w1[kPermWarps], w2[kPermWarps], w3[kPermWarps];
  if (lane == 31) {
    w1[warp] = v1;
    w2[warp] = v2;
    w3[warp] = v3;
  }
  __syncthreads();
  if (warp == 0) {
    int x1 = w1[lane], x2 = w2[lane], x3 = w3[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int a1 = __shfl_up_sync(0xffffffffu, x1, o);
      const int a2 = __shfl_up_sync(0xffffffffu, x2, o);
      const int a3 = __shfl_up_sync(0xffffffffu, x3, o);
      if (lane >= o) {
        x1 += a1;
        x2 += a2;
        x3 += a3;
      }
    }
    w1[lane] = x1;
    w2[lane] = x2;
    w3[lane] = x3;
  }
  __syncthreads();
  const int base1 = (warp ? w1[warp - 1] : 0) + v1 - tot;     // exclusive pair offset
  const int base2 = (warp ? w2[warp - 1] : 0) + v2 - chunks;  // exclusive chunk offset
  if (e < a.n_exp) {
    a.offsets[e] = base1;
    int run = base1;
    for (int w = 0; w < NW; ++w) {
      const int c = cnt[w * a.n_exp + e];
      cnt[w * a.n_exp + e] = run;
      run += c;
    }
    for (int c = 0; c < chunks; ++c) {
      WorkItem it;
      it.expert = e;
      it.row0 = base1 + c * a.chunk;
      it.nrows = min(a.chunk, tot - c * a.chunk);
      it.pad = 0;
      a.work[base2 + c] = it;
    }
  }
  if (threadIdx.x == kPermThreads - 1) {
    if (a.err)
      for (int i = 0; i <= kGemmCounters; ++i) a.err[i] = 0;
    a.offsets[a.n_exp] = w1[kPermWarps - 1];
    *a.n_work = w2[kPermWarps - 1];
    *a.n_active = w3[kPermWarps - 1];
  }
  __syncthreads();

  // placement: each warp walks its own range in order, 32 pairs at a time.
  for (int b = lo; b < hi; b += 32) {
    const int v = b + lane;
    const int i = v < hi ? slot_of(v) : 0;
    const int ex = v < hi ? a.ids[i] : -1;
    const bool ok = (unsigned)ex < (unsigned)a.n_exp;
    if (v < hi && !ok) a.inverse[i] = -1;
    const unsigned act = __ballot_sync(0xffffffffu, ok);
    if (ok) {
      const unsigned peers = __match_any_sync(act, ex);
      const int rank = __popc(peers & lanemask_lt());
      const int pos = cnt[warp * a.n_exp + ex] + rank;
      a.sorted[pos] = i;
      a.inverse[i] = pos;
      __syncwarp(act);
      if (rank == 0) cnt[warp * a.n_exp + ex] += __popc(peers);
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kPermThreads) k_permute(PermArgs a, EpRouteArgs ea) {
  extern __shared__ int psm[];
  grid_dep_wait();
  grid_dep_release();
  permute_block<kPermWarps>(a, psm);
  if (ea.key) {  // expert-parallel source: per-owner counts and owner-local experts in key order
    __syncthreads();  // offsets and sorted complete
    for (int r = threadIdx.x; r < ea.world; r += kPermThreads)
      ea.counts[r] = a.offsets[(r + 1) * ea.e_loc] - a.offsets[r * ea.e_loc];
    for (int q = threadIdx.x; q < a.n; q += kPermThreads) ea.send_expert[q] = ea.key[a.sorted[q]] % ea.e_loc;
  }
}

// Decode-size batches: top-k of every token (warp w takes tokens w, w + 32,
// ...) and the permutation in one CTA, saving a launch and a pass over the
// ids.  Shared memory: kFusedPermRanges x n_exp ints (the permutation's
// counts: at most kFusedRouteMaxT * 65 pairs, counted in 4 ranges).
// Expert-parallel dispatch (ea.key != null): the permutation runs over the
// owner keys (e % world) * e_loc + e / world of the ids, and the per-owner
// counts and owner-local expert of each pair in key order follow (for larger
// T, k_topk writes the keys and k_permute adds the same tail).
constexpr int kFusedPermRanges = 4;
__global__ void __launch_bounds__(kPermThreads) k_topk_permute(TopkArgs ta, PermArgs pa, EpRouteArgs ea) {
  extern __shared__ int fsm[];
  grid_dep_wait();
  grid_dep_release();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < ta.T; t += kPermWarps) topk_token(ta, t, lane);
  __syncthreads();  // the ids written above are visible to the whole CTA
  if (ea.key) {
    for (int p = threadIdx.x; p < pa.n; p += kPermThreads) {
      const int e = ta.ids[p];
      ea.key[p] = (e % ea.world) * ea.e_loc + e / ea.world;
    }
    __syncthreads();
  }
  permute_block<kFusedPermRanges>(pa, fsm);
  if (ea.key) {
    __syncthreads();  // offsets and sorted complete
    for (int r = threadIdx.x; r < ea.world; r += kPermThreads)
      ea.counts[r] = pa.offsets[(r + 1) * ea.e_loc] - pa.offsets[r * ea.e_loc];
    for (int q = threadIdx.x; q < pa.n; q += kPermThreads) ea.send_expert[q] = ea.key[pa.sorted[q]] % ea.e_loc;
  }
  // the decode gate/up GEMM's fp16 rows (after the permutation, whose
  // registers are dead by now)
  if (ta.xh)
    for (int t = warp; t < ta.T; t += kPermWarps)
      prep_xh_row<4, true>(static_cast<const uint4*>(ta.x) + (size_t)t * (ta.H / 8), t, ta.H, ta.gs,
                           static_cast<uint4*>(ta.xh), ta.xsum, ta.xscale, lane);
}

// ---------------------------------------------------------------- launch

cudaError_t launch_router_logits(const void* X, bool x_is_f32, const uint16_t* Wr, int T, int E,
                                 int H, float* logits, cudaStream_t st, const XhOut& xo) {
  if (T <= 0) return cudaSuccess;
  // bf16 activations with H % 256 == 0 (every BASELINE shape): the tiled
  // kernel, its tile chosen by T; the lane-group kernel below (same
  // arithmetic) otherwise
  if (!x_is_f32 && H % kRouterKC == 0) {
    const auto* Xb = static_cast<const __nv_bfloat16*>(X);
    // decode: one or two expert rows per CTA (>= 128 CTAs for the BASELINE layers' E >= 128)
    if (T <= kRouterSmallMaxT) return E >= 256 ? launch_router_small<2>(Xb, Wr, T, E, H, logits, st, xo)
                                               : launch_router_small<1>(Xb, Wr, T, E, H, logits, st, xo);
    if (T < 128) return launch_router_tiled<8, 2, 1, 8>(Xb, Wr, T, E, H, logits, st, xo);  // 8 t x 16 e
    // the largest tile whose grid still keeps the SMs busy: 32 x 32 (half a
    // wave or more: at T = 1024, E = 128 its 128 CTAs beat 512 of 16 x 16),
    // else 16 x 16 (one wave), else 8 x 16 (at T = 512, E = 128 the 32 x 32
    // grid is 64 CTAs; 16 x 16 took it from 27 to 21 us)
    const long sms = router_sm_count();
    const auto ctas = [&](int rt, int re) { return (long)((T + rt - 1) / rt) * ((E + re - 1) / re); };
    if (2 * ctas(32, 32) >= sms) return launch_router_tiled<8, 16, 4, 2>(Xb, Wr, T, E, H, logits, st);  // 32 t x 32 e
    if (ctas(16, 16) >= sms) return launch_router_tiled<8, 4, 2, 4>(Xb, Wr, T, E, H, logits, st);       // 16 t x 16 e
    return launch_router_tiled<8, 2, 1, 8>(Xb, Wr, T, E, H, logits, st);                                 // 8 t x 16 e
  }
  const int threads = 256;
  if (T <= 64) {
    const long groups = (long)T * E;
    const int blocks = (int)((groups * 8 + threads - 1) / threads);
    if (x_is_f32)
      return launch_pdl(k_router_logits<float, 1, 1>, dim3(blocks), dim3(threads), 0, st, (const float*)X, Wr, T, E, H, logits);
    else
      return launch_pdl(k_router_logits<__nv_bfloat16, 1, 1>, dim3(blocks), dim3(threads), 0, st, (const __nv_bfloat16*)X, Wr, T, E, H, logits);
  } else if (T <= 256) {
    constexpr int TW = 2, EW = 2;
    const long groups = (long)((T + TW - 1) / TW) * ((E + EW - 1) / EW);
    const int blocks = (int)((groups * 8 + threads - 1) / threads);
    if (x_is_f32)
      return launch_pdl(k_router_logits<float, TW, EW>, dim3(blocks), dim3(threads), 0, st, (const float*)X, Wr, T, E, H, logits);
    else
      return launch_pdl(k_router_logits<__nv_bfloat16, TW, EW>, dim3(blocks), dim3(threads), 0, st, (const __nv_bfloat16*)X, Wr, T, E, H, logits);
  } else {
    constexpr int TW = 4, EW = 4;
    const long groups = (long)((T + TW - 1) / TW) * ((E + EW - 1) / EW);
    const int blocks = (int)((groups * 8 + threads - 1) / threads);
    if (x_is_f32)
      return launch_pdl(k_router_logits<float, TW, EW>, dim3(blocks), dim3(threads), 0, st, (const float*)X, Wr, T, E, H, logits);
    else
      return launch_pdl(k_router_logits<__nv_bfloat16, TW, EW>, dim3(blocks), dim3(threads), 0, st, (const __nv_bfloat16*)X, Wr, T, E, H, logits);
  }
  return cudaGetLastError();
}

cudaError_t launch_topk(const TopkArgs& a, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  if (a.E > 32 * kTopkSlots || a.k > 64) return cudaErrorInvalidValue;
  return launch_pdl(k_topk, dim3((a.T + 7) / 8), dim3(256), 0, st, a);
}

cudaError_t launch_topk_permute(const TopkArgs& ta, const PermArgs& pa, cudaStream_t st, const EpRouteArgs& ea) {
  if (ta.E > 32 * kTopkSlots || ta.k > 64) return cudaErrorInvalidValue;
  const size_t smem = (size_t)kFusedPermRanges * pa.n_exp * sizeof(int);
  cudaError_t e = cudaFuncSetAttribute(k_topk_permute, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_topk_permute, dim3(1), dim3(kPermThreads), smem, st, ta, pa, ea);
}

cudaError_t launch_permute_ep(const PermArgs& a, const EpRouteArgs& ea, cudaStream_t st) {
  const size_t smem = (size_t)kPermWarps * a.n_exp * sizeof(int);
  cudaError_t e = cudaFuncSetAttribute(k_permute, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_permute, dim3(1), dim3(kPermThreads), smem, st, a, ea);
}
cudaError_t launch_permute(const PermArgs& a, cudaStream_t st) { return launch_permute_ep(a, EpRouteArgs{}, st); }

// ------------------------------------------------------ expert parallelism
// Expert e is owned by rank e % world and is local expert e / world there (the
// reference's DeviceMesh::owner_rank with EpShard::kMod).  Sorting the routed
// pairs by key = owner * e_loc + local id groups them by destination rank, in
// the owner's local expert order.

__global__ void k_fill_i32(int* __restrict__ p, int n, int v) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

cudaError_t launch_fill_i32(int* p, int n, int v, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_fill_i32<<<std::min((n + 255) / 256, 1184), 256, 0, st>>>(p, n, v);
  return cudaGetLastError();
}

}  // namespace llmoc
