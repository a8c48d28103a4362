// int4_gemm.cu — INT4 weight-only grouped GEMM kernels and their helpers.
//
//  k_repack            QLWC layout (src/weights/qlwc_format.h) -> fragment order
//  k_dequant           fragment order -> fp32 W[M,K] (bit-exact with
//                      hal::dequant_int4_row, src/hal/int4_ops.cpp:640-662)
//  k_int4_mma          tensor-core grouped dequant-GEMM for AWQ-sym weights
//                      and bf16 activations (decode and small groups)
//  k_int4_cc           CUDA-core fp32 grouped GEMV for any scheme and fp32 or
//                      bf16 activations (GPTQ-asym, the host-fp32 API)
//  k_combine           y[t] = sum_j w[t,j] * d[t,j] (+ shared), fixed j order
//  k_quant_awq_sym     tools/quantize_int4.py:150-166 on the device
//
// Both GEMM kernels walk a device-built work list (expert, first row of the
// expert-sorted pair list, <= 32 rows) and read one weight row-tile per warp,
// so every selected expert's weights stream from HBM once per 32 of its
// tokens.  The per-group structure of the reference (dot of x with (q - zp)
// per group, times the group scale, accumulated in fp32; int4_ops.cpp:228)
// is kept: the tensor core multiplies exact bf16 integers (q - zp) by bf16
// activations, and the fp32 group partials are scaled on the accumulator.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "kernels.cuh"
#include "route_dev.cuh"

namespace llmoc {

// ------------------------------------------------------------------ repack

__device__ __forceinline__ uint32_t src_nib(const RepackArgs& a, int r, int k) {
  if (r >= a.M || k >= a.K) return 0u;
  const uint8_t b = a.q[(size_t)r * ((a.K + 1) / 2) + (k >> 1)];
  return (k & 1) ? (b >> 4) : (b & 0xFu);
}

__global__ void k_repack(RepackArgs a) {
  const int Mt = (a.M + 15) / 16;
  const size_t n_words = (size_t)Mt * a.Kc * 128;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_words;
       i += (size_t)gridDim.x * blockDim.x) {
    const int wd = (int)(i & 3);
    const int lane = piece_slot((int)((i >> 2) & 31));  // lane whose piece is stored here
    const size_t tc = i >> 7;  // rt * Kc + c
    const int c = (int)(tc % a.Kc);
    const int rt = (int)(tc / a.Kc);
    const int g = lane >> 2, t = lane & 3, kb = wd >> 1, kt = wd & 1;
    const int r0 = rt * 16 + g, r1 = r0 + 8;
    const int k = c * 64 + kb * 32 + t * 8 + kt * 4;
    // nibble slot = (i&1)*4 + (i>>1)*2 + (row g+8 ? 1 : 0)
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int slot = (e & 1) * 4 + (e >> 1) * 2;
      w |= src_nib(a, r0, k + e) << (4 * slot);
      w |= src_nib(a, r1, k + e) << (4 * (slot + 1));
    }
    a.qo[i] = w;
  }
  const size_t n_sc = (size_t)Mt * a.ng * 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_sc;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i & 15);
    const size_t tg = i >> 4;
    const int grp = (int)(tg % a.ng);
    const int rt = (int)(tg / a.ng);
    const int row = rt * 16 + r;
    const bool ok = row < a.M;
    a.so[i] = ok ? a.s[(size_t)row * a.ng + grp] : (uint16_t)0;
    if (a.zo) a.zo[i] = (ok && a.z) ? a.z[(size_t)row * a.ng + grp] : (uint16_t)0;
  }
}

// ----------------------------------------------------------------- dequant

// out[M,K] fp32 = (q - zp) * s (AWQ) or q * s + z (GPTQ), read from the
// fragment-order copy (proves the repack and the kernels' indexing).
__global__ void k_dequant(ProjDev P, int M, int K, int gs, int ng, int Kc, int awq, int zp,
                          float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)M * K;
       i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / K), k = (int)(i % K);
    const int rt = m >> 4, r = m & 15, g = r & 7, hi = r >> 3;
    const int c = k >> 6, kb = (k >> 5) & 1, t = (k >> 3) & 3, kt = (k >> 2) & 1, e = k & 3;
    const int slot32 = piece_slot(g * 4 + t);
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(P.q);
    const uint32_t w = q32[(((size_t)rt * Kc + c) * 32 + slot32) * 4 + kb * 2 + kt];
    const int slot = (e & 1) * 4 + (e >> 1) * 2 + hi;
    const int q = (w >> (4 * slot)) & 0xF;
    const int grp = k / gs;
    const float s = __half2float(P.s[((size_t)rt * ng + grp) * 16 + r]);
    if (awq) {
      out[i] = __fmul_rn((float)(q - zp), s);
    } else {
      const float z = P.z ? __half2float(P.z[((size_t)rt * ng + grp) * 16 + r]) : 0.f;
      out[i] = __fmaf_rn((float)q, s, z);  // q*s is exact, so this equals q*s + z
    }
  }
}

// ---------------------------------------------------- tensor-core grouped GEMM

__device__ __forceinline__ const ProjDev& pick(const ExpertDev& e, int p) {
  return p == 0 ? e.gate : (p == 1 ? e.up : e.down);
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// d = a * b (a fresh accumulator: no zeroing of d beforehand)
__device__ __forceinline__ void mma_bf16_z(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}
__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 forms of the two MMAs (the decode gate/up GEMM's fp16 activation path)
__device__ __forceinline__ void mma_f16_z(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}
__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.f + expf(-g))) * u; }

constexpr int kWarps = 4;  // warps per CTA of the grouped GEMM kernels

// Raw fragment word -> four A registers holding bf16 (128 + q) pairs: one
// lop3 per register (the zero point is removed after the MMA, below).
__device__ __forceinline__ void raw_word(uint32_t w, uint32_t a[4]) {
  a[0] = lop3_and_or(w, 0x000F000Fu, 0x43004300u);
  a[1] = lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u);
  a[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u);
  a[3] = lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u);
}
// The same word -> four A registers as fp16 pairs with one shift: an fp16
// mantissa has room for a nibble at bits 0-3 (1024 + q) and one at bits 4-7
// (1024 + 16 q), so registers 0 and 2 (row g) hold 1024 + q and registers 1
// and 3 (row g + 8) hold 1024 + 16 q.  After the MMA, row g's sum is
// P = 1024 sum(x) + sum(q x) and row g+8's is 1024 sum(x) + 16 sum(q x).
__device__ __forceinline__ void raw_word_f16(uint32_t w, uint32_t a[4]) {
  const uint32_t w8 = w >> 8;
  a[0] = lop3_and_or(w, 0x000F000Fu, 0x64006400u);
  a[1] = lop3_and_or(w, 0x00F000F0u, 0x64006400u);
  a[2] = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);
  a[3] = lop3_and_or(w8, 0x00F000F0u, 0x64006400u);
}

// Grouped INT4 GEMM on the tensor cores.  A warp owns one 16-row tile (both
// projections when NP = 2) of one work item; the ks warps of a CTA that
// share the tile split K into contiguous slices of 128-wide steps (K % 128 ==
// 0, group size 32/64/128, so every group end sits at a fixed place of a
// step).  Memory: each lane runs a private kStagesW-deep pipeline in shared
// memory — cp.async (16 B, L1 bypass) of its own fragment words and its own
// activation bytes for step i + kStagesW - 1 while it computes step i — so
// the bytes in flight do not cost registers and no barrier is needed (a lane
// only reads what it copied; the group scales, shared by the warp, are the
// one item read across lanes, after a __syncwarp).
// The MMA consumes the biased integers (128 + q), exact in bf16, and one
// extra MMA per k16 against an all-ones A fragment gives xs = sum_k x per
// token (shared by both projections).  Per group the fp32 partials become
//     AWQ:  s * (P - (128 + zp) * xs)        GPTQ: s * (P - 128 * xs) + z * xs
// i.e. the reference's  sum_k x * (q - zp) * s  and  sum_k x * (q * s + z).
// K slices meet in shared memory and are summed in warp order.
// grid.x = ceil(Mt * ks / 4), grid.y = work-list bound.
constexpr int kStagesW = 3;

template <int NP, int NT, bool AWQ, bool XH = false, bool ONE = false>
struct WStage {  // bytes of one stage of one warp (ONE: the activations of one row only)
  static constexpr int kW = NP * 1024;         // 2 chunks x 512 B per projection
  static constexpr int kS = NP * 128;          // scales of the step's groups (<= 4 x 32 B)
  static constexpr int kZ = AWQ ? 0 : NP * 128;  // zeros (GPTQ)
  static constexpr int kB = ONE ? 4 * 64 : NT * 4 * 512;  // 4 blocks x 16 B per lane per N-tile (ONE: per t)
  static constexpr int kX = XH ? 128 : 0;      // fp16 path: the 8 columns' group sums (16 B each)
  static constexpr int kBytes = kW + kS + kZ + kB + kX;
  // the K-slice reduction reuses the warp's own stages once they are drained
  static_assert(ONE || kStagesW * kBytes >= NP * NT * 4 * 32 * 4, "reduction slot");
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
// The same with an L2 cache policy (evict_first for weights streamed once per
// forward: they leave the code, the router rows and the activations in L2).
__device__ __forceinline__ void cp_async16_pol(void* dst, const void* src, unsigned long long pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ unsigned long long l2_evict_first() {
  unsigned long long pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// 4 * NG bytes (4, 8 or 16; source aligned to that size) through L1
template <int NG>
__device__ __forceinline__ void cp_async_small(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "n"(4 * NG)
               : "memory");
}

// Correction of one fp32 group partial P of the fp16 path into sum x (q - zp)
// (AWQ; bias = zp) or sum x q (GPTQ; bias = 0): rows g (hi = 0) hold
// 1024 sum x + sum q x, rows g + 8 (hi = 1) 1024 sum x + 16 sum q x.
__device__ __forceinline__ float f16_group(float P, float xs, int hi, float bias) {
  return hi ? __fmaf_rn(-(64.f + bias), xs, P * 0.0625f) : __fmaf_rn(-(1024.f + bias), xs, P);
}

// XH: the fp16 activation path of k_int4_mma_p (gate/up only, NT = 1).
// One CTA's share of k_int4_mma: row-tile block bx (kWarps / ks tiles) of the
// work items by, by + gy, ...; wsm = the CTA's kWarps stage rings.  Also the
// GEMM phases of the fused single-token kernel (k_moe_decode1), which walks a
// virtual grid of such blocks.  ONECOL: items of one row, so only the C
// fragment's column 2t (accumulators r = 0, 2; column 0 in lanes t = 0) is ever
// stored and the group ends skip the others.
template <int MODE, int NT, int GSB, bool AWQ, bool XH, bool ONECOL = false, int STG = kStagesW>
__device__ __forceinline__ void mma_kblock(const GemmArgs& a, int ks, int bx, int by, int gy,
                                           unsigned char* wsm) {
  constexpr int NP = MODE == MODE_GATE_UP ? 2 : 1;
  constexpr int NG = GSB == 4 ? 1 : (GSB == 2 ? 2 : 4);  // groups per step
  static_assert(!XH || (MODE == MODE_GATE_UP && NT == 1), "fp16 activations: gate/up, 8-row items");
  using SG = WStage<NP, NT, AWQ, XH, ONECOL>;
  static_assert(STG >= 2 && STG * SG::kBytes >= NP * NT * 4 * 32 * 4, "stages: a reduction slot");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int slice = warp % ks;
  const int rt = bx * (kWarps / ks) + warp / ks;
  const unsigned long long wpol = l2_evict_first();  // the weights: read once per forward
  // launched with programmatic dependent launch: gate/up waits for its
  // predecessor before reading the work list; the down GEMM (whose
  // predecessor, gate/up, only released it after waiting for the kernel that
  // built the work list) reads the work list and starts its weight copies
  // first, and waits before touching the activations (gate/up's output)
  if (MODE == MODE_GATE_UP) {
    grid_dep_wait();
    grid_dep_release();
  }
  // work items by, by + gy, ... (the grid is sized to
  // the expected items, the loop covers the work list whatever its length)
  const int Mt = (a.M + 15) >> 4;
  const bool live = rt < Mt;
  const int n_items = *a.n_work;
  bool waited = MODE == MODE_GATE_UP;
  for (int item = by; item < n_items; item += gy) {
    const WorkItem it = a.work[item];
    const ExpertDev& ex = a.experts[it.expert];
    const ProjDev* P[2];
    P[0] = MODE == MODE_GATE_UP ? &ex.gate : &pick(ex, a.proj);
    P[1] = &ex.up;
    const int ntc = (it.nrows + 7) >> 3;

    const int nsteps = a.K >> 7;
    const int per = (nsteps + ks - 1) / ks;
    const int s0 = live ? min(nsteps, slice * per) : 0;
    const int s1 = live ? min(nsteps, s0 + per) : 0;
    const int nst = s1 - s0;

    // sources advanced one step per issue
    const unsigned char* bsrc[NT];
    bool bval[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int r = 8 * n + g;
      bval[n] = r < it.nrows && n < ntc;
      const int pos = it.row0 + (r < it.nrows ? r : 0);
      const int row = a.gather ? a.gather[pos] / a.kk : pos;
      bsrc[n] = reinterpret_cast<const unsigned char*>(a.B) + ((size_t)row * a.ldb + 8 * t + s0 * 128) * 2;
    }
    // XH: lanes < 8 copy column `lane`'s group sums with each step; the row
    // scales of columns 2t, 2t + 1 are read now and used by the epilogue
    const float* xsrc = nullptr;
    const bool xval = XH && lane < 8 && lane < it.nrows;
    float bs[2] = {1.f, 1.f};
    if constexpr (XH) {
      const int px = it.row0 + ((lane & 7) < it.nrows ? (lane & 7) : 0);
      xsrc = a.bsum + (size_t)(a.gather ? a.gather[px] / a.kk : px) * a.ng + (size_t)s0 * NG;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = 2 * t + h, pc = it.row0 + (c < it.nrows ? c : 0);
        bs[h] = a.bscale[a.gather ? a.gather[pc] / a.kk : pc];
      }
    }
    const int rtc = live ? rt : 0;
    const unsigned char* wsrc[NP];
    const unsigned char* ssrc[NP];
    const unsigned char* zsrc[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      wsrc[p] = reinterpret_cast<const unsigned char*>(P[p]->q + ((size_t)rtc * a.Kc + 2 * s0) * 32 + piece_slot(lane));
      ssrc[p] = reinterpret_cast<const unsigned char*>(P[p]->s + ((size_t)rtc * a.ng + (size_t)s0 * NG) * 16);
      zsrc[p] = AWQ ? nullptr
                    : reinterpret_cast<const unsigned char*>(P[p]->z + ((size_t)rtc * a.ng + (size_t)s0 * NG) * 16);
    }
    unsigned char* wbase = wsm + (size_t)warp * STG * SG::kBytes;

    // issue the copies of one step into a stage (every lane its own 16 B
    // pieces): the weights (and scales, zeros), then the activations
    auto issue_w = [&](int stage) {
      unsigned char* sb = wbase + stage * SG::kBytes;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        cp_async16_pol(sb + p * 1024 + lane * 16, wsrc[p], wpol);
        cp_async16_pol(sb + p * 1024 + 512 + lane * 16, wsrc[p] + 512, wpol);
        wsrc[p] += 1024;
        if (lane < NG * 2) cp_async16_pol(sb + SG::kW + p * 128 + lane * 16, ssrc[p] + lane * 16, wpol);
        if (!AWQ && lane < NG * 2) cp_async16_pol(sb + SG::kW + SG::kS + p * 128 + lane * 16, zsrc[p] + lane * 16, wpol);
        ssrc[p] += NG * 32;
        if (!AWQ) zsrc[p] += NG * 32;
      }
    };
    auto issue_b = [&](int stage) {
      unsigned char* sb = wbase + stage * SG::kBytes;
#pragma unroll
      for (int n = 0; n < NT; ++n) {  // a lane past the item's rows copies nothing (stale bytes are never stored)
        if (bval[n]) {
#pragma unroll
          for (int b = 0; b < 4; ++b)  // ONECOL: lanes t = 0..3 of row g = 0, [b][t] slots
            cp_async16(sb + SG::kW + SG::kS + SG::kZ + (ONECOL ? b * 64 + t * 16 : (n * 4 + b) * 512 + lane * 16),
                       bsrc[n] + b * 64);
        }
        bsrc[n] += 256;
      }
      if constexpr (XH) {
        if (xval) cp_async_small<NG>(sb + SG::kW + SG::kS + SG::kZ + SG::kB + lane * 16, xsrc);
        xsrc += NG;
      }
    };
    auto issue = [&](int stage) {
      issue_w(stage);
      issue_b(stage);
    };

#pragma unroll
    for (int d = 0; d < STG - 1; ++d)
      if (d < nst) issue_w(d);
    if (!waited) {
      grid_dep_wait();
      grid_dep_release();
      waited = true;
    }
#pragma unroll
    for (int d = 0; d < STG - 1; ++d) {
      if (d < nst) issue_b(d);
      cp_async_commit();
    }

    const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
    const float bias = AWQ ? (float)(128 + a.zp) : 128.f;
    const float zbias = AWQ ? (float)a.zp : 0.f;
    // two partial accumulators per chain (k16 halves kt = 0 / 1) halve the
    // dependent MMA chains; they are added at each group end
    float acc[NP][NT][4], tmp[NP][NT][2][4], xs[NT][2][4];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[p][n][r] = tmp[p][n][0][r] = tmp[p][n][1][r] = 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int r = 0; r < 4; ++r) xs[n][0][r] = xs[n][1][r] = 0.f;

    for (int i = 0; i < nst; ++i) {
      if (i + STG - 1 < nst) issue((i + STG - 1) % STG);
      cp_async_commit();
      cp_async_wait<STG - 1>();
      __syncwarp();  // the scales are copied by lanes 0..2*NG-1 and read by all
      const unsigned char* sb = wbase + (i % STG) * SG::kBytes;
      uint4 wq[NP][2], bv[NT][4];
      float sc[NP][NG][2], zz[NP][NG][2];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        wq[p][0] = *reinterpret_cast<const uint4*>(sb + p * 1024 + lane * 16);
        wq[p][1] = *reinterpret_cast<const uint4*>(sb + p * 1024 + 512 + lane * 16);
#pragma unroll
        for (int q = 0; q < NG; ++q) {
          const __half* sp = reinterpret_cast<const __half*>(sb + SG::kW + p * 128) + q * 16;
          sc[p][q][0] = __half2float(sp[g]);
          sc[p][q][1] = __half2float(sp[g + 8]);
          if (!AWQ) {
            const __half* zp = reinterpret_cast<const __half*>(sb + SG::kW + SG::kS + p * 128) + q * 16;
            zz[p][q][0] = __half2float(zp[g]);
            zz[p][q][1] = __half2float(zp[g + 8]);
          }
        }
      }
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int b = 0; b < 4; ++b)
          bv[n][b] = *reinterpret_cast<const uint4*>(
              sb + SG::kW + SG::kS + SG::kZ + (ONECOL ? b * 64 + t * 16 : (n * 4 + b) * 512 + lane * 16));
      __syncwarp();  // every lane holds its operands before any lane refills this stage

#pragma unroll
      for (int b = 0; b < 4; ++b) {  // 32-wide block b of the step
#pragma unroll
        for (int kt = 0; kt < 2; ++kt) {
          if constexpr (!XH) {
#pragma unroll
            for (int n = 0; n < NT; ++n)
              if (NT == 1 || n < ntc)
                mma_bf16(xs[n][kt], ones, kt ? bv[n][b].z : bv[n][b].x, kt ? bv[n][b].w : bv[n][b].y);
          }
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const uint4& q4 = wq[p][b >> 1];
            const int wi = (b & 1) * 2 + kt;
            const uint32_t wd = wi == 0 ? q4.x : wi == 1 ? q4.y : wi == 2 ? q4.z : q4.w;
            uint32_t af[4];
            if constexpr (XH) {
              raw_word_f16(wd, af);
              mma_f16(tmp[p][0][kt], af, kt ? bv[0][b].z : bv[0][b].x, kt ? bv[0][b].w : bv[0][b].y);
            } else {
              raw_word(wd, af);
#pragma unroll
              for (int n = 0; n < NT; ++n)
                if (NT == 1 || n < ntc)
                  mma_bf16(tmp[p][n][kt], af, kt ? bv[n][b].z : bv[n][b].x, kt ? bv[n][b].w : bv[n][b].y);
            }
          }
        }
        if (XH && (b + 1) % GSB == 0) {  // group end, fp16 path
          const int q = b / GSB;
          const float* xg = reinterpret_cast<const float*>(sb + SG::kW + SG::kS + SG::kZ + SG::kB);
          const float xc[2] = {xg[(2 * t) * 4 + q], xg[(2 * t + 1) * 4 + q]};
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float v = f16_group(tmp[p][0][0][r] + tmp[p][0][1][r], xc[r & 1], r >> 1, zbias);
              acc[p][0][r] = __fmaf_rn(v, sc[p][q][r >> 1], acc[p][0][r]);
              if (!AWQ) acc[p][0][r] = __fmaf_rn(zz[p][q][r >> 1], xc[r & 1], acc[p][0][r]);
              tmp[p][0][0][r] = tmp[p][0][1][r] = 0.f;
            }
        } else if ((b + 1) % GSB == 0) {  // group end
          const int q = b / GSB;
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) xs[n][0][r] += xs[n][1][r];
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
              for (int r = 0; r < 4; ++r) {
                if (ONECOL && (r & 1)) {  // a column no item row reaches
                  tmp[p][n][0][r] = tmp[p][n][1][r] = 0.f;
                  continue;
                }
                const float pr = tmp[p][n][0][r] + tmp[p][n][1][r];
                const float v = __fmaf_rn(-bias, xs[n][0][r], pr);  // sum x*(q - zp)
                acc[p][n][r] = __fmaf_rn(v, sc[p][q][r >> 1], acc[p][n][r]);
                if (!AWQ) acc[p][n][r] = __fmaf_rn(zz[p][q][r >> 1], xs[n][0][r], acc[p][n][r]);
                tmp[p][n][0][r] = tmp[p][n][1][r] = 0.f;
              }
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) xs[n][0][r] = xs[n][1][r] = 0.f;
        }
      }
    }
    cp_async_wait<0>();

    if (ks > 1) {  // K-slice reduction in warp order, in each warp's drained stages
      float* slot = reinterpret_cast<float*>(wbase);
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int r = 0; r < 4; ++r) slot[((p * NT + n) * 4 + r) * 32 + lane] = acc[p][n][r];
      __syncthreads();
      if (slice == 0) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              float v = acc[p][n][r];
              for (int w = 1; w < ks; ++w) {
                const float* o = reinterpret_cast<const float*>(wsm + (size_t)(warp + w) * STG * SG::kBytes);
                v += o[((p * NT + n) * 4 + r) * 32 + lane];
              }
              acc[p][n][r] = v;
            }
      }
    }
    if (live && slice == 0) {
      // C fragment (row g / g+8, col 2t / 2t+1) of each N-tile
      const int m0 = rt * 16 + g, m1 = m0 + 8;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if (n >= ntc) continue;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int col = 8 * n + 2 * t + (r & 1);
          const int m = (r < 2) ? m0 : m1;
          if (col >= it.nrows || m >= a.M) continue;
          const size_t o = (size_t)(it.row0 + col) * a.ldo + m;
          float v = acc[0][n][r];
          if constexpr (XH) v *= bs[r & 1];  // undo the row's 2^-e
          if (!isfinite(v)) v = 0.f;  // non-finite -> 0, as every reference GEMV does
          if (MODE == MODE_GATE_UP) {
            float uu = acc[NP - 1][n][r];
            if constexpr (XH) uu *= bs[r & 1];
            if (!isfinite(uu)) uu = 0.f;
            reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(silu_mul(v, uu));
          } else {
            reinterpret_cast<float*>(a.out)[o] = v;
          }
        }
      }
    }
    if (ks > 1) __syncthreads();  // the next item's copies reuse the reduction slots
  }
}

template <int MODE, int NT, int GSB, bool AWQ, bool XH>
__global__ void __launch_bounds__(kWarps * 32) k_int4_mma(GemmArgs a, int ks) {
  extern __shared__ __align__(128) unsigned char wsm[];
  mma_kblock<MODE, NT, GSB, AWQ, XH>(a, ks, blockIdx.x, blockIdx.y, gridDim.y, wsm);
}

// Persistent form of k_int4_mma for decode-size items (NT = 1: at most 8 rows
// per item; no K split).  The grid stays resident; each warp takes units
// (work item, 16-row tile) from a device counter (a.ctr, zeroed by the
// permutation kernel) and runs their 128-wide K steps back to back through its
// cp.async ring, which never drains between units: while the last steps of a
// unit are multiplied, the first steps of the next one are in flight.  The
// next unit's work item, activation row and weight pointers are fetched when
// the copies enter the current one, so they are in registers when needed.
// Same arithmetic, per unit, as k_int4_mma with ks = 1.
// A unit always carries two weight streams over the same activation rows: the
// gate and up tiles of one 16-row tile (MODE_GATE_UP), or two adjacent 16-row
// tiles of one projection (MODE_PLAIN_F32), so the activation copies, the
// x-sum MMAs and the loop's bookkeeping are shared by 2 KB of weights a step.
// XH (gate/up only): fp16 activations scaled per row (launch_prep_xh), fp16
// weights from raw_word_f16, the group sums of the activations copied in with
// each step instead of the all-ones MMA, and the row scales applied before
// the SiLU*mul epilogue.
template <int MODE, int GSB, bool AWQ, bool XH>
__global__ void __launch_bounds__(kWarps * 32) k_int4_mma_p(GemmArgs a) {
  constexpr int NP = 2;
  constexpr bool PAIR = MODE != MODE_GATE_UP;
  constexpr int NG = GSB == 4 ? 1 : (GSB == 2 ? 2 : 4);  // groups per step
  static_assert(!XH || MODE == MODE_GATE_UP, "fp16 activations: gate/up only");
  using SG = WStage<NP, 1, AWQ, XH>;
  extern __shared__ __align__(128) unsigned char wsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  unsigned char* wbase = wsm + (size_t)warp * kStagesW * SG::kBytes;
  // programmatic dependent launch: as k_int4_mma (the down GEMM starts its
  // first weight copies before it waits for gate/up's output)
  if (MODE == MODE_GATE_UP) {
    grid_dep_wait();
    grid_dep_release();
  }
  const int Mt16 = (a.M + 15) >> 4;  // 16-row tiles
  const int Mt = PAIR ? (Mt16 + 1) >> 1 : Mt16;  // row tiles (pairs) per work item
  const int nunits = *a.n_work * Mt;
  const int nsteps = a.K >> 7;

  // the next unit the copies will enter
  int pu = 0, prow = 0;
  int pxrow = 0;                 // XH: the row of column lane & 7 (its group sums)
  float pbs0 = 1.f, pbs1 = 1.f;  // XH: the row scales of columns 2t, 2t + 1
  WorkItem pit{};
  const uint4* pq[NP];
  const __half* ps[NP];
  const __half* pz[NP];
  auto prefetch = [&]() {
    int u = 0;
    if (lane == 0) u = atomicAdd(a.ctr, 1);
    pu = __shfl_sync(0xffffffffu, u, 0);
    if (pu < nunits) {
      pit = a.work[pu / Mt];
      const int pos = pit.row0 + (g < pit.nrows ? g : 0);
      prow = a.gather ? a.gather[pos] / a.kk : pos;
      if constexpr (XH) {
        const int cx = lane & 7, c0 = 2 * t, c1 = 2 * t + 1;
        const int px = pit.row0 + (cx < pit.nrows ? cx : 0);
        const int p0 = pit.row0 + (c0 < pit.nrows ? c0 : 0), p1 = pit.row0 + (c1 < pit.nrows ? c1 : 0);
        pxrow = a.gather ? a.gather[px] / a.kk : px;
        pbs0 = a.bscale[a.gather ? a.gather[p0] / a.kk : p0];
        pbs1 = a.bscale[a.gather ? a.gather[p1] / a.kk : p1];
      }
      const ExpertDev& ex = a.experts[pit.expert];
      const ProjDev& P0 = MODE == MODE_GATE_UP ? ex.gate : pick(ex, a.proj);
      const ProjDev& P1 = MODE == MODE_GATE_UP ? ex.up : P0;
      pq[0] = P0.q;
      ps[0] = P0.s;
      pz[0] = P0.z;
      pq[1] = P1.q;
      ps[1] = P1.s;
      pz[1] = P1.z;
    }
  };

  // copy side: the unit being copied and its sources, advanced one step per issue
  const unsigned char* wsrc[NP];
  const unsigned char* ssrc[NP];
  const unsigned char* zsrc[NP];
  const unsigned char* bsrc = nullptr;
  const float* xsrc = nullptr;  // XH, lanes < 8: the group sums of column `lane`
  bool bval = false, xval = false;
  int is = 0, entered = 0;
  int n_row0 = 0, n_nrows = 0, n_rt = 0;  // the unit last entered
  float n_bs0 = 1.f, n_bs1 = 1.f;
  auto enter = [&]() {
    const int rt = pu % Mt;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      // tile pair: the second tile of an odd count repeats the first (its
      // results fall on rows >= M and are not stored)
      const int tr = PAIR ? min(2 * rt + p, Mt16 - 1) : rt;
      wsrc[p] = reinterpret_cast<const unsigned char*>(pq[p] + (size_t)tr * a.Kc * 32 + piece_slot(lane));
      ssrc[p] = reinterpret_cast<const unsigned char*>(ps[p] + (size_t)tr * a.ng * 16);
      zsrc[p] = AWQ ? nullptr : reinterpret_cast<const unsigned char*>(pz[p] + (size_t)tr * a.ng * 16);
    }
    bval = g < pit.nrows;
    bsrc = reinterpret_cast<const unsigned char*>(a.B) + ((size_t)prow * a.ldb + 8 * t) * 2;
    if constexpr (XH) {
      xval = lane < 8 && lane < pit.nrows;
      xsrc = a.bsum + (size_t)pxrow * a.ng;
      n_bs0 = pbs0;
      n_bs1 = pbs1;
    }
    n_row0 = pit.row0;
    n_nrows = pit.nrows;
    n_rt = rt;
    is = 0;
    ++entered;
  };
  auto issue_w = [&](int stage) {
    unsigned char* sb = wbase + stage * SG::kBytes;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      cp_async16(sb + p * 1024 + lane * 16, wsrc[p]);
      cp_async16(sb + p * 1024 + 512 + lane * 16, wsrc[p] + 512);
      wsrc[p] += 1024;
      if (lane < NG * 2) cp_async16(sb + SG::kW + p * 128 + lane * 16, ssrc[p] + lane * 16);
      if (!AWQ && lane < NG * 2) cp_async16(sb + SG::kW + SG::kS + p * 128 + lane * 16, zsrc[p] + lane * 16);
      ssrc[p] += NG * 32;
      if (!AWQ) zsrc[p] += NG * 32;
    }
  };
  // a lane past the item's rows copies nothing; its stage bytes are stale
  // and reach only MMA columns that are never stored, so the reads take no
  // predicate
  auto issue_b = [&](int stage) {
    unsigned char* sb = wbase + stage * SG::kBytes;
    if (bval) {
#pragma unroll
      for (int b = 0; b < 4; ++b) cp_async16(sb + SG::kW + SG::kS + SG::kZ + b * 512 + lane * 16, bsrc + b * 64);
    }
    bsrc += 256;
    if constexpr (XH) {
      if (xval) cp_async_small<NG>(sb + SG::kW + SG::kS + SG::kZ + SG::kB + lane * 16, xsrc);
      xsrc += NG;
    }
  };
  bool copying = true;
  // one step of copies; enters the prefetched unit when the current one is done
  auto issue_step = [&](int stage) {
    if (!copying) return;
    if (is == nsteps) {
      if (pu >= nunits) {
        copying = false;
        return;
      }
      enter();
      prefetch();
    }
    issue_w(stage);
    issue_b(stage);
    ++is;
  };

  prefetch();
  if (pu >= nunits) return;  // no unit for this warp (whole warp)
  enter();
  prefetch();
#pragma unroll
  for (int d = 0; d < kStagesW - 1; ++d) issue_w(d);  // nsteps >= kStagesW - 1 (K >= 256)
  if (MODE != MODE_GATE_UP) {
    grid_dep_wait();
    grid_dep_release();
  }
#pragma unroll
  for (int d = 0; d < kStagesW - 1; ++d) {
    issue_b(d);
    ++is;
    cp_async_commit();
  }

  const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
  const float bias = AWQ ? (float)(128 + a.zp) : 128.f;
  const float zbias = AWQ ? (float)a.zp : 0.f;  // XH: the zero point removed at group ends
  float acc[NP][4], tmp[NP][2][4], xs[2][4];  // tmp, xs: a group's partial sums (started fresh)
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[p][r] = 0.f;

  int c_row0 = n_row0, c_nrows = n_nrows, c_rt = n_rt, done = 0, cs = 0;
  float c_bs0 = n_bs0, c_bs1 = n_bs1;
  int st_rd = 0, st_wr = kStagesW - 1;  // ring positions read and filled this step
  for (;;) {
    issue_step(st_wr);
    st_wr = st_wr == kStagesW - 1 ? 0 : st_wr + 1;
    cp_async_commit();
    cp_async_wait<kStagesW - 1>();
    __syncwarp();  // the scales are copied by lanes 0..2*NG-1 and read by all
    const unsigned char* sb = wbase + st_rd * SG::kBytes;
    st_rd = st_rd == kStagesW - 1 ? 0 : st_rd + 1;
    uint4 wq[NP][2], bv[4];
    float sc[NP][NG][2], zz[NP][NG][2];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      wq[p][0] = *reinterpret_cast<const uint4*>(sb + p * 1024 + lane * 16);
      wq[p][1] = *reinterpret_cast<const uint4*>(sb + p * 1024 + 512 + lane * 16);
#pragma unroll
      for (int q = 0; q < NG; ++q) {
        const __half* sp = reinterpret_cast<const __half*>(sb + SG::kW + p * 128) + q * 16;
        sc[p][q][0] = __half2float(sp[g]);
        sc[p][q][1] = __half2float(sp[g + 8]);
        if (!AWQ) {
          const __half* zp = reinterpret_cast<const __half*>(sb + SG::kW + SG::kS + p * 128) + q * 16;
          zz[p][q][0] = __half2float(zp[g]);
          zz[p][q][1] = __half2float(zp[g + 8]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) bv[b] = *reinterpret_cast<const uint4*>(sb + SG::kW + SG::kS + SG::kZ + b * 512 + lane * 16);
    __syncwarp();  // every lane holds its operands before any lane refills this stage

#pragma unroll
    for (int b = 0; b < 4; ++b) {  // 32-wide block b of the step
      const bool fresh = b % GSB == 0;  // first block of a group: new partial sums
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
        if constexpr (!XH) {
          if (fresh)
            mma_bf16_z(xs[kt], ones, kt ? bv[b].z : bv[b].x, kt ? bv[b].w : bv[b].y);
          else
            mma_bf16(xs[kt], ones, kt ? bv[b].z : bv[b].x, kt ? bv[b].w : bv[b].y);
        }
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const uint4& q4 = wq[p][b >> 1];
          const int wi = (b & 1) * 2 + kt;
          const uint32_t wd = wi == 0 ? q4.x : wi == 1 ? q4.y : wi == 2 ? q4.z : q4.w;
          uint32_t af[4];
          if constexpr (XH) {
            raw_word_f16(wd, af);
            if (fresh)
              mma_f16_z(tmp[p][kt], af, kt ? bv[b].z : bv[b].x, kt ? bv[b].w : bv[b].y);
            else
              mma_f16(tmp[p][kt], af, kt ? bv[b].z : bv[b].x, kt ? bv[b].w : bv[b].y);
          } else {
            raw_word(wd, af);
            if (fresh)
              mma_bf16_z(tmp[p][kt], af, kt ? bv[b].z : bv[b].x, kt ? bv[b].w : bv[b].y);
            else
              mma_bf16(tmp[p][kt], af, kt ? bv[b].z : bv[b].x, kt ? bv[b].w : bv[b].y);
          }
        }
      }
      if ((b + 1) % GSB == 0) {  // group end
        const int q = b / GSB;
        if constexpr (XH) {
          // the group sums of columns 2t and 2t+1 (copied with the step)
          const float* xg = reinterpret_cast<const float*>(sb + SG::kW + SG::kS + SG::kZ + SG::kB);
          const float xc[2] = {xg[(2 * t) * 4 + q], xg[(2 * t + 1) * 4 + q]};
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float v = f16_group(tmp[p][0][r] + tmp[p][1][r], xc[r & 1], r >> 1, zbias);
              acc[p][r] = __fmaf_rn(v, sc[p][q][r >> 1], acc[p][r]);
              if (!AWQ) acc[p][r] = __fmaf_rn(zz[p][q][r >> 1], xc[r & 1], acc[p][r]);
            }
        } else {
#pragma unroll
          for (int r = 0; r < 4; ++r) xs[0][r] += xs[1][r];
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float pr = tmp[p][0][r] + tmp[p][1][r];
              const float v = __fmaf_rn(-bias, xs[0][r], pr);  // sum x*(q - zp)
              acc[p][r] = __fmaf_rn(v, sc[p][q][r >> 1], acc[p][r]);
              if (!AWQ) acc[p][r] = __fmaf_rn(zz[p][q][r >> 1], xs[0][r], acc[p][r]);
            }
        }
      }
    }

    if (++cs < nsteps) continue;
    // unit done: C fragment (row g / g+8, col 2t / 2t+1) -> outputs
#pragma unroll
    for (int p = 0; p < (PAIR ? 2 : 1); ++p) {
      const int m0 = (PAIR ? 2 * c_rt + p : c_rt) * 16 + g, m1 = m0 + 8;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int col = 2 * t + (r & 1);
        const int m = (r < 2) ? m0 : m1;
        if (col < c_nrows && m < a.M) {
          const size_t o = (size_t)(c_row0 + col) * a.ldo + m;
          float v = acc[p][r];
          if constexpr (XH) v *= (r & 1) ? c_bs1 : c_bs0;  // undo the row's 2^-e
          if (!isfinite(v)) v = 0.f;  // non-finite -> 0, as every reference GEMV does
          if (MODE == MODE_GATE_UP) {
            float uu = acc[1][r];
            if constexpr (XH) uu *= (r & 1) ? c_bs1 : c_bs0;
            if (!isfinite(uu)) uu = 0.f;
            reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(silu_mul(v, uu));
          } else {
            reinterpret_cast<float*>(a.out)[o] = v;
          }
        }
      }
    }
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[p][r] = 0.f;
    cs = 0;
    // the copies run kStagesW - 1 steps ahead and units have >= kStagesW - 1
    // steps, so the next unit (if any) has been entered by now
    if (++done == entered) break;
    c_row0 = n_row0;
    c_nrows = n_nrows;
    c_rt = n_rt;
    c_bs0 = n_bs0;
    c_bs1 = n_bs1;
  }
  cp_async_wait<0>();
}

template <int MODE, int NT, int GSB, bool AWQ, bool XH>
static void launch_mma_k(const GemmArgs& a, dim3 grid, int ks, cudaStream_t st) {
  constexpr int NP = MODE == MODE_GATE_UP ? 2 : 1;
  const size_t smem = (size_t)kWarps * kStagesW * WStage<NP, NT, AWQ, XH>::kBytes;
  static bool attr = false;  // per template instance
  if (!attr) {
    cudaFuncSetAttribute(k_int4_mma<MODE, NT, GSB, AWQ, XH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    attr = true;
  }
  launch_pdl(k_int4_mma<MODE, NT, GSB, AWQ, XH>, grid, dim3(kWarps * 32), smem, st, a, ks);
}

// Persistent grid: as many 4-warp CTAs as fit on the SMs at once.
template <int MODE, int GSB, bool AWQ, bool XH>
static int mma_p_grid() {
  constexpr int NP = 2;  // two weight streams per unit in both modes
  const size_t smem = (size_t)kWarps * kStagesW * WStage<NP, 1, AWQ, XH>::kBytes;
  static int grid = 0;  // per template instance (one device per process in practice)
  if (!grid) {
    cudaFuncSetAttribute(k_int4_mma_p<MODE, GSB, AWQ, XH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int per_sm = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_int4_mma_p<MODE, GSB, AWQ, XH>, kWarps * 32, smem);
    grid = std::max(1, per_sm) * std::max(1, sms);
  }
  return grid;
}

template <int MODE, int GSB, bool AWQ, bool XH>
static void launch_mma_pk(const GemmArgs& a, cudaStream_t st) {
  constexpr int NP = 2;
  const size_t smem = (size_t)kWarps * kStagesW * WStage<NP, 1, AWQ, XH>::kBytes;
  launch_pdl(k_int4_mma_p<MODE, GSB, AWQ, XH>, dim3(mma_p_grid<MODE, GSB, AWQ, XH>()), dim3(kWarps * 32), smem, st,
             a);
}

template <int MODE, bool AWQ, bool XH>
static int mma_p_grid_gs(int gs) {
  return gs == 32 ? mma_p_grid<MODE, 1, AWQ, XH>()
                  : (gs == 64 ? mma_p_grid<MODE, 2, AWQ, XH>() : mma_p_grid<MODE, 4, AWQ, XH>());
}
static long mma_p_resident_warps(bool gate_up, int gs, int awq, bool xh) {
  int grid;
  if (gate_up && xh)
    grid = awq ? mma_p_grid_gs<MODE_GATE_UP, true, true>(gs) : mma_p_grid_gs<MODE_GATE_UP, false, true>(gs);
  else if (gate_up)
    grid = awq ? mma_p_grid_gs<MODE_GATE_UP, true, false>(gs) : mma_p_grid_gs<MODE_GATE_UP, false, false>(gs);
  else
    grid = awq ? mma_p_grid_gs<MODE_PLAIN_F32, true, false>(gs) : mma_p_grid_gs<MODE_PLAIN_F32, false, false>(gs);
  return (long)grid * kWarps;
}

template <int MODE, bool XH>
static void launch_mma_p(const GemmArgs& a, int awq, cudaStream_t st) {
  if (awq) {
    switch (a.gs) {
      case 32: launch_mma_pk<MODE, 1, true, XH>(a, st); break;
      case 64: launch_mma_pk<MODE, 2, true, XH>(a, st); break;
      default: launch_mma_pk<MODE, 4, true, XH>(a, st); break;
    }
  } else {
    switch (a.gs) {
      case 32: launch_mma_pk<MODE, 1, false, XH>(a, st); break;
      case 64: launch_mma_pk<MODE, 2, false, XH>(a, st); break;
      default: launch_mma_pk<MODE, 4, false, XH>(a, st); break;
    }
  }
}

template <int MODE, int NT, bool AWQ, bool XH>
static void launch_mma_gs(const GemmArgs& a, int max_work, int ks, cudaStream_t st) {
  const int Mt = (a.M + 15) / 16;
  const dim3 grid((Mt * ks + kWarps - 1) / kWarps, max_work);
  switch (a.gs) {
    case 32: launch_mma_k<MODE, NT, 1, AWQ, XH>(a, grid, ks, st); break;
    case 64: launch_mma_k<MODE, NT, 2, AWQ, XH>(a, grid, ks, st); break;
    default: launch_mma_k<MODE, NT, 4, AWQ, XH>(a, grid, ks, st); break;
  }
}

// Items of at most 8 rows (one mma N tile): larger items take the tcgen05
// kernel (int4_umma.cu) or the CUDA-core kernel.
template <int MODE, bool XH>
static void launch_mma(const GemmArgs& a, int max_work, int ks, int awq, cudaStream_t st) {
  if (awq) launch_mma_gs<MODE, 1, true, XH>(a, max_work, ks, st);
  else launch_mma_gs<MODE, 1, false, XH>(a, max_work, ks, st);
}

// ------------------------------------------------------ CUDA-core fp32 GEMV

template <typename BT>
__device__ __forceinline__ void load8(const BT* p, float v[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float v[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float v[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Same work decomposition as k_int4_mma: one 16-row tile per warp; lane
// (g, t) owns rows g and g+8 at the 16 k positions of its fragment words.
// Per group it forms sum x*(q - zp) (AWQ) or sum x*q and sum x (GPTQ) in
// fp32 and accumulates them times the group scale (and zero).  Handles the
// item's rows TOK at a time.
template <int MODE, typename BT, int TOK>
__global__ void __launch_bounds__(128) k_int4_cc(GemmArgs a, int awq) {
  constexpr int NP = MODE == MODE_GATE_UP ? 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = blockIdx.x * 4 + warp;
  if (rt * 16 >= a.M) return;
  if ((int)blockIdx.y >= *a.n_work) return;
  const WorkItem it = a.work[blockIdx.y];
  const ExpertDev& ex = a.experts[it.expert];
  const ProjDev* P[2];
  P[0] = MODE == MODE_GATE_UP ? &ex.gate : &pick(ex, a.proj);
  P[1] = &ex.up;
  const float zp = (float)a.zp;

  for (int r0 = 0; r0 < it.nrows; r0 += TOK) {
    const BT* brow[TOK];
    bool bv[TOK];
#pragma unroll
    for (int j = 0; j < TOK; ++j) {
      bv[j] = r0 + j < it.nrows;
      const int pos = it.row0 + (bv[j] ? r0 + j : 0);
      const int row = a.gather ? a.gather[pos] / a.kk : pos;
      brow[j] = reinterpret_cast<const BT*>(a.B) + (size_t)row * a.ldb + 8 * t;
    }
    float acc[NP][2][TOK];
    float pq[NP][2][TOK], px[TOK];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < TOK; ++j) acc[p][h][j] = pq[p][h][j] = 0.f;
#pragma unroll
    for (int j = 0; j < TOK; ++j) px[j] = 0.f;

    for (int c = 0; c < a.Kc; ++c) {
      uint4 qw[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) qw[p] = ldg_nc(P[p]->q + ((size_t)rt * a.Kc + c) * 32 + piece_slot(lane));
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        const int k32 = c * 64 + kb * 32;
        if (k32 >= a.K) break;
        float xv[TOK][8];
#pragma unroll
        for (int j = 0; j < TOK; ++j) {
          if (bv[j]) {
            load8<BT>(brow[j] + k32, xv[j]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) xv[j][e] = 0.f;
          }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const uint32_t w0 = kb ? qw[p].z : qw[p].x;
          const uint32_t w1 = kb ? qw[p].w : qw[p].y;
          // element e (0..7) of the lane's 8 k values: kt = e>>2, i = e&3
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t w = (e >> 2) ? w1 : w0;
            const int i = e & 3;
            const int slot = (i & 1) * 4 + (i >> 1) * 2;
            const float q0 = (float)((w >> (4 * slot)) & 0xF);
            const float q1 = (float)((w >> (4 * (slot + 1))) & 0xF);
            const float d0 = awq ? q0 - zp : q0;
            const float d1 = awq ? q1 - zp : q1;
#pragma unroll
            for (int j = 0; j < TOK; ++j) {
              pq[p][0][j] = __fmaf_rn(xv[j][e], d0, pq[p][0][j]);
              pq[p][1][j] = __fmaf_rn(xv[j][e], d1, pq[p][1][j]);
            }
          }
        }
        if (!awq) {
#pragma unroll
          for (int j = 0; j < TOK; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) px[j] += xv[j][e];
        }
        if (((k32 + 32) % a.gs) == 0 || k32 + 32 >= a.K) {
          const int grp = k32 / a.gs;
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const size_t so = ((size_t)rt * a.ng + grp) * 16;
            const float s0 = __half2float(P[p]->s[so + g]), s1 = __half2float(P[p]->s[so + g + 8]);
            float z0 = 0.f, z1 = 0.f;
            if (!awq && P[p]->z) {
              z0 = __half2float(P[p]->z[so + g]);
              z1 = __half2float(P[p]->z[so + g + 8]);
            }
#pragma unroll
            for (int j = 0; j < TOK; ++j) {
              acc[p][0][j] = __fmaf_rn(pq[p][0][j], s0, acc[p][0][j]);
              acc[p][1][j] = __fmaf_rn(pq[p][1][j], s1, acc[p][1][j]);
              if (!awq) {
                acc[p][0][j] = __fmaf_rn(px[j], z0, acc[p][0][j]);
                acc[p][1][j] = __fmaf_rn(px[j], z1, acc[p][1][j]);
              }
              pq[p][0][j] = pq[p][1][j] = 0.f;
            }
          }
#pragma unroll
          for (int j = 0; j < TOK; ++j) px[j] = 0.f;
        }
      }
    }
    // reduce over the 4 lanes t of row group g
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < TOK; ++j) {
          float v = acc[p][h][j];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          acc[p][h][j] = v;
        }
    if (t == 0) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int m = rt * 16 + g + 8 * h;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < TOK; ++j) {
          if (!bv[j]) continue;
          const size_t o = (size_t)(it.row0 + r0 + j) * a.ldo + m;
          float v = acc[0][h][j];
          if (!isfinite(v) && !(MODE == MODE_PLAIN_F32 && a.keep_nonfinite)) v = 0.f;
          if (MODE == MODE_GATE_UP) {
            float u = acc[NP - 1][h][j];
            if (!isfinite(u)) u = 0.f;
            const float mid = silu_mul(v, u);
            if (a.out_bf16)
              reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(mid);
            else
              reinterpret_cast<float*>(a.out)[o] = mid;
          } else {
            reinterpret_cast<float*>(a.out)[o] = v;
          }
        }
      }
    }
  }
}

// ----------------------------------------------------------------- combine

// y[t,h] = sum_{j<kk} w[t,j] * d[inverse[t*kk+j], h] in j order (fma), the
// order of the reference's combine (qwen3_6_moe_int4_model.cpp:213, :372).
template <typename OT>
__device__ __forceinline__ void combine_store(OT* y, size_t o, const float (&ap)[4], int n) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i >= n) break;
    if constexpr (sizeof(OT) == 2)
      y[o + i] = __float2bfloat16_rn(ap[i]);
    else
      y[o + i] = ap[i];
  }
}

// A thread owns 4 consecutive h of a column and walks the tokens t =
// blockIdx.y, blockIdx.y + gridDim.y, ... two at a time, with every slot row
// of both tokens requested before the ordered FMAs (streaming loads: each
// partial row is read once).
template <typename OT>
__global__ void __launch_bounds__(256) k_combine(const float* __restrict__ d, const int* __restrict__ inverse,
                                                 const float* __restrict__ w, int T, int kk, int H, OT* y,
                                                 int skip_tiny, const __nv_bfloat16* res) {
  grid_dep_wait();
  grid_dep_release();
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (h >= H) return;
  const bool full4 = h + 3 < H;
  const int nh = full4 ? 4 : H - h;
  for (int t0 = blockIdx.y; t0 < T; t0 += 2 * gridDim.y) {
    const int tt[2] = {t0, t0 + (int)gridDim.y};
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    int live[2] = {0, 0};
    for (int j0 = 0; j0 < kk; j0 += 8) {
      float wj[2][8];
      float4 v[2][8];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u;
          wj[q][u] = 0.f;
          v[q][u] = make_float4(0.f, 0.f, 0.f, 0.f);
          const int src = j < kk && tt[q] < T ? inverse[(size_t)tt[q] * kk + j] : -1;
          if (src >= 0) {  // src < 0: an empty slot (not placed by the permutation)
            ++live[q];
            wj[q][u] = w ? w[(size_t)tt[q] * kk + j] : 1.f;
            const float* row = d + (size_t)src * H + h;
            if (full4) {
              v[q][u] = __ldcs(reinterpret_cast<const float4*>(row));
            } else {  // the last 1-3 columns of a row whose H is not a multiple of 4
              v[q][u].x = row[0];
              if (nh > 1) v[q][u].y = row[1];
              if (nh > 2) v[q][u].z = row[2];
            }
          }
        }
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (j0 + u >= kk || (skip_tiny && fabsf(wj[q][u]) < 1e-12f)) continue;
          acc[q].x = __fmaf_rn(wj[q][u], v[q][u].x, acc[q].x);
          acc[q].y = __fmaf_rn(wj[q][u], v[q][u].y, acc[q].y);
          acc[q].z = __fmaf_rn(wj[q][u], v[q][u].z, acc[q].z);
          acc[q].w = __fmaf_rn(wj[q][u], v[q][u].w, acc[q].w);
        }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (tt[q] >= T || live[q] == 0) continue;  // a row of empty slots only is left untouched
      float ap[4] = {acc[q].x, acc[q].y, acc[q].z, acc[q].w};
      const size_t o = (size_t)tt[q] * H + h;
      if (res)  // residual stream: y = r + sum (one fp32 add; res may alias y, read before written)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i < nh) ap[i] = __fadd_rn(__bfloat162float(res[o + i]), ap[i]);
      combine_store(y, o, ap, nh);
    }
  }
}

// ------------------------------------------- fused single-token decode

// Tag of barrier b of the launch with this epoch (splitmix64's finaliser over
// epoch * 4 + b): neither an older launch's words nor the bytes of an
// uninitialised workspace equal it except by a 2^-64 accident, so the barrier
// words need no reset between launches.
__device__ __forceinline__ unsigned long long decode1_tag(unsigned long long epoch, int b) {
  unsigned long long x = epoch * 4ull + (unsigned long long)b + 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier b of k_moe_decode1 (b = 0, 1, 2): an arrival counter at
// a.bar[0] (its low 32 bits), zero when a launch starts (zeroed by the last
// CTA of the previous launch past its last barrier, or by CTA 0 when the tag
// in a.bar[1] is not this launch's, before it publishes it); a CTA checks
// that tag once before its first arrival (so no arrival lands before a
// reset), then
// every barrier is one release-add and a poll until the count reaches
// (b + 1) * gridDim.x.  Each wait gives up after a.budget SM clocks: bit 2 of
// *a.err is set and the kernel goes on (its outputs are then invalid), so a
// launch never waits without end.  All threads of every CTA call it.
__device__ __forceinline__ void decode1_barrier(const Decode1Args& a, int b) {
  __syncthreads();  // the CTA's writes of this phase are issued
  if (threadIdx.x == 0) {
    bool timed_out = false;
    unsigned int* ctr = reinterpret_cast<unsigned int*>(a.bar);
    if (b == 0) {
      const unsigned long long tag = decode1_tag(a.epoch, 0);
      const long long t0 = clock64();
      while (ld_acquire_gpu_u64(a.bar + 1) != tag) {
        if (clock64() - t0 > a.budget) {
          timed_out = true;
          break;
        }
        __nanosleep(32);
      }
    }
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(ctr), "r"(1u) : "memory");
    const unsigned int target = (unsigned int)(b + 1) * gridDim.x;
    const long long t0 = clock64();
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (clock64() - t0 > a.budget) {
        timed_out = true;
        break;
      }
      __nanosleep(32);
    }
    if (timed_out) atomicOr(a.err, 4);
  }
  __syncthreads();
}

// One token through the whole layer in one cooperative launch (T = 1 decode:
// the chain of separate kernels is bound by its launch boundaries, not its
// bytes).  Phases, split by decode1_barrier:
//   1. router rows r = blockIdx.x, + gridDim.x, ...: W_r row r and the token
//      in shared memory, one warp's ordered FMA chains (router_dot_warp, the
//      arithmetic of k_router_small); the sigmoid router's score of the row
//      too (sigmoid_ref: its double arithmetic once per row, in parallel).
//   2. every CTA: the token's top-k from the logits (topk_token, the same
//      bits in every CTA) into shared memory; slot j becomes work item j (one
//      row of expert ids[j]); CTA 0 writes the routing views (ids, weights,
//      the canonical offsets / sorted / inverse of one token).
//   3. gate/up + SiLU*mul: the blocks of k_int4_mma's grid (gx_gu x kk) dealt
//      round-robin to the CTAs, each run by mma_kblock on the bf16 token row.
//      (A bulk L2 prefetch of each block's weights one block ahead was
//      measured: no gain at Qwen / GLM sizes, and at Kimi's 223 MB per token
//      its ~100 MB in flight were evicted before use: 92 -> 105 us.)
//   4. down: the same over the gate/up rows (gx_dn x kk blocks).
//   5. combine: y = sum_j w_j * partial_j in slot order (k_combine's fmaf
//      order), + the residual, to bf16.
// Ring depths of the GEMM phases (stages of the one-row layout: gate/up
// 2.5 KB, down 1.4 KB per warp).  Measured on the three BASELINE layers, step
// time with gate/up / down stages 3/3, 4/6, 5/8: Qwen 22.6 / 22.9 / 24.2 us,
// GLM 39.0 / 39.9 / 41.3, Kimi 81.9 / 85.9 / 87.4 -- bytes in flight are not
// what bounds these phases, and deeper rings cost registers.
constexpr int kDecode1StagesGu = 3, kDecode1StagesDn = 3;
// Four CTAs per SM (at most 128 registers): more warps to hide the GEMM
// phases' dependency latency; measured on Kimi-K2 (group 32, 142 registers
// uncapped, 3 CTAs per SM), 82.1 -> 79.2 us per token.
template <int GSB, bool AWQ>
__global__ void __launch_bounds__(kWarps * 32, 4) k_moe_decode1(Decode1Args a) {
  extern __shared__ __align__(128) unsigned char wsm[];
  __shared__ WorkItem s_work[kDecode1MaxSlots];
  __shared__ int s_ids[kDecode1MaxSlots];
  __shared__ float s_w[kDecode1MaxSlots];
  __shared__ int s_nwork;
  // slot j's expert (work item j names slot j), after the GEMM rings
  ExpertDev* s_ex = reinterpret_cast<ExpertDev*>(wsm + a.ex_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H, kk = a.ta.kk;
  grid_dep_wait();  // the token row is the predecessor's output
  grid_dep_release();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *a.err = 0;
    // a launch with a new tag (another epoch, or words this kernel did not
    // write) zeroes the barrier's counters, then publishes the tag; a replay
    // of the same launch (a captured graph: same epoch) finds its tag there
    // and the counters already zeroed by the previous replay's last CTA
    const unsigned long long tag = decode1_tag(a.epoch, 0);
    if (ld_acquire_gpu_u64(a.bar + 1) != tag) {
      *reinterpret_cast<unsigned int*>(a.bar) = 0;
      *reinterpret_cast<unsigned int*>(a.bar + 2) = 0;
      __threadfence();
      st_release_gpu_u64(a.bar + 1, tag);
    }
  }

  // 1. router rows (and the sigmoid router's scores)
  {
    const uint16_t* sw = reinterpret_cast<const uint16_t*>(wsm);
    const uint16_t* sx = sw + H;
    const int n8 = H / 8;
    for (int r = blockIdx.x; r < a.rows; r += gridDim.x) {
      for (int i = threadIdx.x; i < 2 * n8; i += blockDim.x) {
        const uint4* src = i < n8 ? reinterpret_cast<const uint4*>(a.Wr + (size_t)r * H) + i
                                  : reinterpret_cast<const uint4*>(a.X) + (i - n8);
        reinterpret_cast<uint4*>(wsm)[i] = __ldg(src);
      }
      __syncthreads();
      if (warp == 0) {
        const float v = router_dot_warp(sw, sx, H, lane);
        if (lane == 0) {
          a.logits[r] = v;
          if (a.sig && r < a.ta.E) a.sig[r] = sigmoid_ref(v);
        }
      }
      __syncthreads();  // the staging is rewritten by the next row
    }
  }
  decode1_barrier(a, 0);

  // 2. top-k and the work list (every CTA), the routing views (CTA 0)
  if (warp == 0) {
    TopkArgs ta = a.ta;
    ta.ids = s_ids;
    ta.weights = s_w;
    ta.ep_key = nullptr;
    ta.shared_w = nullptr;
    topk_token(ta, 0, lane);
  }
  __syncthreads();
  if ((int)threadIdx.x < kk) {
    const int j = threadIdx.x;
    s_ex[j] = a.gu.experts[s_ids[j]];
    WorkItem it;
    it.expert = j;  // into s_ex
    it.row0 = j;
    it.nrows = 1;
    it.pad = 0;
    s_work[j] = it;
  }
  if (threadIdx.x == 0) s_nwork = kk;
  __shared__ int s_active;
  if (threadIdx.x == 0) s_active = 0;
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int j = threadIdx.x; j < kk; j += blockDim.x) {
      const int e = s_ids[j];
      int rank = 0;
      bool first = true;
      for (int i = 0; i < kk; ++i) {
        rank += s_ids[i] < e || (s_ids[i] == e && i < j);
        first = first && !(s_ids[i] == e && i < j);
      }
      a.ta.ids[j] = e;
      a.ta.weights[j] = s_w[j];
      a.sorted[rank] = j;
      a.inverse[j] = rank;
      if (first) atomicAdd(&s_active, 1);
    }
    for (int e = threadIdx.x; e <= a.n_exp; e += blockDim.x) {
      int c = 0;
      for (int i = 0; i < kk; ++i) c += s_ids[i] < e;
      a.offsets[e] = c;
    }
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0) *a.n_active = s_active;

  // 3. gate/up + SiLU*mul
  {
    GemmArgs g = a.gu;
    g.experts = s_ex;
    g.work = s_work;
    g.n_work = &s_nwork;
    g.gather = nullptr;
    g.ldb = 0;  // every slot reads the token's row
    const int nvb = a.gx_gu * kk;
    for (int vb = blockIdx.x; vb < nvb; vb += gridDim.x)
      mma_kblock<MODE_GATE_UP, 1, GSB, AWQ, false, true, kDecode1StagesGu>(g, a.ks_gu, vb % a.gx_gu, vb / a.gx_gu,
                                                                         kk, wsm);
  }
  decode1_barrier(a, 1);

  // 4. down
  {
    GemmArgs d = a.dn;
    d.experts = s_ex;
    d.work = s_work;
    d.n_work = &s_nwork;
    d.gather = nullptr;  // B row = slot j (the gate/up output row)
    d.kk = kk;
    const int nvb = a.gx_dn * kk;
    for (int vb = blockIdx.x; vb < nvb; vb += gridDim.x)
      mma_kblock<MODE_PLAIN_F32, 1, GSB, AWQ, false, true, kDecode1StagesDn>(d, a.ks_dn, vb % a.gx_dn, vb / a.gx_dn,
                                                                           kk, wsm);
  }
  decode1_barrier(a, 2);
  if (threadIdx.x == 0) {  // the last CTA past the last barrier zeroes the counters for the next launch
    unsigned int* done = reinterpret_cast<unsigned int*>(a.bar + 2);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *reinterpret_cast<unsigned int*>(a.bar) = 0;
      *done = 0;
    }
  }

  // 5. combine (+ residual)
  for (int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4; h < H; h += gridDim.x * blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < kk; ++j) {
      const float wj = s_w[j];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a.partial + (size_t)j * H + h));
      acc.x = __fmaf_rn(wj, v.x, acc.x);
      acc.y = __fmaf_rn(wj, v.y, acc.y);
      acc.z = __fmaf_rn(wj, v.z, acc.z);
      acc.w = __fmaf_rn(wj, v.w, acc.w);
    }
    float ap[4] = {acc.x, acc.y, acc.z, acc.w};
    if (a.R)  // read before written (R may alias Y)
#pragma unroll
      for (int i = 0; i < 4; ++i) ap[i] = __fadd_rn(__bfloat162float(a.R[h + i]), ap[i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) a.Y[h + i] = __float2bfloat16_rn(ap[i]);
  }
}

template <int GSB, bool AWQ>
static size_t decode1_smem_k() {
  return std::max((size_t)kWarps * kDecode1StagesGu * WStage<2, 1, AWQ, false, true>::kBytes,
                  (size_t)kWarps * kDecode1StagesDn * WStage<1, 1, AWQ, false, true>::kBytes);
}

// K split and virtual grid width of one GEMM phase: the split (1, 2 or 4 warps
// per 16-row tile) with the fewest 128-wide K steps per warp over the rounds
// of blocks the grid needs; ties keep the smaller split (no reduction).
static void decode1_split(int M, int K, int kk, int grid, int* ks, int* gx) {
  const int Mt = (M + 15) / 16, nsteps = K / 128;
  long best = -1;
  for (int c = 1; c <= kWarps; c *= 2) {
    if (c > 1 && c > nsteps) break;
    const int g = (Mt * c + kWarps - 1) / kWarps;
    const long rounds = ((long)g * kk + grid - 1) / grid;
    const long cost = rounds * ((nsteps + c - 1) / c);
    if (best < 0 || cost < best) {
      best = cost;
      *ks = c;
      *gx = g;
    }
  }
}

template <int GSB, bool AWQ>
static cudaError_t launch_decode1_k(Decode1Args a, cudaStream_t st) {
  // grid: every CTA resident at once (a cooperative launch).  The function's
  // dynamic shared memory limit only grows and the grid is kept per (device,
  // bytes), both under a lock and read into locals, so launches of layers
  // with different needs from several host threads never pair one layer's
  // grid or limit with another's bytes.
  static std::mutex mu;
  static std::map<int, size_t> limit;               // device -> attribute set so far
  static std::map<std::pair<int, size_t>, int> grids;  // (device, bytes) -> resident grid
  static std::atomic<bool> pdl{true};  // programmatic launch together with the cooperative attribute
  a.ex_off = (int)((std::max(decode1_smem_k<GSB, AWQ>(), (size_t)a.H * 4) + 15) / 16 * 16);
  const size_t smem = (size_t)a.ex_off + (size_t)a.ta.kk * sizeof(ExpertDev);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  int dev = 0, grid = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    size_t& lim = limit[dev];
    if (smem > lim) {
      e = cudaFuncSetAttribute(k_moe_decode1<GSB, AWQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      lim = smem;
    }
    int& g = grids[{dev, smem}];
    if (!g) {
      int per_sm = 0, sms = 0;
      if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_moe_decode1<GSB, AWQ>, kWarps * 32, smem);
      if (e != cudaSuccess) return e;
      if (per_sm < 1) return cudaErrorInvalidConfiguration;
      g = std::min(per_sm * sms, kDecode1MaxCtas);
    }
    grid = g;
  }
  decode1_split(a.gu.M, a.gu.K, a.ta.kk, grid, &a.ks_gu, &a.gx_gu);
  decode1_split(a.dn.M, a.dn.K, a.ta.kk, grid, &a.ks_dn, &a.gx_dn);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const bool with_pdl = pdl.load(std::memory_order_relaxed);
  cfg.numAttrs = with_pdl ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, k_moe_decode1<GSB, AWQ>, a);
  if (e != cudaSuccess && with_pdl) {  // refused with both attributes: cooperative alone
    (void)cudaGetLastError();
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k_moe_decode1<GSB, AWQ>, a);
    if (e == cudaSuccess) pdl.store(false, std::memory_order_relaxed);  // it was the pair of attributes
  }
  return e;
}

cudaError_t launch_decode1(Decode1Args a, int awq, cudaStream_t st) {
  const int gs = a.gu.gs;
  if (a.ta.kk > kDecode1MaxSlots || a.H % 256 != 0) return cudaErrorInvalidValue;
  if (awq) {
    switch (gs) {
      case 32: return launch_decode1_k<1, true>(a, st);
      case 64: return launch_decode1_k<2, true>(a, st);
      default: return launch_decode1_k<4, true>(a, st);
    }
  }
  switch (gs) {
    case 32: return launch_decode1_k<1, false>(a, st);
    case 64: return launch_decode1_k<2, false>(a, st);
    default: return launch_decode1_k<4, false>(a, st);
  }
}

// ------------------------------------------- fp16 activation rows (decode)

// One warp per row (launch_prep_xh): prep_xh_row (common.cuh) on row w, or on
// row rows_of[w] for w < *n_valid.
__global__ void __launch_bounds__(256) k_prep_xh(const uint4* __restrict__ X, int R, int H, int gs,
                                                 const int* __restrict__ rows_of, const int* __restrict__ n_valid,
                                                 uint4* __restrict__ Xh, float* __restrict__ xsum,
                                                 float* __restrict__ xscale) {
  grid_dep_wait();
  grid_dep_release();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= R) return;
  int r = w;
  if (rows_of) {
    if (w >= *n_valid) return;
    r = rows_of[w];
  }
  prep_xh_row<16, true>(X + (size_t)r * (H / 8), r, H, gs, Xh, xsum, xscale, lane);
}

cudaError_t launch_prep_xh(const void* X, int R, int H, int gs, const int* rows_of, const int* n_valid, void* Xh,
                           float* xsum, float* xscale, cudaStream_t st) {
  if (R <= 0) return cudaSuccess;
  if (H % 128 || (gs != 32 && gs != 64 && gs != 128)) return cudaErrorInvalidValue;
  return launch_pdl(k_prep_xh, dim3((R + 7) / 8), dim3(256), 0, st, reinterpret_cast<const uint4*>(X), R, H, gs,
                    rows_of, n_valid, reinterpret_cast<uint4*>(Xh), xsum, xscale);
}

// ---------------------------------------------------------------- quantize

// quant_awq_sym: scale = max(absmax / 7, 1e-8); optionally rounded to bf16;
// stored as fp16 (round-to-nearest-even); q = clip(rint(w / scale) + 7, 0, 15).
__global__ void k_quant_awq_sym(const __nv_bfloat16* __restrict__ W, int M, int K, int gs,
                                int bf16_scale, uint8_t* __restrict__ q, __half* __restrict__ sc) {
  const int ng = K / gs;
  const size_t n = (size_t)M * ng;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / ng), grp = (int)(i % ng);
    const __nv_bfloat16* row = W + (size_t)m * K + (size_t)grp * gs;
    float amax = 0.f;
    for (int k = 0; k < gs; ++k) amax = fmaxf(amax, fabsf(__bfloat162float(row[k])));
    float s = __fdiv_rn(amax, 7.0f);
    if (!(s > 1e-8f)) s = 1e-8f;
    if (bf16_scale) s = __bfloat162float(__float2bfloat16_rn(s));
    sc[i] = __float2half_rn(s);
    uint8_t* qo = q + (size_t)m * (K / 2) + (size_t)grp * gs / 2;
    for (int k = 0; k < gs; k += 2) {
      float q0 = rintf(__fdiv_rn(__bfloat162float(row[k]), s)) + 7.f;
      float q1 = rintf(__fdiv_rn(__bfloat162float(row[k + 1]), s)) + 7.f;
      q0 = fminf(fmaxf(q0, 0.f), 15.f);
      q1 = fminf(fmaxf(q1, 0.f), 15.f);
      qo[k / 2] = (uint8_t)((uint32_t)q0 | ((uint32_t)q1 << 4));
    }
  }
}

// ------------------------------------------------------------------ argmax

// Key of row m: the value (non-finite -> -1e30, -0 -> +0) mapped to bits that
// order as the floats do, above 0xFFFFFFFF - m, so the largest key is the
// largest value and, among equal values, the smallest row.
__device__ __forceinline__ unsigned long long argmax_key(float v, int m) {
  if (!isfinite(v)) v = -1e30f;
  if (v == 0.f) v = 0.f;
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)m);
}

__global__ void __launch_bounds__(256) k_argmax_rows(const float* __restrict__ y, int M,
                                                     unsigned long long* key) {
  unsigned long long best = 0;
  for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x)
    best = max(best, argmax_key(__ldg(y + m), m));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ unsigned long long wbest[8];
  if ((threadIdx.x & 31) == 0) wbest[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) best = max(best, wbest[w]);
    atomicMax(key, best);
  }
}

cudaError_t launch_argmax_rows(const float* y, int M, unsigned long long* key, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(key, 0, sizeof(unsigned long long), st);
  if (e != cudaSuccess || M <= 0) return e;
  k_argmax_rows<<<std::min(148 * 4, (M + 255) / 256), 256, 0, st>>>(y, M, key);
  return cudaGetLastError();
}

// -------------------------------------------------------------- launchers

static int grid_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  if (b > 148u * 64u) b = 148u * 64u;
  return (int)(b ? b : 1);
}

cudaError_t launch_repack(const RepackArgs& a, cudaStream_t st) {
  const int Mt = (a.M + 15) / 16;
  const size_t n = (size_t)Mt * a.Kc * 128;
  k_repack<<<grid_for(n, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const ProjDev& P, int M, int K, int gs, int awq, int zp, float* out,
                           cudaStream_t st) {
  const int ng = (K + gs - 1) / gs, Kc = (K + 63) / 64;
  k_dequant<<<grid_for((size_t)M * K, 256), 256, 0, st>>>(P, M, K, gs, ng, Kc, awq, zp, out);
  return cudaGetLastError();
}

cudaError_t launch_gemm(int mode, int path, const GemmArgs& a, int max_work, int awq,
                        int ntiles, cudaStream_t st, int n_groups, int grid_items) {
  if (max_work <= 0) return cudaSuccess;
  const int Mt = (a.M + 15) / 16;
  dim3 grid((Mt + 3) / 4, max_work);
  if (path == 0) {
    // the K-split kernel walks the work list grid-stride: its grid covers the
    // expected items, not the work list's capacity bound
    const int gy = grid_items > 0 ? std::min(max_work, grid_items) : max_work;
    // K split: enough warps to cover the SMs when the expected work is small
    const long units = (long)Mt * gy;
    const long units_est = (long)Mt * std::min(max_work, n_groups > 0 ? n_groups : max_work);
    const int nsteps = a.K / 128;
    const int ks = nsteps >= 8 && units < 148 * 16 ? 4 : (nsteps >= 8 ? 2 : 1);
    // decode-size items: the persistent kernel when the expected units (items ~
    // min(max_work, distinct experts) x row tiles) keep 1.5x its resident warps
    // busy; below that the K-split launch has more warps in flight
    // the fp16 activation path: gate/up with launch_prep_xh's rows and sums
    const bool xh = mode == MODE_GATE_UP && a.bsum != nullptr;
    if (ntiles <= 1 && a.ctr && nsteps >= kStagesW - 1 &&
        2L * units_est >= 3L * mma_p_resident_warps(mode == MODE_GATE_UP, a.gs, awq, xh)) {
      if (xh)
        launch_mma_p<MODE_GATE_UP, true>(a, awq, st);
      else if (mode == MODE_GATE_UP)
        launch_mma_p<MODE_GATE_UP, false>(a, awq, st);
      else
        launch_mma_p<MODE_PLAIN_F32, false>(a, awq, st);
    } else if (ntiles > 1) {
      return cudaErrorInvalidValue;  // items above 8 rows: not this kernel's
    } else if (xh) {
      launch_mma<MODE_GATE_UP, true>(a, gy, ks, awq, st);
    } else if (mode == MODE_GATE_UP) {
      launch_mma<MODE_GATE_UP, false>(a, gy, ks, awq, st);
    } else {
      launch_mma<MODE_PLAIN_F32, false>(a, gy, ks, awq, st);
    }
  } else if (path == 1) {
    if (mode == MODE_GATE_UP)
      k_int4_cc<MODE_GATE_UP, float, 4><<<grid, 128, 0, st>>>(a, awq);
    else
      k_int4_cc<MODE_PLAIN_F32, float, 4><<<grid, 128, 0, st>>>(a, awq);
  } else {
    if (mode == MODE_GATE_UP)
      k_int4_cc<MODE_GATE_UP, __nv_bfloat16, 4><<<grid, 128, 0, st>>>(a, awq);
    else
      k_int4_cc<MODE_PLAIN_F32, __nv_bfloat16, 4><<<grid, 128, 0, st>>>(a, awq);
  }
  return cudaGetLastError();
}

// Expert-parallel combine at the token's source rank: the routed slots' rows
// come back from their owners as bf16 in the dispatch order (ret[inverse[t *
// topk + j]]), the shared expert's fp32 row is computed locally (sh[sh_inv[t]]);
// the same fmaf order as k_combine (routed j = 0..topk-1, then the shared slot).
__global__ void k_combine_ep(const __nv_bfloat16* __restrict__ ret, const int* __restrict__ inverse,
                             const float* __restrict__ w, int T, int topk, int H, const float* __restrict__ sh,
                             const int* __restrict__ sh_inv, float sh_scale, const float* __restrict__ sh_w,
                             __nv_bfloat16* __restrict__ y, FlagWait fw) {
  flag_wait_block(fw);  // every owner's return of this step has landed (bounded)
  const int t = blockIdx.y;
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (t >= T || h >= H) return;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < topk; ++j) {
    const float wj = w[(size_t)t * topk + j];
    const __nv_bfloat16* row = ret + (size_t)inverse[(size_t)t * topk + j] * H;
    for (int i = 0; i < 4 && h + i < H; ++i) acc[i] = __fmaf_rn(wj, __bfloat162float(row[h + i]), acc[i]);
  }
  if (sh) {  // sh_w: per-token weights of the shared expert (its sigmoid gate), else sh_scale
    const float* row = sh + (size_t)sh_inv[t] * H;
    const float ss = sh_w ? sh_w[t] : sh_scale;
    for (int i = 0; i < 4 && h + i < H; ++i) acc[i] = __fmaf_rn(ss, row[h + i], acc[i]);
  }
  for (int i = 0; i < 4 && h + i < H; ++i) y[(size_t)t * H + h + i] = __float2bfloat16_rn(acc[i]);
}

cudaError_t launch_combine_ep(const void* ret, const int* inverse, const float* w, int T, int topk, int H,
                              const float* sh, const int* sh_inv, float sh_scale, const float* sh_w, void* y,
                              cudaStream_t st, const FlagWait& fw) {
  if (T <= 0) return cudaSuccess;
  const int threads = 128;
  dim3 grid(((H + 3) / 4 + threads - 1) / threads, T);
  k_combine_ep<<<grid, threads, 0, st>>>((const __nv_bfloat16*)ret, inverse, w, T, topk, H, sh, sh_inv, sh_scale,
                                         sh_w, (__nv_bfloat16*)y, fw);
  return cudaGetLastError();
}

cudaError_t launch_combine(const float* d, const int* inverse, const float* w, int T, int kk, int H,
                           void* y, int y_bf16, int skip_tiny, cudaStream_t st, const void* res) {
  if (T <= 0) return cudaSuccess;
  const int threads = 256;
  const int gx = ((H + 3) / 4 + threads - 1) / threads;
  // about 8 CTAs per SM in total; each walks its tokens two at a time
  const int gy = std::max(1, std::min((T + 1) / 2, (148 * 8 + gx - 1) / gx));
  const dim3 grid(gx, gy);
  if (y_bf16)
    return launch_pdl(k_combine<__nv_bfloat16>, grid, dim3(threads), 0, st, d, inverse, w, T, kk, H,
                      (__nv_bfloat16*)y, skip_tiny, (const __nv_bfloat16*)res);
  return launch_pdl(k_combine<float>, grid, dim3(threads), 0, st, d, inverse, w, T, kk, H, (float*)y, skip_tiny,
                    (const __nv_bfloat16*)res);
}

cudaError_t launch_quant_awq_sym(const __nv_bfloat16* W, int M, int K, int gs, int bf16_scale,
                                 uint8_t* q, __half* sc, cudaStream_t st) {
  const size_t n = (size_t)M * (K / gs);
  k_quant_awq_sym<<<grid_for(n, 128), 128, 0, st>>>(W, M, K, gs, bf16_scale, q, sc);
  return cudaGetLastError();
}

}  // namespace llmoc
