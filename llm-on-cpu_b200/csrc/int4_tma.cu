// int4_tma.cu — grouped INT4 GEMM for decode-size work items, fed by TMA.
//
// Same arithmetic as k_int4_mma (int4_gemm.cu): the tensor core multiplies
// the exact biased integers (128 + q) by bf16 activations, an all-ones MMA
// gives the per-token sums xs, and per group the fp32 partial is turned into
// the reference's sum_k x * (q - zp) * s (AWQ) or sum_k x * (q * s + z)
// (GPTQ), accumulated in fp32.
//
// Memory side: a CTA covers 4 consecutive 16-row tiles of one work item, one
// per consumer warp; all four walk the same 128-wide K steps with the same
// tokens.  A fifth, producer warp streams each step into a kStages-deep
// shared-memory ring with cp.async.bulk (the 1-D TMA; no multicast), one copy
// per lane in a single SIMT instruction: the fragment words of every (tile,
// projection) (1 KB each, contiguous in the repacked layout), their group
// scales (and zeros), and the step's slice of the item's activation rows
// (gathered, 256 B per row, shared by the four tiles).  Completion is tracked
// with mbarrier transaction counts; each consumer warp releases a stage with
// an mbarrier arrive.  Every wait is bounded (~1 s of %globaltimer): on
// timeout the kernel sets bit 0 of *err and stops waiting.
#include "kernels.cuh"

namespace llmoc {

namespace {

constexpr int kStages = 4;
constexpr int kCWarps = 4;                      // consumer warps = row tiles per CTA
constexpr int kBRow = 256 + 16;                 // padded activation row in smem (bytes)
// stage: weights [tile][proj] 1 KB | scales [tile][proj] 128 B | zeros | 8 activation rows
constexpr int kOffS = kCWarps * 2 * 1024;
constexpr int kOffZ = kOffS + kCWarps * 2 * 128;
constexpr int kOffB = kOffZ + kCWarps * 2 * 128;
constexpr int kStageBytes = kOffB + 8 * kBRow;
constexpr uint64_t kWaitNs = 1000000000ull;     // a bounded wait gives up after ~1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: true when the phase completed, false after ~kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitNs) return false;
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ void raw_word(uint32_t w, uint32_t a[4]) {
  a[0] = lop3_and_or(w, 0x000F000Fu, 0x43004300u);
  a[1] = lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u);
  a[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u);
  a[3] = lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u);
}
__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.f + expf(-g))) * u; }
__device__ __forceinline__ const ProjDev& pick(const ExpertDev& e, int p) {
  return p == 0 ? e.gate : (p == 1 ? e.up : e.down);
}

}  // namespace

// grid.x = ceil(Mt / 4), grid.y = work-list bound; block = 5 warps.
template <int MODE, int GSB, bool AWQ>
__global__ void __launch_bounds__((kCWarps + 1) * 32) k_int4_tma(GemmArgs a) {
  constexpr int NP = MODE == MODE_GATE_UP ? 2 : 1;
  constexpr int NG = GSB == 4 ? 1 : (GSB == 2 ? 2 : 4);  // groups per 128-wide step
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((int)blockIdx.y >= *a.n_work) return;  // uniform over the CTA
  const WorkItem it = a.work[blockIdx.y];
  const ExpertDev& ex = a.experts[it.expert];
  const int Mt = (a.M + 15) >> 4;
  const int rt0 = blockIdx.x * kCWarps;
  const int ntiles = min(kCWarps, Mt - rt0);
  const int nsteps = a.K >> 7;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kCWarps) {
    // ----------------------------- producer warp -----------------------------
    // lane roles: [0, 4*NP) weights of (tile, proj); [8, 8+4*NP) scales;
    // [16, 16+4*NP) zeros (GPTQ); [24, 32) activation rows
    const ProjDev* P[2] = {MODE == MODE_GATE_UP ? &ex.gate : &pick(ex, a.proj), &ex.up};
    const int nb = min(8, it.nrows);
    const int role = lane >> 3, idx = lane & 7;
    const int tile = idx / NP, proj = idx % NP;
    bool act = false;
    const unsigned char* src = nullptr;
    uint32_t dst_off = 0, size = 0;
    size_t step_stride = 0;  // bytes the source advances per step
    if (role < 3) {
      act = idx < kCWarps * NP && tile < ntiles && (role != 2 || !AWQ);
      if (act) {
        const int rt = rt0 + tile;
        if (role == 0) {
          src = reinterpret_cast<const unsigned char*>(P[proj]->q + (size_t)rt * a.Kc * 32);
          dst_off = (tile * 2 + proj) * 1024;
          size = 1024;
          step_stride = 1024;
        } else {
          const __half* base = role == 1 ? P[proj]->s : P[proj]->z;
          src = reinterpret_cast<const unsigned char*>(base + (size_t)rt * a.ng * 16);
          dst_off = (role == 1 ? kOffS : kOffZ) + (tile * 2 + proj) * 128;
          size = NG * 32;
          step_stride = (size_t)NG * 32;
        }
      }
    } else {
      act = idx < nb;
      if (act) {
        const int pos = it.row0 + idx;
        const int row = a.gather ? a.gather[pos] / a.kk : pos;
        src = reinterpret_cast<const unsigned char*>(a.B) + (size_t)row * a.ldb * 2;
        dst_off = kOffB + idx * kBRow;
        size = 256;
        step_stride = 256;
      }
    }
    const uint32_t bytes = (uint32_t)ntiles * NP * (1024u + NG * 32u * (AWQ ? 1u : 2u)) + nb * 256u;
    bool ok = true;
    for (int j = 0; j < nsteps; ++j) {
      const int st = j % kStages;
      if (lane == 0) {
        if (j >= kStages && !mbar_wait(&empty[st], ((j / kStages) - 1) & 1)) ok = false;
        if (ok) mbar_expect_tx(&full[st], bytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (act) bulk_g2s(smem + st * kStageBytes + dst_off, src + (size_t)j * step_stride, size, &full[st]);
    }
    if (!ok && lane == 0 && a.err) atomicOr(a.err, 1);
    return;
  }

  // ------------------------------ consumers --------------------------------
  const int g = lane >> 2, t = lane & 3;
  const int rt = rt0 + warp;
  const bool live = warp < ntiles;
  const float bias = AWQ ? (float)(128 + a.zp) : 128.f;
  const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};

  float acc[NP][4], tmp[NP][4], xs[4];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[p][r] = tmp[p][r] = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) xs[r] = 0.f;

  bool ok = true;
  for (int j = 0; j < nsteps; ++j) {
    const int st = j % kStages;
    if (!mbar_wait(&full[st], (j / kStages) & 1)) {
      ok = false;
      break;
    }
    const unsigned char* sb = smem + st * kStageBytes;
    uint4 wq[NP][2], bv[4];
    float sc[NP][NG][2], zz[NP][NG][2];
    if (live) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const unsigned char* wp = sb + (warp * 2 + p) * 1024 + piece_slot(lane) * 16;
        wq[p][0] = *reinterpret_cast<const uint4*>(wp);
        wq[p][1] = *reinterpret_cast<const uint4*>(wp + 512);
      }
#pragma unroll
      for (int b = 0; b < 4; ++b)
        bv[b] = *reinterpret_cast<const uint4*>(sb + kOffB + g * kBRow + b * 64 + t * 16);
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int q = 0; q < NG; ++q) {
          const __half* sp = reinterpret_cast<const __half*>(sb + kOffS + (warp * 2 + p) * 128) + q * 16;
          sc[p][q][0] = __half2float(sp[g]);
          sc[p][q][1] = __half2float(sp[g + 8]);
          if (!AWQ) {
            const __half* zp = reinterpret_cast<const __half*>(sb + kOffZ + (warp * 2 + p) * 128) + q * 16;
            zz[p][q][0] = __half2float(zp[g]);
            zz[p][q][1] = __half2float(zp[g + 8]);
          }
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // operands are in registers now
    if (!live) continue;

#pragma unroll
    for (int b = 0; b < 4; ++b) {
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
        const uint32_t b0 = kt ? bv[b].z : bv[b].x, b1 = kt ? bv[b].w : bv[b].y;
        mma_bf16(xs, ones, b0, b1);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const uint4& q4 = wq[p][b >> 1];
          const int wi = (b & 1) * 2 + kt;
          const uint32_t wd = wi == 0 ? q4.x : wi == 1 ? q4.y : wi == 2 ? q4.z : q4.w;
          uint32_t af[4];
          raw_word(wd, af);
          mma_bf16(tmp[p], af, b0, b1);
        }
      }
      if ((b + 1) % GSB == 0) {
        const int q = b / GSB;
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float v = __fmaf_rn(-bias, xs[r], tmp[p][r]);
            acc[p][r] = __fmaf_rn(v, sc[p][q][r >> 1], acc[p][r]);
            if (!AWQ) acc[p][r] = __fmaf_rn(zz[p][q][r >> 1], xs[r], acc[p][r]);
            tmp[p][r] = 0.f;
          }
#pragma unroll
        for (int r = 0; r < 4; ++r) xs[r] = 0.f;
      }
    }
  }
  if (!ok && lane == 0 && a.err) atomicOr(a.err, 1);
  if (!live || !ok) return;
  const int m0 = rt * 16 + g, m1 = m0 + 8;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int col = 2 * t + (r & 1);
    const int m = (r < 2) ? m0 : m1;
    if (col >= it.nrows || m >= a.M) continue;
    const size_t o = (size_t)(it.row0 + col) * a.ldo + m;
    float v = acc[0][r];
    if (!isfinite(v)) v = 0.f;
    if (MODE == MODE_GATE_UP) {
      float u = acc[NP - 1][r];
      if (!isfinite(u)) u = 0.f;
      reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(silu_mul(v, u));
    } else {
      reinterpret_cast<float*>(a.out)[o] = v;
    }
  }
}

template <int MODE, bool AWQ>
static cudaError_t launch_t(const GemmArgs& a, int max_work, cudaStream_t st) {
  const int Mt = (a.M + 15) / 16;
  const dim3 grid((Mt + kCWarps - 1) / kCWarps, max_work);
  const size_t smem = (size_t)kStages * kStageBytes;
  const int threads = (kCWarps + 1) * 32;
  cudaError_t e = cudaSuccess;
  switch (a.gs) {
    case 32:
      e = cudaFuncSetAttribute(k_int4_tma<MODE, 1, AWQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) k_int4_tma<MODE, 1, AWQ><<<grid, threads, smem, st>>>(a);
      break;
    case 64:
      e = cudaFuncSetAttribute(k_int4_tma<MODE, 2, AWQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) k_int4_tma<MODE, 2, AWQ><<<grid, threads, smem, st>>>(a);
      break;
    default:
      e = cudaFuncSetAttribute(k_int4_tma<MODE, 4, AWQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) k_int4_tma<MODE, 4, AWQ><<<grid, threads, smem, st>>>(a);
      break;
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_gemm_tma(int mode, const GemmArgs& a, int max_work, int awq, cudaStream_t st) {
  if (max_work <= 0) return cudaSuccess;
  if (mode == MODE_GATE_UP)
    return awq ? launch_t<MODE_GATE_UP, true>(a, max_work, st) : launch_t<MODE_GATE_UP, false>(a, max_work, st);
  return awq ? launch_t<MODE_PLAIN_F32, true>(a, max_work, st)
             : launch_t<MODE_PLAIN_F32, false>(a, max_work, st);
}

}  // namespace llmoc
