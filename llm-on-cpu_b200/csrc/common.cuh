// common.cuh — shared device helpers and the device-side data structures of
// the INT4 MoE expert-FFN library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmoc {

// ---------------------------------------------------------------------------
// Repacked INT4 projection in HBM ("fragment order").
//
// A projection W[M,K] is stored as 16-row tiles.  Within a tile, K is cut
// into 64-wide chunks; each chunk is 512 contiguous bytes = 32 lanes x 16 B,
// so one warp-wide 128-bit load brings a whole 16x64 chunk.  Lane L
// (g = L>>2, t = L&3) owns four 32-bit words w[kb*2+kt] (kb = 32-wide block
// of the chunk, kt = 16-wide tensor-core k-step of the block).  The eight
// nibbles of a word are the A-fragment elements of mma.m16n8k16 for that
// lane, rows g and g+8 at actual k = chunk*64 + kb*32 + 8t + 4kt + {0..3}:
//     n0 = W[g][k+0]  n4 = W[g][k+1]  n2 = W[g][k+2]  n6 = W[g][k+3]
//     n1 = W[g+8][k+0] n5 = W[g+8][k+1] n3 = W[g+8][k+2] n7 = W[g+8][k+3]
// so lop3(w >> 4j, 0x000F000F, 0x43004300) yields A register j as a bf16
// pair (128+q_lo, 128+q_hi).  The matching B (activation) elements of lane t
// are 8 consecutive values x[kb*32 + 8t .. +7], one 16-byte load.
// Lane L's 16 bytes are STORED at slot piece_slot(L) = L ^ ((L >> 3) & 3) of
// the chunk (an involution): a warp still moves the whole 512-byte chunk, and
// a reader that gives each thread one weight row (threads g = 0..7 reading
// the pieces (g, t) of one t) touches eight different shared-memory bank
// quads when the chunk is copied verbatim into shared memory.
// Scales (and GPTQ zeros) are fp16, [M/16][ng][16] (tile, group, row).
// M is padded to a multiple of 16, K to a multiple of 64 (pad nibbles
// encode q = zp, i.e. weight 0, and pad scales are 0).
// ---------------------------------------------------------------------------
struct ProjDev {
  const uint4* q;       // [Mp/16][Kp/64][32] uint4
  const __half* s;      // [Mp/16][ng][16]
  const __half* z;      // GPTQ zeros, same layout, or nullptr
};

// One expert = gate [I,H], up [I,H], down [H,I].
struct ExpertDev {
  ProjDev gate, up, down;
};

// Work item of the grouped kernels: rows [row0, row0+nrows) of the sorted
// (expert-grouped) pair list, all belonging to `expert`.
struct WorkItem {
  int expert;
  int row0;
  int nrows;
  int pad;
};

__host__ __device__ __forceinline__ int piece_slot(int lane) { return lane ^ ((lane >> 3) & 3); }

constexpr int kChunkRows = 32;  // largest work item (tensor-core N = 4 x 8 rows)

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// fp16 activation row for the decode gate/up GEMM, by one warp (all 32 lanes
// call it): x = src (row r of the activations, bf16, H % 128 == 0; global
// memory read through the non-coherent path when GNC, else any generic
// address, e.g. a copy in shared memory) -> Xh[r] = x * 2^-e rounded to fp16,
// with e = (largest finite exponent of the row) - 141, so the row's largest
// finite |x| lands in [2^14, 2^15) and every scaling is exact (e >= -100; an
// all-zero row keeps e = 0); xsum[r][H/gs] = fp32 sums of each group of the
// fp16 values (each lane's 8 values in order, then a fixed xor-shuffle tree
// over the group's lanes); xscale[r] = 2^e.  A lane holds up to P 16-byte
// pieces of the row in registers, all requested at once; rows longer than
// 32 x P pieces are read twice.
__device__ __forceinline__ uint32_t bf16x2_max_exp(uint32_t w, uint32_t m) {
  const uint32_t e0 = (w >> 7) & 0xFFu, e1 = (w >> 23) & 0xFFu;
  if (e0 != 0xFFu) m = max(m, e0);  // non-finite values pick no scale
  if (e1 != 0xFFu) m = max(m, e1);
  return m;
}
template <int P, bool GNC>
__device__ __forceinline__ void prep_xh_row(const uint4* __restrict__ src, int r, int H, int gs, uint4* __restrict__ Xh,
                                            float* __restrict__ xsum, float* __restrict__ xscale, int lane) {
  constexpr int kPrepPieces = P;
  const int n8 = H / 8, ng = H / gs, lpg = gs / 8;  // 16-byte pieces, groups, lanes per group
  uint4* dst = Xh + (size_t)r * n8;
  const bool fits = n8 <= 32 * kPrepPieces;
  uint4 v[kPrepPieces];
  uint32_t mexp = 0;  // largest finite bf16 exponent field
  for (int b0 = 0; b0 < n8; b0 += 32 * kPrepPieces) {
#pragma unroll
    for (int j = 0; j < kPrepPieces; ++j) {
      const int i = b0 + lane + 32 * j;
      v[j] = i < n8 ? (GNC ? __ldg(src + i) : src[i]) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kPrepPieces; ++j) {
      mexp = bf16x2_max_exp(v[j].x, mexp);
      mexp = bf16x2_max_exp(v[j].y, mexp);
      mexp = bf16x2_max_exp(v[j].z, mexp);
      mexp = bf16x2_max_exp(v[j].w, mexp);
    }
  }
  mexp = __reduce_max_sync(0xffffffffu, mexp);
  const int e = mexp == 0 ? 0 : max(-100, (int)mexp - 141);
  const float down = __int_as_float((127 - e) << 23);  // 2^-e (-113 <= -e <= 100)
  for (int b0 = 0; b0 < n8; b0 += 32 * kPrepPieces) {
    if (!fits) {
#pragma unroll
      for (int j = 0; j < kPrepPieces; ++j) {
        const int i = b0 + lane + 32 * j;
        v[j] = i < n8 ? (GNC ? __ldg(src + i) : src[i]) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int j = 0; j < kPrepPieces; ++j) {
      const int i = b0 + lane + 32 * j;
      if (b0 + 32 * j >= n8) break;  // uniform over the warp
      const uint32_t wd[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      uint32_t o[4];
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 h2 = __floats2half2_rn(__uint_as_float(wd[q] << 16) * down,
                                             __uint_as_float(wd[q] & 0xFFFF0000u) * down);
        const float2 f2 = __half22float2(h2);
        s += f2.x;
        s += f2.y;
        o[q] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      if (i < n8) dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
      for (int off = 1; off < lpg; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (i < n8 && lane % lpg == 0) xsum[(size_t)r * ng + (i * 8) / gs] = s;
    }
  }
  if (lane == 0) xscale[r] = __int_as_float((127 + e) << 23);  // 2^e
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  The kernels of one forward are launched with
// launch_pdl, so a kernel's CTAs may start while its predecessor in the stream
// is still running.  Every such kernel calls grid_dep_wait() before it reads
// anything its predecessor wrote (the wait returns once the predecessor has
// completed and its memory is visible; it is a no-op for a normal launch),
// then grid_dep_release() to let its own successor launch.  A kernel may do
// independent work (e.g. fetch static weights of a work list that an earlier,
// already waited-for kernel produced) before waiting.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace llmoc
