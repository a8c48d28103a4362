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
