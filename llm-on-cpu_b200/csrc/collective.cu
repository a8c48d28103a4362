// collective.cu — the ICollective contract (src/contracts/collective.h:9-15:
// world_size, allreduce_sum, alltoall, broadcast) over NVLink peer memory.
//
// The reference ships only stubs behind that contract (a host memcpy for
// alltoall, nothing for broadcast, an fp32 NCCL all-reduce; exec/
// mesh_nccl.cpp:85-134).  Here every rank holds one buffer, exported by CUDA
// IPC, and the ranks' own kernels move the data with plain stores into the
// peers' buffers (no multicast, no TMA from peer memory):
//
//   flags [world] u32   flags[s] = step of source s's data now in stage[.][s]
//   acks  [world] u32   acks[d]  = last step whose staged data rank d consumed
//   stage [2 parities][world][slot bytes]
//
// A collective call is two phases, each a pair of launches on the caller's
// stream:  start = wait until every rank has consumed step seq - 2 (the
// staging parity about to be rewritten), then push this rank's payload into
// the peers' stage[seq & 1][rank] and raise flags[rank] = seq there;
// finish = wait for every rank's flag, consume the staged data, then raise
// acks[rank] = seq at every peer.  Every rank raises its flag and ack at
// every peer on every step, whatever the operation, so the waits are the
// same for all of them.  Flags are written with st.release.sys after the
// step's stores (system fence), read with ld.acquire.sys; a wait gives up
// after its budget of SM clocks (default 2^31, ~1 s; set per collective),
// sets bit 1 of the error word and returns.
#include "kernels.cuh"

namespace llmoc {

namespace {

constexpr int kCollCtas = 148;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* word_at(char* base, size_t off, int i) {
  return reinterpret_cast<uint32_t*>(base + off) + i;
}
__device__ __forceinline__ char* stage_at(char* base, const CollLayout& L, int parity, int src) {
  return base + L.stage + ((size_t)parity * L.world + src) * L.slot;
}

// Last CTA of a grid: every CTA fenced its stores (system scope) before
// counting itself, so once the count is complete all of them are visible.
__device__ __forceinline__ bool last_cta(int* ctr) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(ctr, 1);
    last = prev == (int)gridDim.x - 1;
    if (last) *ctr = 0;
  }
  __syncthreads();
  return last != 0;
}

// Copies n bytes with the whole grid (item k of `items`): 16-byte words when
// both ends and n allow, bytes otherwise.
__device__ __forceinline__ void grid_copy(char* dst, const char* src, size_t n, int item, int items) {
  const size_t tid = ((size_t)item * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nthr = (size_t)items * gridDim.x * blockDim.x;
  if ((((uintptr_t)dst | (uintptr_t)src | n) & 15) == 0) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    const uint4* s = reinterpret_cast<const uint4*>(src);
    for (size_t i = tid; i < n / 16; i += nthr) d[i] = s[i];
  } else {
    for (size_t i = tid; i < n; i += nthr) dst[i] = src[i];
  }
}

}  // namespace

// Waits until every rank's word of `which` (0 flags, 1 acks) has reached
// `target` (one thread per rank, bounded).
__global__ void __launch_bounds__(256) k_coll_wait(CollLayout L, char* base, int which, uint32_t target, int* err,
                                                   long long budget) {
  __shared__ int timed_out;
  if (threadIdx.x == 0) timed_out = 0;
  __syncthreads();
  if (threadIdx.x < L.world) {
    const uint32_t* f = word_at(base, which ? L.acks : L.flags, threadIdx.x);
    const long long t0 = clock64();
    while ((int)(ld_acquire_sys(f) - target) < 0) {
      if (clock64() - t0 > budget) {
        timed_out = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (timed_out && threadIdx.x == 0) atomicOr(err, 2);
}

// This rank's payload into every destination's stage[parity][rank]: dest d
// gets src + d * src_stride (alltoall chunks) or src itself (stride 0);
// n = 0 pushes nothing (a non-root rank of a broadcast).  Then the flags.
__global__ void __launch_bounds__(256) k_coll_push(CollLayout L, char* const* peers, const char* src,
                                                   size_t src_stride, size_t n, int rank, uint32_t seq, int* ctr) {
  const int parity = seq & 1;
  for (int d = 0; d < L.world && n; ++d)
    grid_copy(stage_at(peers[d], L, parity, rank), src + (size_t)d * src_stride, n, 0, 1);
  if (!last_cta(ctr)) return;
  for (int d = threadIdx.x; d < L.world; d += blockDim.x) st_release_sys(word_at(peers[d], L.flags, rank), seq);
}

// Consumes the staged step: op 0 alltoall (dst chunk s <- stage[s], n bytes
// each), 1 allreduce_sum (dst[i] = sum over s in rank order of stage[s][i],
// fp32 accumulation; dtype 0 fp32, 1 bf16 rounded once), 2 broadcast (dst <-
// stage[root]).  Then the acks.
__global__ void __launch_bounds__(256) k_coll_consume(CollLayout L, char* base, char* const* peers, int op,
                                                      char* dst, size_t n, int dtype, int root, int rank,
                                                      uint32_t seq, int* ctr) {
  const int parity = seq & 1;
  if (op == 0) {
    for (int s = 0; s < L.world; ++s) grid_copy(dst + (size_t)s * n, stage_at(base, L, parity, s), n, 0, 1);
  } else if (op == 2) {
    grid_copy(dst, stage_at(base, L, parity, root), n, 0, 1);
  } else {
    const size_t esz = dtype ? 2 : 4, count = n / esz;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, nthr = (size_t)gridDim.x * blockDim.x;
    for (size_t i = tid; i < count; i += nthr) {
      float acc = 0.f;
      for (int s = 0; s < L.world; ++s) {
        const char* p = stage_at(base, L, parity, s);
        acc += dtype ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                     : reinterpret_cast<const float*>(p)[i];
      }
      if (dtype)
        reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(acc);
      else
        reinterpret_cast<float*>(dst)[i] = acc;
    }
  }
  if (!last_cta(ctr)) return;
  for (int d = threadIdx.x; d < L.world; d += blockDim.x) st_release_sys(word_at(peers[d], L.acks, rank), seq);
}

// Plain stream-order launches: a wait kernel must never start before the
// push or consume it follows.
cudaError_t launch_coll_wait(const CollLayout& L, char* base, int which, uint32_t target, int* err, long long budget,
                             cudaStream_t st) {
  k_coll_wait<<<1, 256, 0, st>>>(L, base, which, target, err, budget);
  return cudaGetLastError();
}
cudaError_t launch_coll_push(const CollLayout& L, char* const* peers, const void* src, size_t src_stride, size_t n,
                             int rank, uint32_t seq, int* ctr, cudaStream_t st) {
  k_coll_push<<<kCollCtas, 256, 0, st>>>(L, peers, static_cast<const char*>(src), src_stride, n, rank, seq, ctr);
  return cudaGetLastError();
}
cudaError_t launch_coll_consume(const CollLayout& L, char* base, char* const* peers, int op, void* dst, size_t n,
                                int dtype, int root, int rank, uint32_t seq, int* ctr, cudaStream_t st) {
  k_coll_consume<<<kCollCtas, 256, 0, st>>>(L, base, peers, op, static_cast<char*>(dst), n, dtype, root, rank, seq,
                                            ctr);
  return cudaGetLastError();
}

}  // namespace llmoc
