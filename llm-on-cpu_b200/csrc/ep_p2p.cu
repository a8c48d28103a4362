// ep_p2p.cu — expert-parallel token transport over NVLink peer memory.
//
// The all-to-all of the expert-parallel layer step (ICollective::alltoall,
// src/contracts/collective.h:13, which the reference only declares) done by
// the ranks' own kernels: every rank stores its routed rows directly into the
// owners' receive buffers (peer pointers opened with CUDA IPC; plain stores
// over NVLink, no multicast, no TMA from peer memory), raises a per-source
// sequence flag there, and the owners push the expert outputs back the same
// way.  No host synchronisation and no library collective is on the path.
//
// Buffer of one rank (one cudaMalloc, exported by CUDA IPC), for `world`
// ranks and `cap` rows per source (a source sends at most max_tokens * topk
// rows in total, so cap = that bound):
//   flags     [2 kinds][world] u32   kind 0: dispatch of source s has landed
//                                    kind 1: return of owner s has landed
//   meta      [2 parities][world] {count, offset}: rows from source s and
//             their offset in s's send order (the return goes there)
//   recv_ids  [2 parities][world][cap] i32   owner-local expert of each row
//   recv_rows [2 parities][world][cap][hidden] bf16
//   ret_rows  [2 parities][cap][hidden] bf16  outputs of this rank's rows,
//             in its send order
// Parity = step & 1.  Double buffering is enough without further flow
// control: a rank reaches step s + 2 only after its step s + 1 combine, which
// waited for every owner's step s + 1 return, which each owner pushed after
// finishing step s + 1's (and so step s's) use of its receive parity.
//
// Flags carry the step number (1, 2, ...): written with st.release.sys after
// all the step's rows of that peer are in place, read with ld.acquire.sys.
// A wait gives up after its budget of SM clocks (default 2^31, ~1 s; set per
// transport), sets bit 1 of the
// transport's error word and returns: outputs of that step are invalid, the
// host checks the word, and no GPU is left waiting.
#include "kernels.cuh"

namespace llmoc {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* flag_at(char* base, const EpP2PLayout& L, int kind, int src) {
  return reinterpret_cast<uint32_t*>(base + L.flags) + kind * L.world + src;
}
__device__ __forceinline__ int2* meta_at(char* base, const EpP2PLayout& L, int parity, int src) {
  return reinterpret_cast<int2*>(base + L.meta) + parity * L.world + src;
}
__device__ __forceinline__ int* ids_at(char* base, const EpP2PLayout& L, int parity, int src) {
  return reinterpret_cast<int*>(base + L.recv_ids) + ((size_t)parity * L.world + src) * L.cap;
}
__device__ __forceinline__ uint4* rows_at(char* base, const EpP2PLayout& L, int parity, int src) {
  return reinterpret_cast<uint4*>(base + L.recv_rows + ((size_t)parity * L.world + src) * L.cap * L.row_bytes);
}
__device__ __forceinline__ uint4* ret_at(char* base, const EpP2PLayout& L, int parity) {
  return reinterpret_cast<uint4*>(base + L.ret_rows + (size_t)parity * L.cap * L.row_bytes);
}

// Last CTA of a push grid: every other CTA fenced its stores (system scope)
// before counting itself, so once the count is complete all rows are visible.
__device__ __forceinline__ bool last_cta(int* ctr) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(ctr, 1);
    last = prev == (int)gridDim.x - 1;
    if (last) *ctr = 0;  // ready for the next push (no other CTA touches it now)
  }
  __syncthreads();
  return last != 0;
}

// Copies one row of L.row_bytes (a multiple of 16) with a warp.
__device__ __forceinline__ void copy_row(uint4* dst, const uint4* src, int n16, int lane) {
  for (int c = lane; c < n16; c += 32) dst[c] = src[c];
}

}  // namespace

// Source side: rows of send order q (grouped by owner: counts[d] rows for
// owner d, owners ascending) go to owner d's receive slot q - off[d] of this
// rank's region; then each owner's meta and flag.  A row comes from
// send_rows[q], or (sorted non-null) straight from the token's row
// X[sorted[q] / kk], which spares the gathered copy and its launch.
__global__ void __launch_bounds__(256) k_ep_push_dispatch(EpP2PLayout L, char* const* peers,
                                                          const uint4* __restrict__ send_rows,
                                                          const int* __restrict__ send_expert,
                                                          const int* __restrict__ counts, int rank, uint32_t seq,
                                                          int* ctr, const uint4* __restrict__ X,
                                                          const int* __restrict__ sorted, int kk) {
  __shared__ int off[kEpMaxWorld + 1];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int d = 0; d < L.world; ++d) {
      off[d] = o;
      o += counts[d];
    }
    off[L.world] = o;
  }
  __syncthreads();
  const int parity = seq & 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int n16 = L.row_bytes / 16;
  for (int q = blockIdx.x * nw + warp; q < off[L.world]; q += gridDim.x * nw) {
    int d = 0;
    while (q >= off[d + 1]) ++d;
    const int i = q - off[d];
    char* pb = peers[d];
    const uint4* src = sorted ? X + (size_t)(sorted[q] / kk) * n16 : send_rows + (size_t)q * n16;
    copy_row(rows_at(pb, L, parity, rank) + (size_t)i * n16, src, n16, lane);
    if (lane == 0) ids_at(pb, L, parity, rank)[i] = send_expert[q];
  }
  if (!last_cta(ctr)) return;
  for (int d = threadIdx.x; d < L.world; d += blockDim.x)
    *meta_at(peers[d], L, parity, rank) = make_int2(off[d + 1] - off[d], off[d]);
  __threadfence_system();
  __syncthreads();
  for (int d = threadIdx.x; d < L.world; d += blockDim.x) st_release_sys(flag_at(peers[d], L, 0, rank), seq);
}

// Waits for every peer's flag of `kind` to reach seq (one thread per peer,
// bounded).  The permutation that follows a dispatch wait reads only each
// source's first meta.x slots, so the slots past a count are never read.
__global__ void __launch_bounds__(256) k_ep_wait(EpP2PLayout L, char* base, int kind, uint32_t seq, int* err,
                                                 long long budget) {
  __shared__ int timed_out;
  if (threadIdx.x == 0) timed_out = 0;
  __syncthreads();
  if (threadIdx.x < L.world) {
    const uint32_t* f = flag_at(base, L, kind, threadIdx.x);
    const long long t0 = clock64();
    while ((int)(ld_acquire_sys(f) - seq) < 0) {
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

// Owner side: the down GEMM's fp32 output rows (in expert-sorted order;
// inverse[q] = row of receive slot q) rounded to bf16 and stored straight into
// each source's return buffer at its send offsets; then each source's flag.
__global__ void __launch_bounds__(256) k_ep_push_return(EpP2PLayout L, char* const* peers, char* base,
                                                        const float* __restrict__ partial,
                                                        const int* __restrict__ inverse, int rank, uint32_t seq,
                                                        int* ctr) {
  const int parity = seq & 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int n16 = L.row_bytes / 16, H = L.row_bytes / 2;
  for (int q = blockIdx.x * nw + warp; q < L.world * L.cap; q += gridDim.x * nw) {
    const int s = q / L.cap, i = q % L.cap;
    const int2 m = *meta_at(base, L, parity, s);
    // a source's rows: count m.x at offset m.y of its send order (both within
    // cap unless a wait gave up; then nothing of this step is pushed outside)
    if (i >= m.x || m.x > L.cap || m.y < 0 || m.y + m.x > L.cap) continue;
    const int src = inverse[q];
    if (src < 0) continue;
    const float4* row = reinterpret_cast<const float4*>(partial + (size_t)src * H);
    uint4* dst = ret_at(peers[s], L, parity) + (size_t)(m.y + i) * n16;
    for (int c = lane; c < n16; c += 32) {  // 8 values per 16-byte store
      const float4 a = row[2 * c], b = row[2 * c + 1];
      const __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
      const __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
      uint4 v;
      v.x = *reinterpret_cast<const uint32_t*>(&p0);
      v.y = *reinterpret_cast<const uint32_t*>(&p1);
      v.z = *reinterpret_cast<const uint32_t*>(&p2);
      v.w = *reinterpret_cast<const uint32_t*>(&p3);
      dst[c] = v;
    }
  }
  if (!last_cta(ctr)) return;
  __threadfence_system();
  for (int s = threadIdx.x; s < L.world; s += blockDim.x) st_release_sys(flag_at(peers[s], L, 1, rank), seq);
}

// The transport's kernels are launched in plain stream order (no programmatic
// early launch): a wait kernel must never start before the push it follows.
cudaError_t launch_ep_push_dispatch(const EpP2PLayout& L, char* const* peers, const void* send_rows,
                                    const int* send_expert, const int* counts, int rank, uint32_t seq, int* ctr,
                                    cudaStream_t st, const void* X, const int* sorted, int kk) {
  k_ep_push_dispatch<<<kEpPushCtas, 256, 0, st>>>(L, peers, reinterpret_cast<const uint4*>(send_rows), send_expert,
                                                   counts, rank, seq, ctr, reinterpret_cast<const uint4*>(X), sorted,
                                                   kk);
  return cudaGetLastError();
}
cudaError_t launch_ep_wait(const EpP2PLayout& L, char* base, int kind, uint32_t seq, int* err, long long budget,
                           cudaStream_t st) {
  k_ep_wait<<<1, 256, 0, st>>>(L, base, kind, seq, err, budget);
  return cudaGetLastError();
}
cudaError_t launch_ep_push_return(const EpP2PLayout& L, char* const* peers, char* base, const float* partial,
                                  const int* inverse, int rank, uint32_t seq, int* ctr, cudaStream_t st) {
  k_ep_push_return<<<kEpPushCtas, 256, 0, st>>>(L, peers, base, partial, inverse, rank, seq, ctr);
  return cudaGetLastError();
}

}  // namespace llmoc
