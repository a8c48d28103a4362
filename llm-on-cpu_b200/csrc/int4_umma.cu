// int4_umma.cu — grouped INT4 GEMM on the 5th-generation tensor cores
// (tcgen05.mma) for prefill-size work items.
//
// One CTA per SM, persistent over a list of tiles.  A tile is 128 weight rows
// of one expert against one work item (up to 128 of that expert's tokens):
//     D[m, n] = sum_k W[m, k] * X[n, k]
// MODE_GATE_UP tiles hold 64 gate rows and the same 64 up rows (interleaved
// by 16 so a gate row and its up row sit 16 TMEM lanes apart and meet with one
// shuffle in the SiLU*mul epilogue); MODE_PLAIN_F32 tiles hold 128 rows.
//
// The dequantised weights are the A operand and live in TENSOR MEMORY, not in
// shared memory: each dequantising thread owns one weight row (= one TMEM
// lane) and writes its bf16 values with tcgen05.st, so the only shared-memory
// traffic of the MMA is the activation tile (B).  Accumulators are double-
// buffered in TMEM so the epilogue of tile i overlaps the main loop of i+1.
//
//   TMEM (512 columns x 128 lanes, fp32 words)
//     [0,128) [128,256)   accumulator buffers (N <= 128 columns each)
//     [256 + 32 s, +32)   A slot s (s < kASlots): 128 rows x 64 k, bf16 pairs
//
//   warp 0      TMEM alloc; lane 0 issues tcgen05.mma (A from TMEM, B from a
//               128B-swizzled K-major smem tile) and tcgen05.commit's the A
//               slot, the load slot and, per tile, the accumulator buffer.
//   warp 1      weight loader: cp.async of the block's raw INT4 words (8 x 512
//               B fragment-order sub-tiles, stored XOR-swizzled so the row-per-
//               thread reads below are bank-conflict free) and group scales
//               (and GPTQ zeros); completion via cp.async.mbarrier.arrive.
//   warp 14     activation loader: cp.async gather of the item's token rows
//               (64 bf16 per row per block) into the swizzled B tile.
//   warps 2..9  dequantisers: two per TMEM lane quadrant, alternating blocks;
//               thread = one weight row: 16 words -> 64 bf16 w = (q - zp) * s
//               (or q * s + z), one tcgen05.st.32x32b.x32 per block.
//   warps 10..13 epilogue: tcgen05.ld the accumulator, SiLU*mul (gate/up,
//               bf16 out) or fp32 (down), store to the expert-sorted rows.
//
// Every wait is bounded (about 2^31 SM clocks, ~1 s); a wait that gives up
// sets a CTA-wide abort flag, bit 0 of *err, and every role drains and exits.
// TMEM is always freed.  No TMA multicast is used anywhere.
#include "kernels.cuh"

namespace llmoc {

namespace {

constexpr int kLoad = 8;                   // load-ring depth
constexpr int kASlots = 4;                 // A slots in TMEM
constexpr int kDeqWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kWarps = 3 + kDeqWarps + kEpiWarps;  // MMA, W loader, B loader
constexpr int kUThreads = kWarps * 32;             // 480
constexpr int kBLoaderWarp = 2 + kDeqWarps + kEpiWarps;  // 14
constexpr int kTmemCols = 512;
constexpr int kAccCol = 0;                 // + 128 * buffer
constexpr int kACol = 256;                 // + 32 * slot
// load slot: B tile (<= 128 token rows x 128 B) | raw words 8 x 512 B | scales | zeros
constexpr int kOffQ = 128 * 128;
constexpr int kOffS = kOffQ + 8 * 512;
constexpr int kOffZ = kOffS + 8 * 2 * 32;
constexpr int kSlot = kOffZ + 8 * 2 * 32;  // 21504, a multiple of 1024
constexpr int kUSmem = kLoad * kSlot + 1024;
constexpr long long kWaitCycles = 1ll << 31;

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mb_init(uint64_t* b, uint32_t c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(c) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mb_try(uint64_t* b, uint32_t par) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(par)
      : "memory");
  return ok != 0;
}
// Wait for phase parity `par`.  Gives up when the CTA's abort flag is set or
// after kWaitCycles (then sets the flag so every other role stops too).
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t par, volatile int* abort) {
  if (mb_try(b, par)) return true;
  const long long t0 = clock64();
  while (!mb_try(b, par)) {
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_arrive(uint64_t* b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(b)) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), Blackwell descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);        // start address
  d |= (uint64_t)1u << 16;                       // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;             // stride byte offset
  d |= (uint64_t)1u << 46;                       // version
  d |= (uint64_t)2u << 61;                       // SWIZZLE_128B
  return d;
}
// Instruction descriptor, kind::f16: fp32 D, bf16 A and B, both K-major.
__device__ __forceinline__ uint32_t instr_desc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[tmem] * B[smem]^T, M = 128, K = 16
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   su32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t r[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  const __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  x = __hsub2(x, y);
  return *reinterpret_cast<uint32_t*>(&x);
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  const __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  x = __hmul2(x, y);
  return *reinterpret_cast<uint32_t*>(&x);
}
__device__ __forceinline__ uint32_t h2fma(uint32_t a, uint32_t b, uint32_t c) {
  __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&a);
  const __nv_bfloat162 y = *reinterpret_cast<__nv_bfloat162*>(&b);
  const __nv_bfloat162 z = *reinterpret_cast<__nv_bfloat162*>(&c);
  x = __hfma2(x, y, z);
  return *reinterpret_cast<uint32_t*>(&x);
}
__device__ __forceinline__ uint32_t bf16x2_of(float f) {
  const __nv_bfloat16 h = __float2bfloat16_rn(f);
  const uint16_t u = *reinterpret_cast<const uint16_t*>(&h);
  return (uint32_t)u * 0x10001u;
}
__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.f + expf(-g))) * u; }

// Sub-tile st (16 rows) of a tile: which projection and which 16-row tile.
//   GATE_UP: st = 2q + gu  -> (gu ? up : gate), rows 64 mt + 16 q
//   PLAIN:   st            -> proj,             rows 128 mt + 16 st
template <int MODE>
__device__ __forceinline__ const ProjDev& sub_proj(const ExpertDev& e, int proj, int st) {
  if (MODE == MODE_GATE_UP) return (st & 1) ? e.up : e.gate;
  return proj == 0 ? e.gate : (proj == 1 ? e.up : e.down);
}
template <int MODE>
__device__ __forceinline__ int sub_rt(int mt, int st) {
  return MODE == MODE_GATE_UP ? mt * 4 + (st >> 1) : mt * 8 + st;
}

}  // namespace

template <int MODE, int GSB, bool AWQ>
__global__ void __launch_bounds__(kUThreads, 1) k_int4_umma(GemmArgs a) {
  constexpr int NG = GSB == 1 ? 2 : 1;  // scale groups per 64-wide block
  constexpr int kRowsTile = MODE == MODE_GATE_UP ? 64 : 128;
  extern __shared__ __align__(1024) unsigned char usm[];
  __shared__ __align__(8) uint64_t fullL[kLoad], emptyL[kLoad], fullA[kASlots], emptyA[kASlots];
  __shared__ __align__(8) uint64_t accFull[2], accEmpty[2], done;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nmt = a.M / kRowsTile;
  const int ntiles = *a.n_work * nmt;
  if ((int)blockIdx.x >= ntiles) return;  // uniform over the CTA
  const int nb = a.K >> 6;                // 64-wide K blocks per tile
  unsigned char* ring = usm + ((1024 - (su32(usm) & 1023)) & 1023);  // 1024-aligned (SW128)

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLoad; ++s) {
      mb_init(&fullL[s], 64);  // 32 lanes of each loader warp (cp.async arrive)
      mb_init(&emptyL[s], 1);
    }
    for (int s = 0; s < kASlots; ++s) {
      mb_init(&fullA[s], 4);   // the four dequantising warps of the block
      mb_init(&emptyA[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mb_init(&accFull[b], 1);
      mb_init(&accEmpty[b], kEpiWarps);
    }
    mb_init(&done, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      uint32_t j = 0, i = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++i) {
        const WorkItem it = a.work[tile / nmt];
        const uint32_t idesc = instr_desc(128, (it.nrows + 15) & ~15);
        const uint32_t b = i & 1;
        if (i >= 2 && !mb_wait(&accEmpty[b], ((i >> 1) - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem + kAccCol + 128 * b;
        for (int kb = 0; kb < nb; ++kb, ++j) {
          const uint32_t sa = j % kASlots, sl = j % kLoad;
          if (!mb_wait(&fullA[sa], (j / kASlots) & 1, &abort_flag) ||
              !mb_wait(&fullL[sl], (j / kLoad) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // cp.async data -> MMA
          tc_fence_after();
          const uint32_t bb = su32(ring + sl * kSlot);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_ts(dcol, tmem + kACol + 32 * sa + 8 * kk, smem_desc(bb + kk * 32), idesc, (kb | kk) != 0);
          umma_commit(&emptyA[sa]);
          umma_commit(&emptyL[sl]);
        }
        if (ok) umma_commit(&accFull[b]);
      }
      // every MMA issued above has completed once `done` fires
      umma_commit(&done);
      const long long t0 = clock64();
      while (!mb_try(&done, 0))
        if (clock64() - t0 > kWaitCycles) {
          ok = false;
          break;
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // --------------------------- weight loader -----------------------------------
    const int g = lane >> 2, t = lane & 3;
    const uint32_t qdst = kOffQ + g * 64 + (((t ^ (g >> 1)) & 3) << 4);
    const bool shas = lane < 16 * NG;         // lanes carrying one 16 B scale piece
    const int s_st = lane / (2 * NG), s_w = lane % (2 * NG);
    const uint32_t sdst = (s_st * NG + (s_w >> 1)) * 32 + (s_w & 1) * 16;
    uint32_t j = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int mt = tile % nmt;
      const ExpertDev& ex = a.experts[a.work[tile / nmt].expert];
      const uint4* qb[8];
#pragma unroll
      for (int st = 0; st < 8; ++st)
        qb[st] = sub_proj<MODE>(ex, a.proj, st).q + (size_t)sub_rt<MODE>(mt, st) * a.Kc * 32 + lane;
      const ProjDev& sp = sub_proj<MODE>(ex, a.proj, s_st);
      const size_t so = ((size_t)sub_rt<MODE>(mt, s_st) * a.ng + (s_w >> 1)) * 16 + (s_w & 1) * 8;
      const __half* sb = sp.s + so;
      const __half* zb = AWQ ? nullptr : sp.z + so;
      for (int kb = 0; kb < nb; ++kb, ++j) {
        const uint32_t sl = j % kLoad;
        if (j >= kLoad && !mb_wait(&emptyL[sl], ((j / kLoad) - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t base = su32(ring + sl * kSlot);
#pragma unroll
        for (int st = 0; st < 8; ++st) cp16(base + qdst + st * 512, qb[st] + (size_t)kb * 32);
        if (shas) {
          const int grp0 = GSB == 4 ? (kb >> 1) : (GSB == 2 ? kb : kb * 2);
          cp16(base + kOffS + sdst, sb + (size_t)grp0 * 16);
          if (!AWQ) cp16(base + kOffZ + sdst, zb + (size_t)grp0 * 16);
        }
        cp_arrive(&fullL[sl]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kBLoaderWarp) {
    // --------------------------- activation loader -------------------------------
    // lane: 16-byte chunk c of rows n0 + 4 i (i < 32) of the item
    const int c = lane & 7, n0 = lane >> 3;
    const uint32_t bd0 = n0 * 128 + ((c ^ n0) << 4);
    const uint32_t bd1 = (n0 + 4) * 128 + ((c ^ (n0 + 4)) << 4);
    const __nv_bfloat16* Bp = reinterpret_cast<const __nv_bfloat16*>(a.B);
    uint32_t j = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const WorkItem it = a.work[tile / nmt];
      uint32_t boff[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int n = n0 + 4 * i;
        const int pos = it.row0 + (n < it.nrows ? n : 0);
        const int row = a.gather ? a.gather[pos] / a.kk : pos;
        boff[i] = (uint32_t)row * (uint32_t)a.ldb + c * 8;
      }
      for (int kb = 0; kb < nb; ++kb, ++j) {
        const uint32_t sl = j % kLoad;
        if (j >= kLoad && !mb_wait(&emptyL[sl], ((j / kLoad) - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t base = su32(ring + sl * kSlot);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n0 + 4 * i < it.nrows)
            cp16(base + (i >> 1) * 1024 + ((i & 1) ? bd1 : bd0), Bp + boff[i] + (size_t)kb * 64);
        cp_arrive(&fullL[sl]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp < 2 + kDeqWarps) {
    // ------------------------------- dequantisers -------------------------------
    const int quad = warp & 3;                  // TMEM lanes 32 quad .. +31
    const uint32_t h = (warp - 2) >> 2;         // blocks j with j % 2 == h
    const int st = 2 * quad + (lane >> 4);      // sub-tile of this thread's row
    const int r16 = lane & 15, g = r16 & 7, hi = r16 >> 3;
    const uint32_t shift = 4 * hi;              // nibbles of row g+8 sit 4 bits higher
    uint32_t qsrc[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) qsrc[t] = kOffQ + st * 512 + g * 64 + (((t ^ (g >> 1)) & 3) << 4);
    const uint32_t ssrc = kOffS + st * NG * 32 + r16 * 2;
    const float zpf = AWQ ? (float)(128 + a.zp) : 128.f;
    const uint32_t zp2 = bf16x2_of(zpf);
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + kACol;
    uint32_t j = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nb; ++kb, ++j) {
        if ((j & 1) != h) continue;
        const uint32_t sl = j % kLoad, sa = j % kASlots;
        if (!mb_wait(&fullL[sl], (j / kLoad) & 1, &abort_flag) ||
            (j >= kASlots && !mb_wait(&emptyA[sa], ((j / kASlots) - 1) & 1, &abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const unsigned char* sb = ring + sl * kSlot;
        uint4 q4[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) q4[t] = *reinterpret_cast<const uint4*>(sb + qsrc[t]);
        uint32_t sc[NG], zc[NG];
#pragma unroll
        for (int q = 0; q < NG; ++q) {
          sc[q] = bf16x2_of(__half2float(*reinterpret_cast<const __half*>(sb + ssrc + q * 32)));
          if (!AWQ)
            zc[q] = bf16x2_of(__half2float(*reinterpret_cast<const __half*>(sb + ssrc + q * 32 + kOffZ - kOffS)));
        }
        uint32_t r[32];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t wds[4] = {q4[t].x, q4[t].y, q4[t].z, q4[t].w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            // word (kb2 = wi >> 1, kt = wi & 1) covers k = 32 kb2 + 8 t + 4 kt + {0..3}
            const int kb2 = wi >> 1, kt = wi & 1, q = NG == 2 ? kb2 : 0;
            const uint32_t v = wds[wi] >> shift;
            uint32_t p0 = lop3_and_or(v, 0x000F000Fu, 0x43004300u);       // k+0, k+1
            uint32_t p1 = lop3_and_or(v >> 8, 0x000F000Fu, 0x43004300u);  // k+2, k+3
            p0 = h2sub(p0, zp2);                                           // exact: q - zp (or q)
            p1 = h2sub(p1, zp2);
            if (AWQ) {
              p0 = h2mul(p0, sc[q]);
              p1 = h2mul(p1, sc[q]);
            } else {
              p0 = h2fma(p0, sc[q], zc[q]);
              p1 = h2fma(p1, sc[q], zc[q]);
            }
            const int col = kb2 * 16 + 4 * t + 2 * kt;  // TMEM column = k / 2
            r[col] = p0;
            r[col + 1] = p1;
          }
        }
        tmem_st32(tl + 32 * sa, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mb_arrive(&fullA[sa]);
      }
    }
  } else {
    // --------------------------------- epilogue ---------------------------------
    const int quad = warp & 3;
    const uint32_t tq = tmem + ((uint32_t)(quad * 32) << 16) + kAccCol;
    uint32_t i = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++i) {
      const WorkItem it = a.work[tile / nmt];
      const int mt = tile % nmt;
      const int N = (it.nrows + 15) & ~15;
      const uint32_t b = i & 1;
      if (!mb_wait(&accFull[b], (i >> 1) & 1, &abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ta = tq + 128 * b;
      for (int c0 = 0; c0 < N; c0 += 16) {
        float v[16];
        tmem_ld16(ta + c0, v);
        if (MODE == MODE_GATE_UP) {
          // lanes 0..15: gate rows, lanes 16..31: the same up rows; the pair
          // (c, c+1) is split: gate lane -> column c, up lane -> column c+1
          const int gu = lane >> 4;
          const int m = mt * 64 + quad * 16 + (lane & 15);
#pragma unroll
          for (int cc = 0; cc < 16; cc += 2) {
            const float send = gu ? v[cc] : v[cc + 1];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
            float gv = gu ? recv : v[cc];
            float uv = gu ? v[cc + 1] : recv;
            if (!isfinite(gv)) gv = 0.f;
            if (!isfinite(uv)) uv = 0.f;
            const int n = c0 + cc + gu;
            if (n < it.nrows)
              reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)(it.row0 + n) * a.ldo + m] =
                  __float2bfloat16_rn(silu_mul(gv, uv));
          }
        } else {
          const int m = mt * 128 + quad * 32 + lane;
#pragma unroll
          for (int cc = 0; cc < 16; ++cc) {
            const int n = c0 + cc;
            if (n < it.nrows) {
              const float x = v[cc];
              reinterpret_cast<float*>(a.out)[(size_t)(it.row0 + n) * a.ldo + m] = isfinite(x) ? x : 0.f;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mb_arrive(&accEmpty[b]);
    }
  }

  if (!ok && a.err) atomicOr(a.err, 1);
  tc_fence_before();
  __syncthreads();
  if (abort_flag && threadIdx.x == 0 && a.err) atomicOr(a.err, 1);
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

namespace {
int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}
}  // namespace

template <int MODE, int GSB, bool AWQ>
static cudaError_t launch_u(const GemmArgs& a, int max_work, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(k_int4_umma<MODE, GSB, AWQ>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kUSmem);
  if (e != cudaSuccess) return e;
  const int nmt = a.M / (MODE == MODE_GATE_UP ? 64 : 128);
  const long long tiles = (long long)max_work * nmt;
  const int grid = (int)std::min<long long>(tiles, sm_count());
  k_int4_umma<MODE, GSB, AWQ><<<grid, kUThreads, kUSmem, st>>>(a);
  return cudaGetLastError();
}

template <int MODE, bool AWQ>
static cudaError_t launch_u_gs(const GemmArgs& a, int max_work, cudaStream_t st) {
  switch (a.gs) {
    case 32: return launch_u<MODE, 1, AWQ>(a, max_work, st);
    case 64: return launch_u<MODE, 2, AWQ>(a, max_work, st);
    default: return launch_u<MODE, 4, AWQ>(a, max_work, st);
  }
}

// Requires M % 64 (gate/up) or M % 128 (down) == 0, K % 128 == 0, items of
// at most 128 rows, gs in {32, 64, 128}.
cudaError_t launch_gemm_umma(int mode, const GemmArgs& a, int max_work, int awq, cudaStream_t st) {
  if (max_work <= 0) return cudaSuccess;
  if (mode == MODE_GATE_UP)
    return awq ? launch_u_gs<MODE_GATE_UP, true>(a, max_work, st)
               : launch_u_gs<MODE_GATE_UP, false>(a, max_work, st);
  return awq ? launch_u_gs<MODE_PLAIN_F32, true>(a, max_work, st)
             : launch_u_gs<MODE_PLAIN_F32, false>(a, max_work, st);
}

}  // namespace llmoc
