// int4_umma.cu — grouped INT4 GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulator in TMEM) for prefill-size work items.
//
// One CTA computes a 128-row tile of one projection (two, gate and up, in
// MODE_GATE_UP) for one work item (one expert, up to 128 of its tokens):
//     D[m, n] = sum_k W[m, k] * X[n, k]
// with K walked in 64-wide blocks through a kStages-deep shared-memory ring.
//
//   warps 1..4  producers.  A kLoad-deep load ring receives, by cp.async, the
//               raw INT4 fragment words (each lane copies exactly the words it
//               will dequantise), their group scales (and zeros), and the
//               block's slice of the item's activation rows, gathered into the
//               128-byte-swizzled K-major layout the MMA reads; loads run
//               kAhead blocks ahead and reuse the slot of block kb - 2, so a
//               producer never waits for the MMA it has just fed.  Each
//               block's words are then dequantised (w = (q - zp) * s, or
//               q * s + z, rounded once to bf16) into a kASlots-deep A ring in
//               the same swizzled layout; then fence.proxy.async and arrive on
//               full[a].
//   warp 0      allocates TMEM; lane 0 waits full[a], issues the four K=16
//               tcgen05.mma per projection (M = 128, N = rows rounded up to 16),
//               and tcgen05.commit's both the A slot (emptyA) and the load slot
//               (emptyL) back to the producers; a final commit signals `done`.
//   warps 1..4  epilogue: tcgen05.ld the accumulators (warp w reads TMEM
//               lanes 32*(w%4)..+31 = rows), SiLU*mul (gate/up) or fp32 (down),
//               store to the expert-sorted output rows.
//
// Every mbarrier wait is bounded (~1 s of %globaltimer); on timeout the
// kernel sets bit 0 of *err, stops waiting, and still frees its TMEM.
// No TMA multicast is used anywhere.
#include "kernels.cuh"

namespace llmoc {

namespace {

constexpr int kLoad = 4;                   // load-ring depth (raw words, scales, activations)
constexpr int kAhead = kLoad - 2;          // blocks the loads run ahead (one MMA of slack)
constexpr int kASlots = 3;                 // dequantised-A ring depth
constexpr int kUProd = 4;                  // producer / epilogue warps
constexpr int kUThreads = (1 + kUProd) * 32;
constexpr int kTileA = 128 * 128;          // 128 rows x 64 bf16 (one swizzle atom wide)
constexpr int kTileB = 128 * 128;          // up to 128 token rows x 64 bf16
constexpr int kRawQ = 128 * 32;            // 128 rows x 64 nibbles (fragment order)
constexpr int kRawS = 8 * 128;             // scales: 8 sub-tiles x up to 4 groups x 32 B
constexpr uint64_t kUWaitNs = 1000000000ull;

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
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
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t par) {
  if (mb_try(b, par)) return true;
  const uint64_t t0 = gns();
  while (!mb_try(b, par))
    if (gns() - t0 > kUWaitNs) return false;
  return true;
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
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
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   su32(bar))
               : "memory");
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
__device__ __forceinline__ const ProjDev& pick(const ExpertDev& e, int p) {
  return p == 0 ? e.gate : (p == 1 ? e.up : e.down);
}
__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.f + expf(-g))) * u; }

// byte offset of element (row, k) (k a multiple of 4 here) in a SW128 K-major tile
__device__ __forceinline__ uint32_t swz(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7))) << 4) + ((k & 7) << 1));
}

}  // namespace

// Shared-memory plan (bytes), per projection count NP:
//   A ring   kASlots x NP x kTileA        dequantised weights (swizzled)
//   load     kLoad x [B kTileB | raw q NP x kRawQ | scales NP x kRawS | zeros NP x kRawS]
template <int NP, bool AWQ>
struct USmem {
  static constexpr int kA = kASlots * NP * kTileA;
  static constexpr int kOffQ = kTileB;
  static constexpr int kOffS = kOffQ + NP * kRawQ;
  static constexpr int kOffZ = kOffS + NP * kRawS;
  static constexpr int kLoadSlot = kOffZ + (AWQ ? 0 : NP * kRawS);  // multiple of 1024
  static constexpr int kBytes = kA + kLoad * kLoadSlot;
};

// grid.x = ceil(M / 128), grid.y = work-list bound.  Work items hold <= 128 rows.
template <int MODE, int GSB, bool AWQ>
__global__ void __launch_bounds__(kUThreads, 1) k_int4_umma(GemmArgs a) {
  constexpr int NP = MODE == MODE_GATE_UP ? 2 : 1;
  constexpr int NG = GSB == 4 ? 1 : (GSB == 2 ? 1 : 2);  // groups per 64-wide block
  using SM = USmem<NP, AWQ>;
  extern __shared__ __align__(1024) unsigned char usm[];
  __shared__ __align__(8) uint64_t fullA[kASlots], emptyA[kASlots], emptyL[kLoad], done;
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((int)blockIdx.y >= *a.n_work) return;  // uniform over the CTA
  const WorkItem it = a.work[blockIdx.y];
  const ExpertDev& ex = a.experts[it.expert];
  const int m0 = blockIdx.x * 128;
  const int nb = a.K >> 6;                       // 64-wide K blocks
  const int N = (it.nrows + 15) & ~15;           // MMA N (multiple of 16 for M = 128)
  // 1024-byte aligned base (the swizzle pattern is tied to absolute address bits)
  unsigned char* base = usm + ((1024 - (su32(usm) & 1023)) & 1023);
  unsigned char* ringA = base;
  unsigned char* ringL = base + SM::kA;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kASlots; ++s) {
      mb_init(&fullA[s], kUProd);
      mb_init(&emptyA[s], 1);
    }
    for (int s = 0; s < kLoad; ++s) mb_init(&emptyL[s], 1);
    mb_init(&done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // TMEM: NP accumulators of 128 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(NP * 128));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      const uint32_t idesc = instr_desc(128, N);
      for (int kb = 0; kb < nb; ++kb) {
        const int sa = kb % kASlots, sl = kb % kLoad;
        if (!mb_wait(&fullA[sa], (kb / kASlots) & 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t ab = su32(ringA + sa * NP * kTileA);
        const uint32_t bb = su32(ringL + sl * SM::kLoadSlot);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t db = smem_desc(bb + kk * 32);
#pragma unroll
          for (int p = 0; p < NP; ++p)
            umma(tmem + p * 128, smem_desc(ab + p * kTileA + kk * 32), db, idesc, (kb | kk) != 0);
        }
        umma_commit(&emptyA[sa]);
        umma_commit(&emptyL[sl]);
      }
      umma_commit(&done);  // fires when every MMA issued above has completed
    }
    __syncwarp();
  } else {
    // --------------------------- producers (warps 1..4) ----------------------------
    const int pw = warp - 1;             // 0..3: sub-tiles 2pw, 2pw+1 (rows 32pw .. 32pw+31)
    const int ptid = threadIdx.x - 32;   // 0..127
    const int g = lane >> 2, t = lane & 3;
    const ProjDev* P[2] = {MODE == MODE_GATE_UP ? &ex.gate : &pick(ex, a.proj), &ex.up};
    const int Mt = (a.M + 15) >> 4;
    int rts[2];
    bool rv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rt = (m0 >> 4) + 2 * pw + h;
      rv[h] = rt < Mt;
      rts[h] = rv[h] ? rt : 0;
    }
    // activation pieces of this thread (8 per block): row n = piece / 8, chunk c = piece % 8
    const unsigned char* bsrc[8];
    uint32_t bdst[8];
    bool bok[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int piece = ptid + 128 * i;
      const int n = piece >> 3, c = piece & 7;
      bok[i] = n < it.nrows;
      const int pos = it.row0 + (bok[i] ? n : 0);
      const int row = a.gather ? a.gather[pos] / a.kk : pos;
      bsrc[i] = reinterpret_cast<const unsigned char*>(a.B) + ((size_t)row * a.ldb + c * 8) * 2;
      bdst[i] = (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4));
    }
    // scale pieces of this warp's two sub-tiles: per (p, h) NG groups x 32 B = 2*NG pieces
    const float zpf = AWQ ? (float)(128 + a.zp) : 128.f;
    const uint32_t zp2 = bf16x2_of(zpf);

    auto issue = [&](int kb) {  // block kb's loads into load slot kb % kLoad
      unsigned char* sl = ringL + (kb % kLoad) * SM::kLoadSlot;
      const uint32_t slu = su32(sl);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (bok[i]) cp16(slu + bdst[i], bsrc[i] + (size_t)kb * 128);
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (rv[h]) cp16(slu + SM::kOffQ + p * kRawQ + ((2 * pw + h) * 32 + lane) * 16,
                          P[p]->q + ((size_t)rts[h] * a.Kc + kb) * 32 + lane);
          // scales (and zeros) of the block's group(s): lanes 0 .. 2*NG-1
          const int grp0 = GSB == 4 ? (kb >> 1) : (GSB == 2 ? kb : kb * 2);
          if (rv[h] && lane < 2 * NG) {
            const size_t go = ((size_t)rts[h] * a.ng + grp0) * 16;
            const int so = p * kRawS + (2 * pw + h) * 128 + lane * 16;
            cp16(slu + SM::kOffS + so, reinterpret_cast<const unsigned char*>(P[p]->s + go) + lane * 16);
            if (!AWQ) cp16(slu + SM::kOffZ + so, reinterpret_cast<const unsigned char*>(P[p]->z + go) + lane * 16);
          }
        }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // prologue: blocks 0 .. kAhead-1 (their slots are fresh)
#pragma unroll
    for (int d = 0; d < kAhead; ++d) {
      if (d < nb) issue(d);
      else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int kb = 0; kb < nb && ok; ++kb) {
      // (1) loads for block kb + kAhead, once the MMA released its slot (block kb + kAhead - kLoad)
      const int kn = kb + kAhead;
      if (kn < nb) {
        if (kn >= kLoad && !mb_wait(&emptyL[kn % kLoad], ((kn / kLoad) - 1) & 1)) {
          ok = false;
          break;
        }
        issue(kn);
      } else {
        asm volatile("cp.async.commit_group;" ::: "memory");
      }
      // (2) block kb's own pieces have landed (this lane's words, scales, activations)
      asm volatile("cp.async.wait_group %0;" ::"n"(kAhead) : "memory");
      __syncwarp();  // scale pieces were copied by other lanes of this warp
      // (3) dequantise into A slot kb % kASlots once the MMA of block kb - kASlots is done
      const int sa = kb % kASlots;
      if (kb >= kASlots && !mb_wait(&emptyA[sa], ((kb / kASlots) - 1) & 1)) {
        ok = false;
        break;
      }
      const unsigned char* sl = ringL + (kb % kLoad) * SM::kLoadSlot;
      unsigned char* sA = ringA + sa * NP * kTileA;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 q4 = *reinterpret_cast<const uint4*>(sl + SM::kOffQ + p * kRawQ + ((2 * pw + h) * 32 + lane) * 16);
          const __half* sp = reinterpret_cast<const __half*>(sl + SM::kOffS + p * kRawS + (2 * pw + h) * 128);
          const __half* zq = reinterpret_cast<const __half*>(sl + SM::kOffZ + p * kRawS + (2 * pw + h) * 128);
          uint32_t sc[NG][2], zc[NG][2];
#pragma unroll
          for (int q = 0; q < NG; ++q) {
            sc[q][0] = bf16x2_of(__half2float(sp[q * 16 + g]));
            sc[q][1] = bf16x2_of(__half2float(sp[q * 16 + g + 8]));
            if (!AWQ) {
              zc[q][0] = bf16x2_of(__half2float(zq[q * 16 + g]));
              zc[q][1] = bf16x2_of(__half2float(zq[q * 16 + g + 8]));
            }
          }
          const uint32_t wds[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const int kbb = wi >> 1, kt = wi & 1;  // 32-wide half of the block, k16 step
            const int q = NG == 2 ? kbb : 0;
            const uint32_t w = wds[wi];
            uint32_t r[4];
            r[0] = lop3_and_or(w, 0x000F000Fu, 0x43004300u);        // row g,   k+0, k+1
            r[1] = lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u);   // row g+8, k+0, k+1
            r[2] = lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u);   // row g,   k+2, k+3
            r[3] = lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u);  // row g+8, k+2, k+3
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t qd = h2sub(r[j], zp2);  // exact: q - zp (or q)
              r[j] = AWQ ? h2mul(qd, sc[q][j & 1]) : h2fma(qd, sc[q][j & 1], zc[q][j & 1]);
            }
            const int row = (2 * pw + h) * 16 + g;  // row in the 128-row tile
            const int k = kbb * 32 + 8 * t + 4 * kt;
            *reinterpret_cast<uint2*>(sA + p * kTileA + swz(row, k)) = make_uint2(r[0], r[2]);
            *reinterpret_cast<uint2*>(sA + p * kTileA + swz(row + 8, k)) = make_uint2(r[1], r[3]);
          }
        }
      }
      // (4) publish A (generic writes) and B (cp.async writes) to the MMA proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mb_arrive(&fullA[sa]);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (!ok && lane == 0 && a.err) atomicOr(a.err, 1);

    // -------------------------------- epilogue --------------------------------
    if (!mb_wait(&done, 0)) {
      if (lane == 0 && a.err) atomicOr(a.err, 1);
    } else {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int quad = warp & 3;                 // TMEM lanes 32*quad .. +31
      const int m = m0 + quad * 32 + lane;       // output row of this thread
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
      for (int c0 = 0; c0 < N; c0 += 16) {
        float gv[16], uv[16];
        tmem_ld16(tl + c0, gv);
        if (MODE == MODE_GATE_UP) tmem_ld16(tl + 128 + c0, uv);
        if (m < a.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = c0 + j;
            if (n >= it.nrows) break;
            const size_t o = (size_t)(it.row0 + n) * a.ldo + m;
            float v = gv[j];
            if (!isfinite(v)) v = 0.f;
            if (MODE == MODE_GATE_UP) {
              float u = uv[j];
              if (!isfinite(u)) u = 0.f;
              reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(silu_mul(v, u));
            } else {
              reinterpret_cast<float*>(a.out)[o] = v;
            }
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NP * 128));
  }
  if (!ok && (threadIdx.x & 31) == 0 && a.err) atomicOr(a.err, 1);
}

template <int MODE, int GSB, bool AWQ>
static cudaError_t launch_u(const GemmArgs& a, int max_work, cudaStream_t st) {
  constexpr int NP = MODE == MODE_GATE_UP ? 2 : 1;
  const size_t smem = (size_t)USmem<NP, AWQ>::kBytes + 1024;
  cudaError_t e = cudaFuncSetAttribute(k_int4_umma<MODE, GSB, AWQ>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.M + 127) / 128, max_work);
  k_int4_umma<MODE, GSB, AWQ><<<grid, kUThreads, smem, st>>>(a);
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

cudaError_t launch_gemm_umma(int mode, const GemmArgs& a, int max_work, int awq, cudaStream_t st) {
  if (max_work <= 0) return cudaSuccess;
  if (mode == MODE_GATE_UP)
    return awq ? launch_u_gs<MODE_GATE_UP, true>(a, max_work, st)
               : launch_u_gs<MODE_GATE_UP, false>(a, max_work, st);
  return awq ? launch_u_gs<MODE_PLAIN_F32, true>(a, max_work, st)
             : launch_u_gs<MODE_PLAIN_F32, false>(a, max_work, st);
}

}  // namespace llmoc
