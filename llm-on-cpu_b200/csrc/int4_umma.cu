// int4_umma.cu — grouped INT4 GEMM on the 5th-generation tensor cores
// (tcgen05.mma) for work items of tens to hundreds of rows.
//
// One CTA per SM, persistent over a list of tiles.  A tile is 128 weight rows
// of one expert against one work item (up to NMAX = 64 or 256 of that
// expert's tokens):
//     D[m, n] = sum_k W[m, k] * X[n, k]
// MODE_GATE_UP tiles hold 64 gate rows and the same 64 up rows (interleaved
// by 16 so a gate row and its up row sit 16 TMEM lanes apart and meet with one
// shuffle in the SiLU*mul epilogue); MODE_PLAIN_F32 tiles hold 128 rows.
//
// The dequantised weights are the A operand and live in TENSOR MEMORY, not in
// shared memory: each dequantising thread owns one weight row (= one TMEM
// lane) and writes its bf16 values with tcgen05.st, so the only shared-memory
// operand of the MMA is the activation tile (B).
//
// Issue cost sets the shape.  Measured on B200: an M = 128, K = 16 MMA costs
// the issuing thread about 100 SM cycles whatever its N (only N = 256, ~128
// cycles of math, keeps the tensor pipe busy from one thread), and an
// mbarrier wait about 190; MMAs issued by threads of different warps overlap
// (two issuing warps of N = 128 MMAs doubled the SM's rate, four of N = 64
// reached 1.4 PFLOP/s).  So the K blocks go in pairs (the A slots and B slots
// of two 64-wide blocks share one "full" barrier, on which the four
// dequantising warps arrive once per pair and the B loaders once per block, and one "empty"
// barrier, the MMA commit: one wait per eight MMAs), and a tile's pairs are
// dealt round-robin to up to kIssuers issuing warps, each summing into its
// own accumulator, as many as fit in TMEM next to the A slots.
//
//   TMEM (512 columns x 128 lanes, fp32 words), NMAX 256 / NMAX 64
//     [0, 384) / [0, 256)        accumulators: nis of N columns, single-buffered
//     [384 + 32 s) / [256 + 32 s) A slot s (s < kStages = 4 / 8): 128 rows x 64 k,
//                                 bf16 pairs
//
//   shared memory: the B slots (kStages x NMAX token rows x 128 B, 128-byte
//   swizzled K-major, one 64-wide K block each) and a weight ring (kWS slots of
//   kSlotBlocks K blocks: raw INT4 words + group scales (+ GPTQ zeros)).
//
//   warps 0..3   lane 0 issues tcgen05.mma (A from TMEM, B from smem) for its
//                pairs of each tile, commits each pair and, per tile, its
//                accumulator; warp 0 holds the TMEM allocation.
//   warps 4..5   weight loaders (alternate slot uses): one instruction per
//                slot whose lanes issue the 3-D TMA boxes of the raw words
//                (fragment-order 512-byte chunks, whose piece order makes the
//                row-per-thread reads below bank-conflict free), the scales
//                and the zeros, from per-expert tensor maps built at layer
//                creation.
//   warps 6..7   activation loaders (alternate blocks): one TMA 2-D box (64 bf16
//                x 32/64/128/256 token rows, 128-byte swizzle) of the item's
//                rows, which are contiguous: the down GEMM reads the
//                expert-sorted gate/up output, and the gate/up GEMM a copy of
//                the tokens gathered into expert-sorted order (k_gather_rows).
//   dequantisers: kDeqPerQuad per TMEM lane quadrant, taking block pairs in
//                turn; thread = one weight row: 16 words -> 64 bf16 w = (q -
//                zp) * s (or q * s + z), one tcgen05.st.32x32b.x32 per block.
//                A pair's weight-slot share is released as soon as its words
//                are in registers.
//   epilogue:    kEpiPerQuad per lane quadrant (a share of the columns each):
//                tcgen05.ld the tile's partial accumulators and add them in
//                issuer order, SiLU*mul (gate/up, bf16 out) or fp32 (down),
//                store to the expert-sorted rows.
//
// Every wait is bounded (about 2^31 SM clocks, ~1 s); a wait that gives up
// sets a CTA-wide abort flag, bit 0 of *err, and every role drains and exits.
// TMEM is always freed.  No TMA multicast is used anywhere.
#include <cstring>
#include <cuda.h>  // CUtensorMap and its encode enums (the encoder is reached through cudart)

#include "kernels.cuh"

namespace llmoc {

namespace {

// Stage ring: an A slot (TMEM) and a B slot (smem) per K block; the blocks go
// in pairs through one full and one empty barrier, so the MMA issuer waits
// once per 128 k (an mbarrier wait costs the issuing thread about as much as
// two of its MMAs).
// Pair pr (blocks 2 pr, 2 pr + 1) uses barriers full/empty[pr % kPairBars]:
// the slots of pair pr were last read by pair pr - kStages / 2, whose empty
// barrier a slot writer waits for.  With twice as many barriers as slot pairs
// a barrier is reused only every kStages pairs, and pair pr + kStages / 2
// cannot fill before pair pr is consumed (it rewrites pr's slots), so no
// parity wait can be two phases stale, whichever issuer consumes a pair.  The
// same reuse bounds the issuers' overlap to kStages / 2 pairs in flight.
//
// Two geometries (NMAX, the most rows an item holds):
//   NMAX 256  4 stages of 32 KB B slots; A slots in TMEM columns [384, 512),
//             accumulators below them;
//   NMAX 64   8 stages of 8 KB B slots; A slots in [256, 512), accumulators in
//             [0, 256).  Four slot pairs in flight let four issuers overlap.
template <int NMAX>
struct UCfg {
  static_assert(NMAX == 64 || NMAX == 256, "item geometries");
  static constexpr int kStages = NMAX == 64 ? 8 : 4;
  static constexpr int kPairBars = kStages;
  static constexpr int kBSlot = NMAX * 128;                 // NMAX token rows x 64 bf16
  static constexpr int kACol = 512 - 32 * kStages;          // A slot s at kACol + 32 s
  static constexpr int kAccCols = kACol;                    // accumulators in [0, kACol)
  static constexpr int kBoxKinds = NMAX == 64 ? 2 : 4;      // B boxes of 32 << kind rows
  static_assert(kStages % 2 == 0 && kAccCols >= NMAX, "stage pairs, one accumulator");
};
// Dequantising and epilogue warps per TMEM lane quadrant (20 warps in all).
//
// Why every parity wait is sound (a wait for the phase of pair pr on a barrier
// reused every R pairs passes early if the barrier has not yet completed the
// phase of pr - R, so that phase must be known complete).  Pairs may be
// consumed out of order, several issuers taking them; but both B loaders
// handle EVERY pair in order, each waiting for pair q - S consumed (S =
// kStages / 2 slot pairs) before loading pair q, so once any pair q is full,
// every pair <= q - S has been consumed (and its weight slot has landed).
// * A dequantising warp takes every kDeqPerQuad-th pair of the CTA's pair
//   sequence (counted over all its tiles); before its pair pr it passed the
//   A-slot wait of its previous pair pr - d (d = kDeqPerQuad), so pair pr - d
//   - S was full and every pair <= pr - d - 2S consumed.  Its A-slot wait (empty barrier of pair pr - S, reused every 2S
//   pairs) needs pr - 3S: kDeqPerQuad <= S.  Its weight-slot wait (slot = pair,
//   reused every kWS pairs) needs the slot of pr - kWS landed: kWS >=
//   kDeqPerQuad + 2S.
// * An issuer's previous wait on a full barrier was for its previous phase
//   (tile_issuers: nis divides kPairBars); at a tile start every earlier pair
//   has been consumed (accEmpty).
// * Each loader warp handles every other slot (weights) or every pair (B), so
//   its own previous wait covers the barrier's previous phase.
template <int NMAX>
struct URoles {
  static constexpr int kDeqPerQuad = NMAX == 64 ? 4 : 2;
  static constexpr int kEpiPerQuad = 5 - kDeqPerQuad;
  static constexpr int kDeqWarps = 4 * kDeqPerQuad;
  static constexpr int kEpiWarps = 4 * kEpiPerQuad;
  static constexpr int S = UCfg<NMAX>::kStages / 2;
  static_assert(kDeqPerQuad <= S, "dequantiser stride: at most S pairs");
};
// Warp roles.  TMA copies are latency-bound (~2.5k cycles from L2 whatever
// their size), so each instruction carries a large box and the rings are deep.
constexpr int kIssuers = 4;                // warps 0..3: lane 0 issues MMAs (warp 0 holds TMEM)
constexpr int kWLoaders = 2;               // warps 4, 5: weight slots u % 2
constexpr int kBLoaders = 2;               // warps 6, 7: B blocks j % 2
constexpr int kWLoader0 = kIssuers;
constexpr int kBLoader0 = kWLoader0 + kWLoaders;          // 6
constexpr int kDeq0 = kBLoader0 + kBLoaders;              // 8: the dequantisers (lane quadrants 0,1,2,3, ...)
constexpr int kWarps = kDeq0 + 20;                        // then the epilogue warps (URoles)
constexpr int kUThreads = kWarps * 32;                    // 896
constexpr int kTmemCols = 512;
constexpr int kBBoxKinds = 4;              // B tensor maps of 32, 64, 128, 256 rows
// A weight slot holds one K-block pair (kSlotBlocks = 2 64-wide blocks) of the
// tile's 128 rows, so slot u is pair u of the CTA's stage sequence (no tile
// ends in a partial slot: K % 128 == 0):
//   raw words  [op][tile][block][512 B]  (2 ops x 4 tiles for gate/up, 1 x 8 for down)
//   scales     [op][tile][group][32 B]   (groups of the slot's 128 k), then zeros (GPTQ)
// Each part arrives in ONE TMA box per op.
constexpr int kSlotBlocks = 2;
constexpr int kWRaw = 8 * kSlotBlocks * 512;              // 8 KB
constexpr int kWSc = 8 * (2 * kSlotBlocks) * 32;          // up to 2 kSlotBlocks groups per slot (gs 32)
constexpr int kWOffS = kWRaw;
constexpr int kWOffZ = kWRaw + kWSc;
// A weight slot's TMA boxes land ~3.5k SM cycles after they are issued and a
// slot is reissued only once all four lane quadrants have dequantised it.  The
// ring takes the shared memory the B ring leaves: 16 slots (pairs) beside the
// 64 KB B ring of NMAX 64, 8 beside the 128 KB of NMAX 256 (powers of two: the
// slot index is a mask), deep enough for the parity argument at URoles.
template <bool AWQ, int NMAX>
struct WRing {
  static constexpr int kSlot = kWRaw + kWSc * (AWQ ? 1 : 2);  // 9 / 10 KB
  static constexpr int kDepth = NMAX == 64 ? 16 : 8;
};
template <bool AWQ, int NMAX>
constexpr int umma_smem() {  // B ring + weight ring + alignment slack
  return UCfg<NMAX>::kStages * UCfg<NMAX>::kBSlot + WRing<AWQ, NMAX>::kDepth * WRing<AWQ, NMAX>::kSlot + 1024;
}
static_assert(umma_smem<false, 256>() <= 227 * 1024 && umma_smem<false, 64>() <= 227 * 1024, "shared memory");
static_assert((WRing<false, 64>::kDepth & (WRing<false, 64>::kDepth - 1)) == 0 &&
                  (WRing<false, 256>::kDepth & (WRing<false, 256>::kDepth - 1)) == 0,
              "weight ring depth: a power of two");
static_assert(WRing<false, 64>::kDepth >= URoles<64>::kDeqPerQuad + 2 * URoles<64>::S &&
                  WRing<false, 256>::kDepth >= URoles<256>::kDeqPerQuad + 2 * URoles<256>::S,
              "weight ring depth: covers a dequantiser's parity argument");
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
__device__ __forceinline__ void mb_arrive_n(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
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
// As mb_try, but a waiting thread is suspended (not spinning, so it takes no
// issue slots from the working warps) until the phase completes or about
// kSuspendNs have passed.
constexpr uint32_t kSuspendNs = 1000000;
__device__ __forceinline__ bool mb_try_sleep(uint64_t* b, uint32_t par) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(par), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Wait for phase parity `par`.  Gives up when the CTA's abort flag is set or
// after kWaitCycles (then sets the flag so every other role stops too).
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t par, volatile int* abort) {
  if (mb_try(b, par)) return true;
  const long long t0 = clock64();
  while (!mb_try_sleep(b, par)) {
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void mb_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
// global -> shared bulk copy on the TMA engine (no multicast); 16-byte aligned,
// size a multiple of 16; completes `bytes` of the barrier's transaction count
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}
// Before a loader exits: wait (bounded, whatever the abort flag says) until the
// copies it issued into the last `depth` uses of a ring have landed, so no
// asynchronous write reaches shared memory after the CTA is gone.
__device__ __forceinline__ void drain_ring(uint64_t* full, int depth, uint32_t issued, uint32_t first,
                                           uint32_t step) {
  // uses first, first + step, ... < issued; only the last `depth` can be in flight
  for (uint32_t u = first; u < issued; u += step) {
    if (u + depth < issued) continue;
    const long long t0 = clock64();
    while (!mb_try(&full[u % depth], (u / depth) & 1))
      if (clock64() - t0 > kWaitCycles) return;
  }
}
// TMA 2-D tile load (no multicast) of box (x, y) into a 1024-byte aligned
// destination; completes the box's bytes on the barrier
// L2 policy for data read exactly once (the weights): evicted first, so the
// streamed weights do not push the activation tiles (re-read by every M tile
// of an item) out of L2
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(su32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
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
// D[tmem] (+)= A[tmem] * B[smem]^T over one 64-wide K block: four M = 128,
// K = 16 MMAs in one asm statement.  A: columns ta, ta + 8, ta + 16, ta + 24
// (bf16 pairs); B: the descriptor db of the block's first 16 k, the next ones
// 32 bytes further (descriptor start address + 2).  `accumulate` = 0 starts a
// new sum with the first MMA.  The descriptor is built once per kernel and
// only offset here: rebuilding it per MMA costs more issue time than an
// M = 128, N = 128 MMA takes to run.
__device__ __forceinline__ void umma_ts_k64(uint32_t tmem_d, uint32_t ta, uint64_t db, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %6, %3, 1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %8, %3, 1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], %10, %3, 1;\n\t}\n" ::"r"(tmem_d),
      "r"(ta), "l"(db), "r"(idesc), "r"(accumulate), "r"(ta + 8), "l"(db + 2), "r"(ta + 16), "l"(db + 4),
      "r"(ta + 24), "l"(db + 6));
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
// 16 accumulator columns of this warp's lane quadrant: the load is issued by
// tmem_ld16_issue and its registers are valid after tmem_ld16_wait, which
// names them as operands so that no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  tmem_ld16_issue(taddr, r);
  tmem_ld16_wait(r);
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
// (128 + q_lo, 128 + q_hi) as a bf16 pair -> bf16 pair of q * s + z
__device__ __forceinline__ uint32_t gptq_pair(uint32_t v, float s, float z) {
  const float lo = __uint_as_float(v << 16) - 128.f, hi = __uint_as_float(v & 0xFFFF0000u) - 128.f;
  const __nv_bfloat162 r = __floats2bfloat162_rn(__fmaf_rn(lo, s, z), __fmaf_rn(hi, s, z));
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf16x2_of(float f) {
  const __nv_bfloat16 h = __float2bfloat16_rn(f);
  const uint16_t u = *reinterpret_cast<const uint16_t*>(&h);
  return (uint32_t)u * 0x10001u;
}
// SiLU(g) * u with the fast exponential and division (the epilogue of a
// 256-column tile computes 32K of them while the single accumulator waits;
// both approximations are a few ulp, far below the bf16 output's rounding)
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float e = __expf(-g);
  return g < -80.f ? 0.f : __fdividef(g, 1.f + e) * u;
}

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

// Issuers of a tile of N accumulator columns and np K-block pairs: the most
// of 4, 2, 1 (at most np) whose accumulators (each at a multiple of 32
// columns, `stride` apart) all fit below the A slots.  Issuer i takes the
// tile's pairs i, i + nis, ... into the accumulator at column i * stride; the
// epilogue adds the nis partial sums in issuer order.  nis divides kPairBars,
// so an issuer's previous wait on a full barrier was for that barrier's
// previous phase and a parity wait cannot be two phases stale.
template <int NMAX>
__device__ __forceinline__ int tile_issuers(int N, int np, int* stride) {
  static_assert(UCfg<NMAX>::kPairBars % kIssuers == 0, "issuers divide the pair barriers");
  int nis = kIssuers;
  while (nis > 1 && (nis > np || ((UCfg<NMAX>::kAccCols / nis) & ~31) < N)) nis >>= 1;
  *stride = (UCfg<NMAX>::kAccCols / nis) & ~31;
  return nis;
}

}  // namespace

// B operand tensor maps: boxes of 64 bf16 x {32, 64, 128, 256} token rows
// (128-byte swizzle); an item reads the smallest box that covers its rows.
struct BMaps {
  CUtensorMap m[kBBoxKinds];
};

template <int MODE, int GSB, bool AWQ, int NMAX>
__global__ void __launch_bounds__(kUThreads, 1) k_int4_umma(GemmArgs a, const __grid_constant__ BMaps tmB) {
  using C = UCfg<NMAX>;
  constexpr int kStages = C::kStages, kPairBars = C::kPairBars, kBSlot = C::kBSlot, kACol = C::kACol;
  constexpr int kDeqPerQuad = URoles<NMAX>::kDeqPerQuad, kEpiPerQuad = URoles<NMAX>::kEpiPerQuad;
  constexpr int kDeqWarps = URoles<NMAX>::kDeqWarps, kEpiWarps = URoles<NMAX>::kEpiWarps;
  constexpr int kEpi0 = kDeq0 + kDeqWarps;
  constexpr int NG = GSB == 1 ? 2 : 1;  // scale groups per 64-wide block
  constexpr int kRowsTile = MODE == MODE_GATE_UP ? 64 : 128;
  constexpr int kWS = WRing<AWQ, NMAX>::kDepth;
  constexpr int kWSlot = WRing<AWQ, NMAX>::kSlot;
  extern __shared__ __align__(1024) unsigned char usm[];
  __shared__ __align__(8) uint64_t fullW[kWS], emptyW[kWS];
  __shared__ __align__(8) uint64_t full[kPairBars], empty[kPairBars];
  __shared__ __align__(8) uint64_t accFull, accEmpty, done[kIssuers];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_dep_wait();
  grid_dep_release();
  const int nmt = a.M / kRowsTile;
  const int ntiles = *a.n_work * nmt;
  if ((int)blockIdx.x >= ntiles) return;  // uniform over the CTA
  const int nb = a.K >> 6;                // 64-wide K blocks per tile (even: K % 128 == 0)
  const int G = gridDim.x;
  const uint32_t my_tiles = (uint32_t)((ntiles - (int)blockIdx.x + G - 1) / G);
  const int nsl = (nb + kSlotBlocks - 1) / kSlotBlocks;  // weight-slot uses per tile
  constexpr int kGps = kSlotBlocks * 64 / (GSB * 32);      // scale groups per weight slot
  constexpr int kOps = MODE == MODE_GATE_UP ? 2 : 1;     // TMA boxes per part (gate, up)
  constexpr int kTilesOp = 8 / kOps;                     // 16-row tiles per box
  unsigned char* ringB = usm + ((1024 - (su32(usm) & 1023)) & 1023);  // 1024-aligned (SW128)
  unsigned char* ringW = ringB + kStages * kBSlot;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWS; ++s) {
      mb_init(&fullW[s], 1);           // weight loader's expect_tx (+ the bulk copies' bytes)
      mb_init(&emptyW[s], 4 * kSlotBlocks);  // one arrival per (lane quadrant, block) of the slot
    }
    for (int s = 0; s < kPairBars; ++s) {
      mb_init(&full[s], 6);  // per pair: 4 dequantising warps (one per lane quadrant) + the B loaders' 2 expect_tx
      mb_init(&empty[s], 1);  // MMA commit
    }
    mb_init(&accFull, kIssuers);  // every issuer, each tile (a commit, or an arrival if it has no pairs)
    mb_init(&accEmpty, kEpiWarps);
    for (int i = 0; i < kIssuers; ++i) mb_init(&done[i], 1);
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

  if (warp < kIssuers) {
    // ------------------------------- MMA issuers -------------------------------
    // Per pair of 64-wide K blocks: one wait (both A slots dequantised, both B
    // boxes landed), eight M = 128 MMAs of N = the item's rows rounded up to 16,
    // one commit that frees the pair's slots.  An MMA costs its issuing thread
    // about 100 cycles whatever its N, but issuers in different warps run
    // concurrently, so a tile's pairs are dealt round-robin to `nis` issuers
    // (tile_issuers), each summing into its own accumulator: small-N tiles are
    // issued up to four times faster.  The accumulators are single-buffered:
    // tile i starts once the epilogue has drained tile i - 1 (the loaders and
    // dequantisers keep filling the stage ring meanwhile).
    if (lane == 0) {
      const int me = warp;
      const int np = nb >> 1;
      uint32_t j = 0;  // block counter (stage ring), over all of this CTA's tiles
      const uint64_t dB0 = smem_desc(su32(ringB));
      int nrows = a.work[blockIdx.x / nmt].nrows;
      uint32_t i = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += G, ++i, j += nb) {
        const int nxt = tile + G < ntiles ? a.work[(tile + G) / nmt].nrows : 0;  // prefetch
        const int N = min(NMAX, (nrows + 15) & ~15);  // items hold at most NMAX rows (the permutation's chunk)
        int stride;
        const int nis = tile_issuers<NMAX>(N, np, &stride);
        const uint32_t idesc = instr_desc(128, N);
        const uint32_t dacc = tmem + (uint32_t)(me * stride);
        if (i >= 1 && !mb_wait(&accEmpty, (i - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (me >= nis) {  // no pairs of this tile: its MMAs of earlier tiles completed before accEmpty
          mb_arrive(&accFull);
          nrows = nxt;
          continue;
        }
        for (int pt = me; pt < np; pt += nis) {
          const uint32_t jj = j + 2 * pt, pr = jj >> 1, p = pr % kPairBars;
          if (!mb_wait(&full[p], (pr / kPairBars) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t s0 = jj % kStages, s1 = (jj + 1) % kStages;
          umma_ts_k64(dacc, tmem + kACol + 32 * s0, dB0 + ((s0 * kBSlot) >> 4), idesc, pt != me);
          umma_ts_k64(dacc, tmem + kACol + 32 * s1, dB0 + ((s1 * kBSlot) >> 4), idesc, 1);
          umma_commit(&empty[p]);
        }
        if (ok) umma_commit(&accFull);
        nrows = nxt;
      }
      // every MMA this thread issued has completed once its `done` fires
      umma_commit(&done[me]);
      const long long t0 = clock64();
      while (!mb_try(&done[me], 0))
        if (clock64() - t0 > kWaitCycles) {
          ok = false;
          break;
        }
    }
    __syncwarp();
  } else if (warp >= kWLoader0 && warp < kWLoader0 + kWLoaders) {
    // --------------------------- weight loaders -----------------------------------
    // warp kWLoader0 + w fills weight-slot uses u = w, w + kWLoaders, ...; per use
    // ONE instruction in which lane i < kOps * (AWQ ? 2 : 3) issues one 3-D TMA
    // box: raw words {128 words, kSlotBlocks chunks, kTilesOp tiles} of op
    // (gate/up), then its scales {16 rows, kGps groups, kTilesOp tiles}, then
    // its zeros
    constexpr uint32_t kWBytes = kWRaw + 256 * kGps * (AWQ ? 1 : 2);
    const uint32_t wl = warp - kWLoader0;
    const int part = lane / kOps, op = lane % kOps;  // part 0 raw, 1 scales, 2 zeros
    const bool active = part == 0 || part == 1 || (!AWQ && part == 2);
    const int proj = MODE == MODE_GATE_UP ? op : a.proj;  // gate, up / a.proj (down)
    const uint32_t dst_off = part == 0 ? op * (kWRaw / kOps)
                                       : (part == 1 ? kWOffS : kWOffZ) + op * (kTilesOp * kGps * 32);
    const int ystep = part == 0 ? kSlotBlocks : kGps;
    const CUtensorMap* maps = reinterpret_cast<const CUtensorMap*>(a.wmaps);
    const uint64_t pol = l2_evict_first();
    uint32_t u = 0;
    int e_cur = a.work[blockIdx.x / nmt].expert;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += G) {
      const int e_nxt = tile + G < ntiles ? a.work[(tile + G) / nmt].expert : 0;  // prefetch
      const int t0 = (tile % nmt) * kTilesOp;
      const CUtensorMap* map = maps + (size_t)e_cur * kMapsPerExpert + (active ? part : 0) * 3 + proj;
      for (int sidx = 0; sidx < nsl; ++sidx, ++u) {
        if (u % kWLoaders != wl) continue;
        const uint32_t sw = u % kWS;
        if (u >= (uint32_t)kWS && !mb_wait(&emptyW[sw], ((u / kWS) - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) mb_expect(&fullW[sw], kWBytes);
        __syncwarp();
        if (active) tma_load_3d(su32(ringW + sw * kWSlot) + dst_off, map, 0, sidx * ystep, t0, &fullW[sw], pol);
      }
      e_cur = e_nxt;
    }
    if (lane == 0) drain_ring(fullW, kWS, u, wl, kWLoaders);
  } else if (warp >= kBLoader0 && warp < kBLoader0 + kBLoaders) {
    // --------------------------- activation loaders -----------------------------
    // warp kBLoader0 + b loads blocks j = b, b + kBLoaders, ... of the stage
    // ring: one TMA box of the item's rows (the smallest of 32/64/128/256 rows
    // that covers them; rows past the item belong to the next item or are out
    // of bounds and zero-filled, and their accumulator columns are never stored).
    uint32_t j = 0;
    WorkItem it = a.work[blockIdx.x / nmt];
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += G) {
      const WorkItem nit = tile + G < ntiles ? a.work[(tile + G) / nmt] : it;  // prefetch
      const int kind = min(C::kBoxKinds - 1, it.nrows <= 32 ? 0 : (it.nrows <= 64 ? 1 : (it.nrows <= 128 ? 2 : 3)));
      const uint32_t bytes = (32u << kind) * 128u;
      for (int kb = 0; kb < nb; ++kb, ++j) {
        if (j % kBLoaders != (uint32_t)(warp - kBLoader0)) continue;
        const uint32_t s = j % kStages, pr = j >> 1, p = pr % kPairBars, po = pr - kStages / 2;
        // slot s was last read by pair po
        if (j >= (uint32_t)kStages && !mb_wait(&empty[po % kPairBars], (po / kPairBars) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mb_expect(&full[p], bytes);
          tma_load_2d(su32(ringB + s * kBSlot), &tmB.m[kind], kb * 64, it.row0, &full[p]);
        }
        __syncwarp();
      }
      it = nit;
    }
    // the stage barriers also count the dequantisers' arrivals, so after an
    // abort they may never complete: give the boxes in flight time to land
    if (!ok && lane == 0) {
      const long long t0 = clock64();
      while (clock64() - t0 < (1ll << 22)) {
      }
    }
  } else if (warp >= kDeq0 && warp < kDeq0 + kDeqWarps) {
    // ------------------------------- dequantisers -------------------------------
    const int quad = warp & 3;                  // TMEM lanes 32 quad .. +31
    const int h = (warp - kDeq0) >> 2;          // pairs pt with pt % kDeqPerQuad == h
    const int r16 = lane & 15, g = r16 & 7, hi = r16 >> 3;
    // this thread's row: box op and tile within the box
    const int op = MODE == MODE_GATE_UP ? (lane >> 4) : 0;
    const int tt = MODE == MODE_GATE_UP ? quad : 2 * quad + (lane >> 4);
    const uint32_t shift = 4 * hi;              // nibbles of row g+8 sit 4 bits higher
    uint32_t qsrc[4];
#pragma unroll
    for (int t = 0; t < 4; ++t)
      qsrc[t] = op * (kWRaw / kOps) + tt * kSlotBlocks * 512 + g * 64 + (((t ^ (g >> 1)) & 3) << 4);
    const uint32_t ssrc = kWOffS + op * (kTilesOp * kGps * 32) + tt * kGps * 32 + r16 * 2;
    const float zpf = AWQ ? (float)(128 + a.zp) : 128.f;
    const uint32_t zp2 = bf16x2_of(zpf);
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + kACol;
    const int np = nb >> 1;  // K-block pairs per tile (a pair never straddles a weight slot)
    uint32_t j = 0;          // block counter (stage ring)
    for (uint32_t ti = 0; ti < my_tiles && ok; ++ti) {
      // the quadrant's warps take the pairs in turn by their index over all of
      // the CTA's tiles, so a warp's successive pairs are exactly kDeqPerQuad
      // apart across tile ends too (a per-tile restart would leave up to
      // 2 kDeqPerQuad - 1 when np is not a multiple of it; URoles needs at most
      // S): one weight-slot wait, one A-slot wait and one arrival on the
      // pair's full barrier per two blocks
      const int p0 = (int)((j >> 1) % kDeqPerQuad);
      for (int pt = (h - p0 + kDeqPerQuad) % kDeqPerQuad; pt < np; pt += kDeqPerQuad) {
        const int kb0 = 2 * pt, c0 = kb0 % kSlotBlocks;
        const uint32_t jb = j + kb0;
        const uint32_t u = ti * nsl + kb0 / kSlotBlocks, sw = u % kWS;
        const uint32_t pra = jb >> 1, pa = pra % kPairBars, poa = pra - kStages / 2;
        if (!mb_wait(&fullW[sw], (u / kWS) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        const unsigned char* wsl = ringW + sw * kWSlot;
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int c = c0 + bi;
          uint4 q4[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) q4[t] = *reinterpret_cast<const uint4*>(wsl + qsrc[t] + c * 512);
          // groups of this block within the slot: gs 128 -> c/2, gs 64 -> c, gs 32 -> 2c, 2c+1
          const int gq = GSB == 4 ? (c >> 1) : (GSB == 2 ? c : 2 * c);
          uint32_t sc[NG];       // AWQ: the scale as a bf16 pair
          float sf[NG], zf[NG];  // GPTQ: scale and zero in fp32 (exact fp16 values)
#pragma unroll
          for (int q = 0; q < NG; ++q) {
            const float s16 = __half2float(*reinterpret_cast<const __half*>(wsl + ssrc + (gq + q) * 32));
            if (AWQ) {
              sc[q] = bf16x2_of(s16);
            } else {
              sf[q] = s16;
              zf[q] = __half2float(*reinterpret_cast<const __half*>(wsl + ssrc + (gq + q) * 32 + kWOffZ - kWOffS));
            }
          }
          if (bi == 1) {  // both blocks' words are in registers: release this quadrant's share of the slot
            __syncwarp();
            if (lane == 0) mb_arrive_n(&emptyW[sw], kSlotBlocks);
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
              if (AWQ) {  // (q - zp) * s: an exact integer times the scale, rounded once
                p0 = h2mul(h2sub(p0, zp2), sc[q]);
                p1 = h2mul(h2sub(p1, zp2), sc[q]);
              } else {  // q * s + z in fp32 (q * s exact), rounded once to bf16
                p0 = gptq_pair(p0, sf[q], zf[q]);
                p1 = gptq_pair(p1, sf[q], zf[q]);
              }
              const int col = kb2 * 16 + 4 * t + 2 * kt;  // TMEM column = k / 2
              r[col] = p0;
              r[col + 1] = p1;
            }
          }
          if (bi == 0) {  // the pair's A slots were last read by pair poa
            if (jb >= (uint32_t)kStages && !mb_wait(&empty[poa % kPairBars], (poa / kPairBars) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          tmem_st32(tl + 32 * ((jb + bi) % kStages), r);
        }
        if (!ok) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mb_arrive(&full[pa]);
      }
      j += nb;
    }
  } else {
    // --------------------------------- epilogue ---------------------------------
    // kEpiPerQuad warps per TMEM lane quadrant, each draining its share of the
    // N columns; a column's value is the sum of the tile's nis partial
    // accumulators, added in issuer order
    const int quad = warp & 3;
    const int part = (warp - kEpi0) >> 2;
    const int np = nb >> 1;
    const uint32_t tq = tmem + ((uint32_t)(quad * 32) << 16);
    uint32_t i = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += G, ++i) {
      const WorkItem it = a.work[tile / nmt];  // loads while the accumulator fills
      const int mt = tile % nmt;
      if (!mb_wait(&accFull, i & 1, &abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int N = min(NMAX, (it.nrows + 15) & ~15);
      int stride;
      const int nis = tile_issuers<NMAX>(N, np, &stride);
      const int share = ((N >> 4) + kEpiPerQuad - 1) / kEpiPerQuad * 16;
      const int cbeg = part * share, cend = min(N, cbeg + share);
      // one chunk's 16 columns (values of this thread's TMEM lane) to the outputs
      auto emit = [&](int c0, const float (&v)[16]) {
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
      };
      auto as_f = [](const uint32_t (&r)[16], float (&v)[16]) {
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = __uint_as_float(r[c]);
      };
      if (MODE == MODE_GATE_UP && nis == 1) {
        // one accumulator: the next chunk's TMEM load is in flight while this
        // chunk's SiLU*mul is computed and stored (two register sets,
        // alternating; measured 1-2 % off gate/up, while the fp32 down
        // epilogue, with less work per column, did not gain)
        uint32_t ra[16], rb[16];
        float v[16];
        if (cbeg < cend) {
          tmem_ld16_issue(tq + cbeg, ra);
          tmem_ld16_wait(ra);
        }
        for (int c0 = cbeg; c0 < cend; c0 += 32) {
          const bool more = c0 + 16 < cend;
          if (more) tmem_ld16_issue(tq + c0 + 16, rb);
          as_f(ra, v);
          emit(c0, v);
          if (!more) break;
          tmem_ld16_wait(rb);
          const bool more2 = c0 + 32 < cend;
          if (more2) tmem_ld16_issue(tq + c0 + 32, ra);
          as_f(rb, v);
          emit(c0 + 16, v);
          if (more2) tmem_ld16_wait(ra);
        }
      } else {
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
          float v[16];
          tmem_ld16(tq + c0, v);
          for (int q = 1; q < nis; ++q) {
            float w[16];
            tmem_ld16(tq + (uint32_t)(q * stride + c0), w);
#pragma unroll
            for (int c = 0; c < 16; ++c) v[c] += w[c];
          }
          emit(c0, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mb_arrive(&accEmpty);
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

// Rows of the gate/up activations in expert-sorted order: Xs[p] = X[sorted[p] / kk]
// for p < *n_valid (the placed pairs; empty slots are not placed), one warp per
// row, 16-byte pieces, so every work item's rows are contiguous and its B
// tiles are plain TMA boxes.
__global__ void __launch_bounds__(256) k_gather_rows(const uint4* __restrict__ X, int H8,
                                                     const int* __restrict__ sorted, int kk, int n,
                                                     const int* __restrict__ n_valid, uint4* __restrict__ Xs) {
  grid_dep_wait();
  grid_dep_release();
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (p >= n || (n_valid && p >= *n_valid)) return;
  const uint4* src = X + (size_t)(sorted[p] / kk) * H8;
  uint4* dst = Xs + (size_t)p * H8;
  for (int c = threadIdx.x & 31; c < H8; c += 32) dst[c] = __ldg(src + c);
}

cudaError_t launch_gather_rows(const void* X, int H, const int* sorted, int kk, int n, const int* n_valid,
                               void* Xs, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  return launch_pdl(k_gather_rows, dim3((n + 7) / 8), dim3(256), 0, st, reinterpret_cast<const uint4*>(X), H / 8,
                    sorted, kk, n, n_valid, reinterpret_cast<uint4*>(Xs));
}

namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled tensor_map_encoder() {
  static const EncodeTiled fn = []() -> EncodeTiled {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}
// B operand: `rows` x K bf16, row stride ld elements; boxes of 64 elements
// (128 B, the 128-byte swizzle span) x box_rows rows; out-of-bounds rows read zero.
bool b_tensor_map(CUtensorMap* m, const void* base, int K, int rows, int ld, int box_rows) {
  const EncodeTiled enc = tensor_map_encoder();
  if (!enc || rows <= 0 || K <= 0 || (reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

bool build_umma_weight_maps(const ExpertDev* h, int n_exp, int inter, int hidden, int gs, bool gptq,
                            void* host_out) {
  static_assert(sizeof(CUtensorMap) == kTensorMapBytes, "tensor map size");
  const EncodeTiled enc = tensor_map_encoder();
  if (!enc || gs <= 0 || (kSlotBlocks * 64) % gs) return false;
  CUtensorMap* out = static_cast<CUtensorMap*>(host_out);
  memset(host_out, 0, (size_t)n_exp * kMapsPerExpert * sizeof(CUtensorMap));
  for (int e = 0; e < n_exp; ++e)
    for (int proj = 0; proj < 3; ++proj) {
      const ProjDev& P = proj == 0 ? h[e].gate : (proj == 1 ? h[e].up : h[e].down);
      const int M = proj < 2 ? inter : hidden, K = proj < 2 ? hidden : inter;
      const cuuint64_t Kc = (cuuint64_t)(K / 64), Mt = (cuuint64_t)(M / 16), ng = (cuuint64_t)(K / gs);
      const cuuint32_t tiles = proj < 2 ? 4 : 8;  // 16-row tiles per box (64 or 128 weight rows)
      const cuuint32_t estr[3] = {1, 1, 1};
      {  // raw words: {128 words of a 512-byte chunk, chunk, tile}
        const cuuint64_t dims[3] = {128, Kc, Mt};
        const cuuint64_t strides[2] = {512, Kc * 512};
        const cuuint32_t box[3] = {128, (cuuint32_t)kSlotBlocks, tiles};
        if (enc(out + e * kMapsPerExpert + proj, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint4*>(P.q), dims,
                strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
          return false;
      }
      for (int part = 1; part <= (gptq ? 2 : 1); ++part) {  // scales / zeros: {16 rows, group, tile}
        const cuuint64_t dims[3] = {16, ng, Mt};
        const cuuint64_t strides[2] = {32, ng * 32};
        const cuuint32_t box[3] = {16, (cuuint32_t)(kSlotBlocks * 64 / gs), tiles};
        const __half* base = part == 1 ? P.s : P.z;
        if (!base || enc(out + e * kMapsPerExpert + part * 3 + proj, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3,
                         const_cast<__half*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
          return false;
      }
    }
  return true;
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

template <int MODE, int GSB, bool AWQ, int NMAX>
static cudaError_t launch_u(const GemmArgs& a, int max_work, int b_rows, cudaStream_t st) {
  BMaps tmB;
  memset(&tmB, 0, sizeof(tmB));
  for (int k = 0; k < UCfg<NMAX>::kBoxKinds; ++k)
    if (!b_tensor_map(&tmB.m[k], a.B, a.K, b_rows, a.ldb, 32 << k)) return cudaErrorInvalidValue;
  constexpr int smem = umma_smem<AWQ, NMAX>();
  static bool attr = false;  // per template instance
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k_int4_umma<MODE, GSB, AWQ, NMAX>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int nmt = a.M / (MODE == MODE_GATE_UP ? 64 : 128);
  const long long tiles = (long long)max_work * nmt;
  const int grid = (int)std::min<long long>(tiles, sm_count());
  return launch_pdl(k_int4_umma<MODE, GSB, AWQ, NMAX>, dim3(grid), dim3(kUThreads), (size_t)smem, st, a, tmB);
}

template <int MODE, bool AWQ, int NMAX>
static cudaError_t launch_u_gs(const GemmArgs& a, int max_work, int b_rows, cudaStream_t st) {
  switch (a.gs) {
    case 32: return launch_u<MODE, 1, AWQ, NMAX>(a, max_work, b_rows, st);
    case 64: return launch_u<MODE, 2, AWQ, NMAX>(a, max_work, b_rows, st);
    default: return launch_u<MODE, 4, AWQ, NMAX>(a, max_work, b_rows, st);
  }
}

template <int NMAX>
static cudaError_t launch_u_n(int mode, const GemmArgs& a, int max_work, int awq, int b_rows, cudaStream_t st) {
  if (mode == MODE_GATE_UP)
    return awq ? launch_u_gs<MODE_GATE_UP, true, NMAX>(a, max_work, b_rows, st)
               : launch_u_gs<MODE_GATE_UP, false, NMAX>(a, max_work, b_rows, st);
  return awq ? launch_u_gs<MODE_PLAIN_F32, true, NMAX>(a, max_work, b_rows, st)
             : launch_u_gs<MODE_PLAIN_F32, false, NMAX>(a, max_work, b_rows, st);
}

// Requires M % 64 (gate/up) or M % 128 (down) == 0, K % 128 == 0, items of
// at most item_rows rows (kUmmaSmallRows or kUmmaRows), gs in {32, 64, 128},
// and B = b_rows contiguous expert-sorted rows (a.gather is not used).
cudaError_t launch_gemm_umma(int mode, const GemmArgs& a, int max_work, int awq, int b_rows, int item_rows,
                             cudaStream_t st) {
  if (max_work <= 0) return cudaSuccess;
  if (item_rows == kUmmaSmallRows) return launch_u_n<kUmmaSmallRows>(mode, a, max_work, awq, b_rows, st);
  if (item_rows == kUmmaRows) return launch_u_n<kUmmaRows>(mode, a, max_work, awq, b_rows, st);
  return cudaErrorInvalidValue;
}

}  // namespace llmoc
