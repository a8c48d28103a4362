// kernels.cuh — argument structs and launchers shared by the kernel files
// (route.cu, int4_gemm.cu) and the host runtime (runtime.cu).
#pragma once
#include <cstring>

#include "common.cuh"

namespace llmoc {

// ---- route.cu
struct TopkArgs {
  const float* logits;   // [T,ld]: E routed logits (+ the shared gate's at column E)
  const float* bias;     // [E] (sigmoid router)
  int T, E, k, kk;       // kk = k + has_shared
  int ld = 0;            // logits row stride (0: E)
  int router;            // 0 softmax, 1 sigmoid+bias
  float routed_scaling;
  float shared_scale;
  int has_shared;
  int shared_gate = 0;   // the shared expert's weight is sigmoid(logits[t][E]) per token
  float* shared_w = nullptr;  // [T] per-token shared weights (expert-parallel source; may be null)
  // sigmoid router: the scores sigmoid_ref(logit), laid out as the logits,
  // made where the logits were (null: computed from the logits here)
  const float* sig = nullptr;
  int* ids;              // [T,kk]
  float* weights;        // [T,kk]
  // expert parallelism: also each pair's owner key (e % world) * e_loc + e / world
  int* ep_key = nullptr;  // [T,kk] (null: none)
  int ep_world = 1, ep_e_loc = 1;
  // the token's fp16 row for the decode gate/up GEMM, made by the same warp
  // (prep_xh_row; xh null: none)
  const void* x = nullptr;  // bf16 [T][H]
  int H = 0, gs = 0;
  void* xh = nullptr;
  float* xsum = nullptr;
  float* xscale = nullptr;
};

// A bounded wait for peers' step flags, folded into the kernel that first
// reads what they guard (the NVLink transport): threads 0..n-1 each poll
// flags[i] with ld.acquire.sys until it reaches seq, giving up after `budget`
// SM clocks (then bit 1 of *err is set and the kernel goes on).  Every thread
// of the block calls flag_wait_block (it synchronises the block).
struct FlagWait {
  const uint32_t* flags = nullptr;  // null: no wait
  int n = 0;
  uint32_t seq = 0;
  int* err = nullptr;
  long long budget = 0;
};
#ifdef __CUDACC__
__device__ __forceinline__ void flag_wait_block(const FlagWait& fw) {
  if (!fw.flags) return;  // uniform over the block
  __shared__ int fw_timed_out;
  if (threadIdx.x == 0) fw_timed_out = 0;
  __syncthreads();
  if ((int)threadIdx.x < fw.n) {
    const uint32_t* f = fw.flags + threadIdx.x;
    const long long t0 = clock64();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if ((int)(v - fw.seq) >= 0) break;
      if (clock64() - t0 > fw.budget) {
        fw_timed_out = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (fw_timed_out && threadIdx.x == 0 && fw.err) atomicOr(fw.err, 2);
}
#endif

struct PermArgs {
  const int* ids;   // [n] expert id per pair, n = T*kk, pair p = t*kk + j
  int n;
  int n_exp;        // experts incl. the shared one
  int* offsets;     // [n_exp+1]
  int* sorted;      // [n]
  int* inverse;     // [n]
  WorkItem* work;   // [max_work]
  int* n_work;
  int* n_active;
  int* err;         // device error word + kGemmCounters unit counters, all cleared here for the kernels that follow
  int chunk;        // rows per work item (8, 16 or 32)
  // segmented input (seg_len > 0): ids form n_seg segments of seg_len slots
  // (n = n_seg * seg_len) of which the first seg_count[s * seg_stride]
  // (clamped to [0, seg_len]) are occupied; only those are read, counted and
  // placed (sorted / inverse), in slot order -- the NVLink transport's
  // per-source receive regions
  const int* seg_count;
  int seg_stride, seg_len, n_seg;
  FlagWait wait;    // the sources' dispatch flags, waited for before anything is read
};

constexpr int kGemmCounters = 2;  // err[1], err[2]: unit counters of the gate/up and down GEMMs
constexpr int kPermThreads = 1024;
constexpr int kPermWarps = kPermThreads / 32;
constexpr int kMaxExpPerm = 512;  // experts (incl. shared) the permutation CTA handles

// The decode gate/up GEMM's fp16 rows (prep_xh_row) of the router's tokens,
// made by the decode router (T <= kRouterSmallMaxT) from its copy of them.
struct XhOut {
  void* xh = nullptr;  // null: none
  float* xsum = nullptr;
  float* xscale = nullptr;
  int gs = 0;
};
constexpr int kRouterSmallMaxT = 8;
cudaError_t launch_router_logits(const void* X, bool x_is_f32, const uint16_t* Wr, int T, int E,
                                 int H, float* logits, cudaStream_t st, const XhOut& xo = XhOut{});
cudaError_t launch_topk(const TopkArgs& a, cudaStream_t st);
struct EpRouteArgs;
cudaError_t launch_permute(const PermArgs& a, cudaStream_t st);
// the same with the expert-parallel tail (per-owner counts, owner-local expert
// of each pair in key order; pa.ids are the owner keys)
cudaError_t launch_permute_ep(const PermArgs& a, const EpRouteArgs& ea, cudaStream_t st);
// top-k and permutation in one CTA (decode-size T; pa.ids must be ta.ids, or,
// for the expert-parallel dispatch, ea.key: the permutation then runs over the
// owner keys, and the per-owner counts and owner-local experts are written)
constexpr int kFusedRouteMaxT = 16;
struct EpRouteArgs {
  int world = 1, e_loc = 0;
  int* key = nullptr;          // [n] owner key of each pair (null: not expert-parallel)
  int* counts = nullptr;       // [world]
  int* send_expert = nullptr;  // [n] owner-local expert of each pair in key order
};
cudaError_t launch_topk_permute(const TopkArgs& ta, const PermArgs& pa, cudaStream_t st,
                                const EpRouteArgs& ea = EpRouteArgs{});
cudaError_t launch_fill_i32(int* p, int n, int v, cudaStream_t st);
// sh_w: per-token shared weights (null: sh_scale for every token)
// fw: the owners' return flags, waited for before the returned rows are read
cudaError_t launch_combine_ep(const void* ret, const int* inverse, const float* w, int T, int topk, int H,
                              const float* sh, const int* sh_inv, float sh_scale, const float* sh_w, void* y,
                              cudaStream_t st, const FlagWait& fw = FlagWait{});

// ---- ep_p2p.cu: expert-parallel transport over NVLink peer memory
constexpr int kEpMaxWorld = 64;
constexpr int kEpPushCtas = 148;  // push grids: one CTA per SM
// byte offsets of the regions of one rank's transport buffer
struct EpP2PLayout {
  int world, cap, row_bytes;  // row_bytes = hidden * 2
  size_t flags, meta, recv_ids, recv_rows, ret_rows, total;
};
// send_rows [q] = the q-th pair's row, or (sorted non-null) X[sorted[q] / kk]
// read directly (no gathered copy)
cudaError_t launch_ep_push_dispatch(const EpP2PLayout& L, char* const* peers, const void* send_rows,
                                    const int* send_expert, const int* counts, int rank, uint32_t seq, int* ctr,
                                    cudaStream_t st, const void* X = nullptr, const int* sorted = nullptr,
                                    int kk = 1);
// budget: SM clock cycles after which a wait gives up (sets bit 1 of *err)
constexpr long long kDefaultWaitCycles = 1ll << 31;  // ~1.1 s at 1.965 GHz
cudaError_t launch_ep_wait(const EpP2PLayout& L, char* base, int kind, uint32_t seq, int* err, long long budget,
                           cudaStream_t st);
// partial: the owner's down output rows (fp32, expert-sorted), inverse: row of each receive slot
cudaError_t launch_ep_push_return(const EpP2PLayout& L, char* const* peers, char* base, const float* partial,
                                  const int* inverse, int rank, uint32_t seq, int* ctr, cudaStream_t st);

// ---- collective.cu: ICollective over NVLink peer memory (layout there)
struct CollLayout {
  int world;
  size_t slot;  // bytes of one staging slot (the largest payload)
  size_t flags, acks, stage, total;
};
cudaError_t launch_coll_wait(const CollLayout& L, char* base, int which, uint32_t target, int* err, long long budget,
                             cudaStream_t st);
cudaError_t launch_coll_push(const CollLayout& L, char* const* peers, const void* src, size_t src_stride, size_t n,
                             int rank, uint32_t seq, int* ctr, cudaStream_t st);
cudaError_t launch_coll_consume(const CollLayout& L, char* base, char* const* peers, int op, void* dst, size_t n,
                                int dtype, int root, int rank, uint32_t seq, int* ctr, cudaStream_t st);

// ---- int4_gemm.cu
struct RepackArgs {
  const uint8_t* q;      // QLWC [M, ceil(K/2)]
  const uint16_t* s;     // [M, ng] fp16
  const uint16_t* z;     // [M, ng] fp16 or nullptr
  int M, K, gs, ng, Kc;  // Kc = ceil(K/64)
  uint32_t* qo;          // [Mt][Kc][32][4] words
  uint16_t* so;          // [Mt][ng][16]
  uint16_t* zo;          // [Mt][ng][16] or nullptr
};

enum { MODE_GATE_UP = 0, MODE_PLAIN_F32 = 1 };

struct GemmArgs {
  const ExpertDev* experts;
  int proj;               // MODE_PLAIN_F32: 0 gate, 1 up, 2 down
  int M, K, Kc, gs, ng;
  int zp;                 // AWQ zero point
  const void* B;          // activations (bf16 for mma; bf16 or fp32 for cc)
  int ldb;
  const int* gather;      // B row of sorted pos p = gather[p] / kk (nullptr: row p)
  int kk;
  const WorkItem* work;
  const int* n_work;
  void* out;              // GATE_UP: mid [pos][ldo]; PLAIN: fp32 [pos][ldo]
  int ldo;
  int out_bf16;           // GATE_UP output type (cc kernel): 1 bf16, 0 fp32
  int* err;               // device error word: bit 0 = a bounded wait gave up (may be null)
  const void* wmaps;      // tcgen05 path: per-expert TMA maps of the weights (build_umma_weight_maps)
  int* ctr;               // persistent decode kernel: unit counter, zeroed by the permutation (or null)
  int keep_nonfinite;     // cc kernel, PLAIN_F32: store non-finite sums as they are (argmax input)
  // fp16 activation form of the decode gate/up GEMM (bsum != null): B holds
  // the rows as fp16 scaled by 2^-e per row, bsum [row][ng] the per-group sums
  // of those fp16 values, bscale [row] = 2^e (launch_prep_xh)
  const float* bsum = nullptr;
  const float* bscale = nullptr;
};

// fp16 activation rows for the decode gate/up GEMM.  Row r (r < R, or, with
// rows_of, row rows_of[p] for p < min(R, *n_valid)) of X (bf16 [.][H]):
// Xh = x * 2^-e rounded to fp16, e chosen so the row's largest |x| lands in
// [2^14, 2^15) (exact for every value within 2^28 of the largest; e = 0 for an
// all-zero or non-finite row), xsum [.][H/gs] the fp32 sums of each group of
// Xh (a fixed order), xscale = 2^e.  H % 128 == 0, gs in {32, 64, 128}.
cudaError_t launch_prep_xh(const void* X, int R, int H, int gs, const int* rows_of, const int* n_valid, void* Xh,
                           float* xsum, float* xscale, cudaStream_t st);

// Argmax over y[M] (hal::gemm_int4_argmax semantics: non-finite -> -1e30,
// the first of equal maxima): *key = max over rows of the key of (y[m], m),
// the value's order-preserving bits above ~m; decode with argmax_decode.
cudaError_t launch_argmax_rows(const float* y, int M, unsigned long long* key, cudaStream_t st);
inline void argmax_decode(unsigned long long key, int32_t* index, float* value) {
  const uint32_t b = (uint32_t)(key >> 32);
  const uint32_t bits = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  float v;
  memcpy(&v, &bits, 4);
  *value = v;
  *index = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

cudaError_t launch_repack(const RepackArgs& a, cudaStream_t st);
cudaError_t launch_dequant(const ProjDev& P, int M, int K, int gs, int awq, int zp, float* out,
                           cudaStream_t st);
// path: 0 tensor-core (AWQ, bf16 B), 1 CUDA-core fp32 B, 2 CUDA-core bf16 B
// n_groups: experts (groups) the rows can reach, for the decode kernel choice (0: unknown);
// grid_items: work items expected (0: max_work), the tensor-core K-split grid's height
cudaError_t launch_gemm(int mode, int path, const GemmArgs& a, int max_work, int awq, int ntiles,
                        cudaStream_t st, int n_groups = 0, int grid_items = 0);
// int4_umma.cu: tcgen05.mma (TMEM accumulator) grouped GEMM for work items of
// up to item_rows rows: kUmmaRows (prefill-size groups) or kUmmaSmallRows
// (groups of tens of rows, up to four MMA issuers per tile); same K /
// group-size conditions.  B is b_rows contiguous expert-sorted rows read by
// TMA (a.gather unused).
constexpr int kUmmaRows = 256;
constexpr int kUmmaSmallRows = 64;
cudaError_t launch_gemm_umma(int mode, const GemmArgs& a, int max_work, int awq, int b_rows, int item_rows,
                             cudaStream_t st);
// TMA tensor maps (128 bytes each) of every expert's repacked weights for the
// tcgen05 kernel, kMapsPerExpert per expert: [part * 3 + proj], part 0 raw
// words, 1 scales, 2 zeros (GPTQ); proj 0 gate, 1 up, 2 down.  Built once per
// layer on the host (host_out: n_exp * kMapsPerExpert * 128 bytes).
constexpr int kMapsPerExpert = 9;
constexpr int kTensorMapBytes = 128;
bool build_umma_weight_maps(const ExpertDev* host_table, int n_exp, int inter, int hidden, int gs, bool gptq,
                            void* host_out);
// Xs[p, :] = X[sorted[p] / kk, :] for p < min(n, *n_valid) (bf16 rows of H
// elements, H % 8 == 0; n_valid may be null).
cudaError_t launch_gather_rows(const void* X, int H, const int* sorted, int kk, int n, const int* n_valid,
                               void* Xs, cudaStream_t st);
// y[t] (+)= sum_j w[t,j] * d[inverse[t*kk+j]]; res (bf16 [T,H], may alias y):
// y = res + sum, the residual stream of the caller's decoder layer.
cudaError_t launch_combine(const float* d, const int* inverse, const float* w, int T, int kk, int H,
                           void* y, int y_bf16, int skip_tiny, cudaStream_t st, const void* res = nullptr);
cudaError_t launch_quant_awq_sym(const __nv_bfloat16* W, int M, int K, int gs, int bf16_scale,
                                 uint8_t* q, __half* sc, cudaStream_t st);

// Fused single-token decode (k_moe_decode1, int4_gemm.cu): the router rows,
// the top-k, gate/up + SiLU*mul, down and the weighted combine of one token in
// one cooperative launch, with grid-wide barriers between the phases.  The
// arithmetic of each phase is that of the separate kernels (router_dot_warp,
// topk_token, mma_kblock, k_combine's ordered FMAs).
constexpr int kDecode1MaxCtas = 2048;  // grid cap of the fused kernel
constexpr int kDecode1MaxSlots = 65;   // topk <= 64, + the shared expert
struct Decode1Args {
  const __nv_bfloat16* X;  // [1][H]
  const uint16_t* Wr;      // [rows][H] bf16 router rows (E routed, then the shared gate's)
  int rows, H;
  float* logits;           // [rows] the router's output
  TopkArgs ta;             // T = 1 over logits; ids / weights: the routing views
  float* sig;              // [rows] the sigmoid router's scores (ta.sig), or null
  GemmArgs gu, dn;         // work, n_work and gather are set in the kernel (shared memory)
  int ks_gu, gx_gu, ks_dn, gx_dn;  // K split and virtual grid width of each GEMM phase
  int ex_off;              // byte offset of the slots' expert table in dynamic shared memory
  const float* partial;    // dn.out
  __nv_bfloat16* Y;
  const __nv_bfloat16* R;  // residual (may alias Y) or null
  int n_exp;               // routed + shared experts: offsets has n_exp + 1 entries
  int* offsets;
  int* sorted;
  int* inverse;
  int* n_active;
  int* err;                // bit 2: a barrier wait gave up
  unsigned long long* bar;  // [3]: the barrier's arrival counter and the count of CTAs past the last barrier
                           // (low 32 bits of [0] and [2]), the launch's tag [1]
  unsigned long long epoch;  // distinct per launch: barrier tags never match an older launch's words
  long long budget;        // SM clocks per barrier wait
};
// Launches k_moe_decode1 (a.ks_* / a.gx_* are filled here from the grid).
cudaError_t launch_decode1(Decode1Args a, int awq, cudaStream_t st);

}  // namespace llmoc
