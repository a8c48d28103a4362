// runtime.cu — host side of the C ABI (include/llmoc_b200.h).
//
// Mirrors the reference's hal::cuda process-global backend
// (src/hal/cuda_backend.cpp:155 mutex, :604-688 INT4 residency keyed by the
// host qweight pointer with an LRU under a VRAM budget, :2692 try_gemm_int4,
// :5217 try_moe_ffn_int4) on top of this library's kernels, and adds the
// device-resident batched MoE layer (llmoc_moe_*).  No CPU fallback exists:
// when the GPU path cannot run, the try_* calls return 0 and the batched
// calls return an error status.
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/llmoc_b200.h"
#include "kernels.cuh"


using namespace llmoc;

namespace {

// ------------------------------------------------------------------ state

std::atomic<uint64_t> g_launches{0};
thread_local std::string t_err;
std::mutex g_mu;  // serialises the process-global backend, like the reference's g_mu
bool g_probed = false, g_available = false, g_enabled = false;
int g_ndev = 0;
std::string g_status = "not probed";
size_t g_budget = 0, g_used = 0;
uint64_t g_tick = 0;
cudaStream_t g_stream = nullptr;

constexpr int kMaxExperts = kMaxExpPerm - 1;  // routed experts per layer (+1 shared) in the permutation CTA
constexpr int kMaxTopk = 64;      // qwen3_6_moe_int4_model.cpp:384

int fail(const std::string& msg) {
  t_err = msg;
  return 0;
}
llmoc_status fails(llmoc_status s, const std::string& msg) {
  t_err = msg;
  return s;
}
bool cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  t_err = std::string(what) + ": " + cudaGetErrorString(e);
  return false;
}
void count_launch(int n = 1) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Geometry of one repacked projection.
struct Geo {
  int M = 0, K = 0, gs = 0, ng = 0, Kc = 0, Mt = 0;
  size_t qbytes = 0, sbytes = 0, zbytes = 0;
  size_t total() const { return align256(qbytes) + align256(sbytes) + align256(zbytes); }
};
Geo make_geo(int M, int K, int gs, bool zeros) {
  Geo g;
  g.M = M;
  g.K = K;
  g.gs = gs;
  g.ng = (K + gs - 1) / gs;
  g.Kc = (K + 63) / 64;
  g.Mt = (M + 15) / 16;
  g.qbytes = (size_t)g.Mt * g.Kc * 512;
  g.sbytes = (size_t)g.Mt * g.ng * 16 * 2;
  g.zbytes = zeros ? g.sbytes : 0;
  return g;
}

// Shapes the kernels accept: K a multiple of 32, group size a multiple of 32.
bool shape_ok(int M, int K, int gs, std::string* why) {
  if (M <= 0 || K <= 0 || gs <= 0) {
    *why = "non-positive M/K/group_size";
    return false;
  }
  if (K % 32 != 0 || gs % 32 != 0) {
    *why = "K and group_size must be multiples of 32";
    return false;
  }
  return true;
}

// Upload a QLWC projection (host or device source) into `dst` (repacked).
bool repack_into(const llmoc_int4_view& W, bool src_on_device, const Geo& g, char* dst,
                 cudaStream_t st, ProjDev* out) {
  const bool awq = W.scheme == LLMOC_SCHEME_AWQ_SYM;
  const size_t rb = (size_t)((W.K + 1) / 2);
  const size_t qsrc = rb * W.M, ssrc = (size_t)W.M * g.ng * 2;
  const uint8_t* q = W.qweight;
  const uint16_t* s = W.scales;
  const uint16_t* z = (!awq && W.zeros) ? W.zeros : nullptr;
  void* staging = nullptr;
  if (!src_on_device) {
    const size_t need = align256(qsrc) + align256(ssrc) + (z ? align256(ssrc) : 0);
    if (!cuda_ok(cudaMallocAsync(&staging, need, st), "cudaMallocAsync(staging)")) return false;
    char* p = (char*)staging;
    if (!cuda_ok(cudaMemcpyAsync(p, q, qsrc, cudaMemcpyHostToDevice, st), "H2D qweight")) return false;
    q = (const uint8_t*)p;
    p += align256(qsrc);
    if (!cuda_ok(cudaMemcpyAsync(p, s, ssrc, cudaMemcpyHostToDevice, st), "H2D scales")) return false;
    s = (const uint16_t*)p;
    p += align256(ssrc);
    if (z) {
      if (!cuda_ok(cudaMemcpyAsync(p, z, ssrc, cudaMemcpyHostToDevice, st), "H2D zeros")) return false;
      z = (const uint16_t*)p;
    }
  }
  RepackArgs ra;
  ra.q = q;
  ra.s = s;
  ra.z = z;
  ra.M = W.M;
  ra.K = W.K;
  ra.gs = g.gs;
  ra.ng = g.ng;
  ra.Kc = g.Kc;
  ra.qo = (uint32_t*)dst;
  ra.so = (uint16_t*)(dst + align256(g.qbytes));
  ra.zo = g.zbytes ? (uint16_t*)(dst + align256(g.qbytes) + align256(g.sbytes)) : nullptr;
  const bool ok = cuda_ok(launch_repack(ra, st), "repack");
  count_launch();
  if (staging) cudaFreeAsync(staging, st);
  out->q = (const uint4*)ra.qo;
  out->s = (const __half*)ra.so;
  out->z = (const __half*)ra.zo;
  return ok;
}

// --------------------------------------------------- resident weight cache

struct Resident {
  char* buf = nullptr;
  Geo geo;
  ProjDev dev{};
  ExpertDev* table = nullptr;  // 1-entry device table with gate = dev (dense GEMM)
  int scheme = LLMOC_SCHEME_AWQ_SYM;
  int zp = 7;
  size_t bytes = 0;
  bool pinned = false;
  uint64_t last_use = 0;
};
std::unordered_map<const void*, Resident> g_cache;

void free_resident(Resident& r) {
  if (r.buf) cudaFree(r.buf);
  if (r.table) cudaFree(r.table);
  r.buf = nullptr;
  r.table = nullptr;
}

int view_zp(const llmoc_int4_view& W) { return W.awq_zp > 0 ? W.awq_zp : 7; }

// ensure_int4_resident (cuda_backend.cpp:604-688), caller holds g_mu.
Resident* ensure_resident(const llmoc_int4_view* Wp) {
  if (!g_enabled) {
    t_err = "CUDA backend not enabled";
    return nullptr;
  }
  if (!Wp || !Wp->qweight || !Wp->scales) {
    t_err = "null INT4 view";
    return nullptr;
  }
  const llmoc_int4_view& W = *Wp;
  std::string why;
  const int gs = W.group_size > 0 ? W.group_size : 128;
  if (!shape_ok(W.M, W.K, gs, &why)) {
    t_err = why;
    return nullptr;
  }
  auto it = g_cache.find(W.qweight);
  if (it != g_cache.end()) {
    if (it->second.geo.M != W.M || it->second.geo.K != W.K) {
      t_err = "resident weight shape mismatch for the same qweight pointer";
      return nullptr;
    }
    it->second.last_use = ++g_tick;
    return &it->second;
  }
  const bool awq = W.scheme == LLMOC_SCHEME_AWQ_SYM;
  const Geo g = make_geo(W.M, W.K, gs, !awq && W.zeros);
  const size_t total = g.total() + sizeof(ExpertDev);
  if (g_budget > 0 && g_used + total > g_budget) {
    std::vector<std::pair<uint64_t, const void*>> items;
    for (auto& kv : g_cache)
      if (!kv.second.pinned) items.push_back({kv.second.last_use, kv.first});
    std::sort(items.begin(), items.end());
    for (auto& p : items) {
      if (g_used + total <= g_budget) break;
      auto e = g_cache.find(p.second);
      g_used -= e->second.bytes;
      free_resident(e->second);
      g_cache.erase(e);
    }
    if (g_used + total > g_budget) {
      t_err = "VRAM budget exhausted";
      return nullptr;
    }
  }
  Resident r;
  r.geo = g;
  r.scheme = awq ? LLMOC_SCHEME_AWQ_SYM : LLMOC_SCHEME_GPTQ_ASYM;
  r.zp = view_zp(W);
  r.bytes = total;
  if (!cuda_ok(cudaMalloc(&r.buf, g.total()), "cudaMalloc(weights)")) return nullptr;
  if (!cuda_ok(cudaMalloc(&r.table, sizeof(ExpertDev)), "cudaMalloc(table)")) {
    free_resident(r);
    return nullptr;
  }
  if (!repack_into(W, false, g, r.buf, g_stream, &r.dev)) {
    cudaStreamSynchronize(g_stream);
    free_resident(r);
    return nullptr;
  }
  ExpertDev ed;
  ed.gate = ed.up = ed.down = r.dev;
  if (!cuda_ok(cudaMemcpyAsync(r.table, &ed, sizeof ed, cudaMemcpyHostToDevice, g_stream),
               "H2D table") ||
      !cuda_ok(cudaStreamSynchronize(g_stream), "upload")) {
    free_resident(r);
    return nullptr;
  }
  r.last_use = ++g_tick;
  g_used += total;
  auto res = g_cache.emplace(W.qweight, r);
  return &res.first->second;
}

// Growable device scratch for the host-pointer entry points.
struct Scratch {
  char* p = nullptr;
  size_t cap = 0;
  bool ensure(size_t n) {
    if (n <= cap) return true;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    if (!cuda_ok(cudaMalloc(&p, n), "cudaMalloc(scratch)")) return false;
    cap = n;
    return true;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
} g_scratch;

// Dense Y[n,M] = X[n,K] . W^T through the CUDA-core fp32 kernel; X, Y host.
// With `am` (n = 1, Y unused): only the argmax of y comes back (index, value).
struct ArgmaxOut {
  int32_t* index;
  float* value;
};
int dense_gemm_host(const float* X, int n, const llmoc_int4_view* W, float* Y, const ArgmaxOut* am = nullptr) {
  if (!X || (!Y && !am) || n <= 0 || (am && n != 1)) return fail("bad arguments");
  Resident* r = ensure_resident(W);
  if (!r) return 0;
  const Geo& g = r->geo;
  const int nwork = (n + kChunkRows - 1) / kChunkRows;
  const size_t xb = align256((size_t)n * g.K * 4), yb = align256((size_t)n * g.M * 4);
  const size_t wb = align256((size_t)nwork * sizeof(WorkItem) + 16);
  if (!g_scratch.ensure(xb + yb + wb + 256)) return 0;
  char* p = g_scratch.p;
  float* dX = (float*)p;
  float* dY = (float*)(p + xb);
  WorkItem* dW = (WorkItem*)(p + xb + yb);
  int* dN = (int*)(dW + nwork);
  unsigned long long* dKey = (unsigned long long*)(p + xb + yb + wb);
  std::vector<WorkItem> work(nwork);
  for (int i = 0; i < nwork; ++i) work[i] = WorkItem{0, i * kChunkRows, std::min(kChunkRows, n - i * kChunkRows), 0};
  cudaStream_t st = g_stream;
  if (!cuda_ok(cudaMemcpyAsync(dX, X, (size_t)n * g.K * 4, cudaMemcpyHostToDevice, st), "H2D x") ||
      !cuda_ok(cudaMemcpyAsync(dW, work.data(), nwork * sizeof(WorkItem), cudaMemcpyHostToDevice, st), "H2D work") ||
      !cuda_ok(cudaMemcpyAsync(dN, &nwork, sizeof(int), cudaMemcpyHostToDevice, st), "H2D n"))
    return 0;
  GemmArgs a{};
  a.experts = r->table;
  a.proj = 0;
  a.M = g.M;
  a.K = g.K;
  a.Kc = g.Kc;
  a.gs = g.gs;
  a.ng = g.ng;
  a.zp = r->zp;
  a.B = dX;
  a.ldb = g.K;
  a.gather = nullptr;
  a.kk = 1;
  a.work = dW;
  a.n_work = dN;
  a.out = dY;
  a.ldo = g.M;
  a.keep_nonfinite = am ? 1 : 0;  // the argmax maps non-finite rows to -1e30, not 0
  if (!cuda_ok(launch_gemm(MODE_PLAIN_F32, 1, a, nwork, r->scheme == LLMOC_SCHEME_AWQ_SYM, 1, st),
               "gemm launch"))
    return 0;
  count_launch();
  if (am) {
    unsigned long long key = 0;
    if (!cuda_ok(launch_argmax_rows(dY, g.M, dKey, st), "argmax launch") ||
        !cuda_ok(cudaMemcpyAsync(&key, dKey, sizeof(key), cudaMemcpyDeviceToHost, st), "D2H argmax") ||
        !cuda_ok(cudaStreamSynchronize(st), "gemm argmax"))
      return 0;
    count_launch();
    argmax_decode(key, am->index, am->value);
    return 1;
  }
  if (!cuda_ok(cudaMemcpyAsync(Y, dY, (size_t)n * g.M * 4, cudaMemcpyDeviceToHost, st), "D2H y") ||
      !cuda_ok(cudaStreamSynchronize(st), "gemm"))
    return 0;
  return 1;
}

}  // namespace

// =================================================================== layer

struct llmoc_moe_layer {
  llmoc_moe_layer_desc d{};
  int device = 0;
  int n_exp = 0;  // routed + shared experts held by this layer object
  int kk = 0;     // slots per token
  int ep_rank = 0, ep_world = 1;  // expert parallelism: this rank holds experts e % ep_world == ep_rank
  int e_loc = 0;                  // routed experts held (n_experts / ep_world), as local ids e / ep_world
  Geo gu, dn;     // gate/up [I,H] and down [H,I] geometry
  char* arena = nullptr;
  size_t weight_bytes = 0;    // packed q + scales (+zeros), as streamed
  ExpertDev* table = nullptr; // device [n_exp]
  void* wmaps = nullptr;      // device TMA maps of the weights (tcgen05 path), or null
  std::vector<ExpertDev> htable;
  uint16_t* router_w = nullptr;   // device [E (+1: the shared expert's gate row, when set)][H] bf16
  int shared_gate = 0;            // router_w holds the shared gate row (llmoc_moe_layer_set_shared_gate)
  float* bias = nullptr;
  long long wait_cycles = llmoc::kDefaultWaitCycles;  // budget of the fused decode kernel's barrier waits
  // stage timing (llmoc_moe_set_stage_timing): 7 events per timed call
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::array<cudaEvent_t, 7>> ev_calls;
};

namespace {

// Rows per work item for `pairs` (row, expert) pairs over `groups` experts:
// decode-size groups (about 8 pairs per expert or fewer) use one mma N tile (8
// rows), so that kernel variant has no per-tile branches; groups of up to
// kSmallAvg pairs on average use kUmmaSmallRows-row items (the tcgen05 kernel
// with several MMA issuers per tile); larger ones kUmmaRows-row items (or, on
// shapes the tensor-core kernels do not take, the CUDA-core kernel, which
// walks any item length).
constexpr long kSmallAvg = 40;
int chunk_for_rows(long pairs, int groups) {
  const long g = std::max(1, groups);
  if (pairs <= 8 * g + g / 2) return 8;
  return pairs <= kSmallAvg * g ? kUmmaSmallRows : kUmmaRows;
}
// A forward over T tokens: T <= 128 keeps the 8-row items (the decode GEMMs)
int chunk_rows(const llmoc_moe_layer* L, int T) {
  return T <= 128 ? 8 : ((long)T * L->kk <= kSmallAvg * L->n_exp ? kUmmaSmallRows : kUmmaRows);
}

struct WsLayout {
  size_t logits, ids, weights, offsets, sorted, inverse, work, n_work, n_active, err, mid, partial,
      xs, xh, xsum, xscale, bar, sig, total;
  int max_work;
};

// The tcgen05 prefill GEMMs run when K of both GEMMs is a multiple of 128, the
// group is 32/64/128 wide (every BASELINE shape) and the items are kUmmaRows rows.
bool tc_shapes(const llmoc_moe_layer* L) {
  const int gs = L->d.group_size;
  return L->d.hidden % 128 == 0 && L->d.inter % 128 == 0 && (gs == 32 || gs == 64 || gs == 128);
}

// A layer with tensor-core shapes always holds its weight maps (creation
// fails without them), so its kUmmaSmallRows- and kUmmaRows-row items always
// take the tcgen05 kernel: the register-fed kernel handles at most 8 rows per item.
bool use_umma_c(const llmoc_moe_layer* L, int chunk) {
  return tc_shapes(L) && L->wmaps && (chunk == kUmmaRows || chunk == kUmmaSmallRows);
}

// Workspace of one grouped run over T rows with kk slots each, permuted over
// n_perm groups; `logits` adds the router's [T, n_experts] logits.
WsLayout ws_layout_g(const llmoc_moe_layer* L, int T, int kk, int n_perm, int chunk, bool logits) {
  WsLayout w{};
  const size_t n = (size_t)T * kk;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes);
    return at;
  };
  w.max_work = (int)(std::min<size_t>((size_t)n_perm, n) + (n + chunk - 1) / chunk);
  w.logits = logits ? take((size_t)T * (L->d.n_experts + L->shared_gate) * 4) : 0;
  w.ids = take(n * 4);
  w.weights = take(n * 4);
  w.offsets = take((size_t)(n_perm + 1) * 4);
  w.sorted = take(n * 4);
  w.inverse = take(n * 4);
  w.work = take((size_t)std::max(1, w.max_work) * sizeof(WorkItem));
  w.n_work = take(4);
  w.n_active = take(4);
  w.err = take(4 * (1 + kGemmCounters));  // error word, then the GEMM unit counters
  w.mid = take(n * L->d.inter * 2);
  w.partial = take(n * L->d.hidden * 4);
  w.xs = use_umma_c(L, chunk) ? take(n * L->d.hidden * 2) : 0;  // rows in expert-sorted order
  if (tc_shapes(L) && !use_umma_c(L, chunk)) {  // decode gate/up: fp16 rows, group sums, row scales
    w.xh = take((size_t)T * L->d.hidden * 2);
    w.xsum = take((size_t)T * (L->d.hidden / L->d.group_size) * 4);
    w.xscale = take((size_t)T * 4);
  }
  // the fused single-token kernel's barrier words (a whole-layer forward of one token)
  w.bar = logits && T == 1 ? take(24) : 0;
  w.sig = logits && T == 1 ? take((size_t)(L->d.n_experts + L->shared_gate) * 4) : 0;  // sigmoid scores
  w.total = o;
  return w;
}

WsLayout ws_layout(const llmoc_moe_layer* L, int T) {
  return ws_layout_g(L, T, L->kk, L->n_exp, chunk_rows(L, T), true);
}

llmoc_status validate_desc(const llmoc_moe_layer_desc* d) {
  if (!d) return fails(LLMOC_ERR_INVALID, "null layer desc");
  if (d->hidden <= 0 || d->inter <= 0 || d->n_experts <= 0 || d->topk <= 0)
    return fails(LLMOC_ERR_INVALID, "non-positive layer dimension");
  if (d->topk > kMaxTopk || d->topk > d->n_experts)
    return fails(LLMOC_ERR_INVALID, "topk must be <= 64 and <= n_experts");
  if (d->n_experts > kMaxExperts)
    return fails(LLMOC_ERR_UNSUPPORTED, "more than 511 routed experts per layer");
  if (d->router != LLMOC_ROUTER_SOFTMAX && d->router != LLMOC_ROUTER_SIGMOID_BIAS)
    return fails(LLMOC_ERR_INVALID, "unknown router");
  if (d->scheme != LLMOC_SCHEME_AWQ_SYM && d->scheme != LLMOC_SCHEME_GPTQ_ASYM)
    return fails(LLMOC_ERR_INVALID, "unknown INT4 scheme");
  std::string why;
  if (!shape_ok(d->inter, d->hidden, d->group_size, &why) ||
      !shape_ok(d->hidden, d->inter, d->group_size, &why))
    return fails(LLMOC_ERR_UNSUPPORTED, why);
  if (d->hidden % 8 != 0) return fails(LLMOC_ERR_UNSUPPORTED, "hidden must be a multiple of 8");
  return LLMOC_OK;
}

bool view_matches(const llmoc_int4_view& v, int M, int K, const llmoc_moe_layer_desc* d) {
  const int gs = v.group_size > 0 ? v.group_size : 128;
  const int scheme = v.scheme == LLMOC_SCHEME_AWQ_SYM ? LLMOC_SCHEME_AWQ_SYM : LLMOC_SCHEME_GPTQ_ASYM;
  return v.qweight && v.scales && v.M == M && v.K == K && gs == d->group_size && scheme == d->scheme &&
         (scheme == LLMOC_SCHEME_AWQ_SYM || v.zeros);
}

// world > 1: an expert-parallel shard holding the routed experts e with
// e % world == rank (local id e / world), the router and the shared expert.
llmoc_status layer_create(const llmoc_moe_layer_desc* d, const uint16_t* router_w, const float* bias,
                          const llmoc_int4_view* experts, const llmoc_int4_view* shared, int device,
                          bool on_device, llmoc_moe_layer** out, int rank = 0, int world = 1) {
  if (!out) return fails(LLMOC_ERR_INVALID, "null out");
  *out = nullptr;
  llmoc_status s = validate_desc(d);
  if (s != LLMOC_OK) return s;
  if (!router_w || !experts) return fails(LLMOC_ERR_INVALID, "null router or experts");
  if (d->router == LLMOC_ROUTER_SIGMOID_BIAS && !bias)
    return fails(LLMOC_ERR_INVALID, "sigmoid router needs a bias");
  if (d->has_shared && !shared) return fails(LLMOC_ERR_INVALID, "has_shared without shared views");
  const int E = d->n_experts, H = d->hidden, I = d->inter;
  if (world < 1 || rank < 0 || rank >= world || E % world != 0)
    return fails(LLMOC_ERR_INVALID, "expert parallelism needs 0 <= rank < world and n_experts % world == 0");
  const int e_loc = E / world;
  const int n_exp = e_loc + (d->has_shared ? 1 : 0);
  auto view_of = [&](int e) { return e < e_loc ? experts + 3 * ((size_t)e * world + rank) : shared; };
  for (int e = 0; e < n_exp; ++e) {
    const llmoc_int4_view* v = view_of(e);
    if (!view_matches(v[0], I, H, d) || !view_matches(v[1], I, H, d) || !view_matches(v[2], H, I, d))
      return fails(LLMOC_ERR_INVALID, "expert " + std::to_string(e) + " view does not match the layer");
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fails(LLMOC_ERR_NO_DEVICE, "no such CUDA device");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  auto* L = new llmoc_moe_layer();
  L->d = *d;
  if (L->d.awq_zp <= 0) L->d.awq_zp = 7;
  L->device = device;
  L->n_exp = n_exp;
  L->kk = d->topk + (d->has_shared ? 1 : 0);
  L->ep_rank = rank;
  L->ep_world = world;
  L->e_loc = e_loc;
  const bool z = d->scheme == LLMOC_SCHEME_GPTQ_ASYM;
  L->gu = make_geo(I, H, d->group_size, z);
  L->dn = make_geo(H, I, d->group_size, z);
  const size_t per_exp = 2 * L->gu.total() + L->dn.total();
  L->weight_bytes = (size_t)n_exp * (2 * (L->gu.qbytes + L->gu.sbytes + L->gu.zbytes) +
                                     (L->dn.qbytes + L->dn.sbytes + L->dn.zbytes));
  cudaStream_t st = nullptr;
  llmoc_status rc = LLMOC_OK;
  auto bail = [&](llmoc_status code, const std::string& msg) {
    rc = fails(code, msg);
    return rc;
  };
  do {
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
      bail(LLMOC_ERR_CUDA, "stream create");
      break;
    }
    if (cudaMalloc(&L->arena, per_exp * n_exp) != cudaSuccess) {
      bail(LLMOC_ERR_NO_MEMORY, "cudaMalloc(expert arena) failed");
      break;
    }
    if (cudaMalloc(&L->table, sizeof(ExpertDev) * n_exp) != cudaSuccess ||
        cudaMalloc(&L->router_w, (size_t)E * H * 2) != cudaSuccess) {
      bail(LLMOC_ERR_NO_MEMORY, "cudaMalloc(router/table) failed");
      break;
    }
    if (bias && cudaMalloc(&L->bias, (size_t)E * 4) != cudaSuccess) {
      bail(LLMOC_ERR_NO_MEMORY, "cudaMalloc(bias) failed");
      break;
    }
    const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    if (cudaMemcpyAsync(L->router_w, router_w, (size_t)E * H * 2, kind, st) != cudaSuccess ||
        (bias && cudaMemcpyAsync(L->bias, bias, (size_t)E * 4, kind, st) != cudaSuccess)) {
      bail(LLMOC_ERR_CUDA, "router upload failed");
      break;
    }
    L->htable.resize(n_exp);
    char* p = L->arena;
    for (int e = 0; e < n_exp && rc == LLMOC_OK; ++e) {
      const llmoc_int4_view* v = view_of(e);
      ExpertDev& ed = L->htable[e];
      if (!repack_into(v[0], on_device, L->gu, p, st, &ed.gate)) bail(LLMOC_ERR_CUDA, t_err);
      p += L->gu.total();
      if (rc == LLMOC_OK && !repack_into(v[1], on_device, L->gu, p, st, &ed.up)) bail(LLMOC_ERR_CUDA, t_err);
      p += L->gu.total();
      if (rc == LLMOC_OK && !repack_into(v[2], on_device, L->dn, p, st, &ed.down)) bail(LLMOC_ERR_CUDA, t_err);
      p += L->dn.total();
    }
    if (rc != LLMOC_OK) break;
    if (cudaMemcpyAsync(L->table, L->htable.data(), sizeof(ExpertDev) * n_exp,
                        cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
      bail(LLMOC_ERR_CUDA, std::string("layer upload: ") + cudaGetErrorString(cudaGetLastError()));
      break;
    }
    if (tc_shapes(L)) {  // TMA maps of the resident weights for the tcgen05 prefill GEMMs
      std::vector<unsigned char> maps((size_t)n_exp * kMapsPerExpert * kTensorMapBytes);
      if (!build_umma_weight_maps(L->htable.data(), n_exp, I, H, d->group_size, z, maps.data())) {
        bail(LLMOC_ERR_CUDA, "cuTensorMapEncodeTiled refused a weight tensor map");
        break;
      }
      if (cudaMalloc(&L->wmaps, maps.size()) != cudaSuccess ||
          cudaMemcpy(L->wmaps, maps.data(), maps.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        bail(LLMOC_ERR_NO_MEMORY, "weight tensor maps");
        break;
      }
    }
  } while (false);
  if (st) {
    cudaStreamSynchronize(st);
    cudaStreamDestroy(st);
  }
  cudaSetDevice(prev);
  if (rc != LLMOC_OK) {
    llmoc_moe_layer_destroy(L);
    return rc;
  }
  *out = L;
  return LLMOC_OK;
}

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
    else prev = -1;
  }
  ~DevGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Event recorder for one timed forward (no-op when timing is off).
struct StageEvents {
  llmoc_moe_layer* L = nullptr;
  std::array<cudaEvent_t, 7> ev{};
  int next = 0;
  StageEvents(const llmoc_moe_layer* layer) {
    if (!layer->timing) return;
    L = const_cast<llmoc_moe_layer*>(layer);
    for (auto& e : ev) {
      if (!L->ev_pool.empty()) {
        e = L->ev_pool.back();
        L->ev_pool.pop_back();
      } else if (cudaEventCreate(&e) != cudaSuccess) {
        e = nullptr;
      }
    }
  }
  void mark(cudaStream_t st) {
    if (L && next < 7 && ev[next]) cudaEventRecord(ev[next], st);
    ++next;
  }
  void commit() {
    if (L && next == 7) {
      L->ev_calls.push_back(ev);
      L = nullptr;
    }
  }
  ~StageEvents() {
    if (L)
      for (auto e : ev)
        if (e) L->ev_pool.push_back(e);
  }
};

PermArgs perm_args(const int* ids, int n, int n_perm, int chunk, const WsLayout& w, char* ws) {
  PermArgs pa{};
  pa.ids = ids;
  pa.n = n;
  pa.n_exp = n_perm;
  pa.offsets = (int*)(ws + w.offsets);
  pa.sorted = (int*)(ws + w.sorted);
  pa.inverse = (int*)(ws + w.inverse);
  pa.work = (WorkItem*)(ws + w.work);
  pa.n_work = (int*)(ws + w.n_work);
  pa.n_active = (int*)(ws + w.n_active);
  pa.err = (int*)(ws + w.err);
  pa.chunk = chunk;
  return pa;
}

// Segments (seg_len > 0): ids are n_seg regions of seg_len slots, the first
// seg_count[s * seg_stride] of each occupied (PermArgs).
struct PermSegs {
  const int* count = nullptr;
  int stride = 0, len = 0, n = 0;
  FlagWait wait;  // the sources' flags, waited for by the permutation kernel itself
};

llmoc_status run_permute(const int* ids, int n, int n_perm, int chunk, const WsLayout& w, char* ws,
                         cudaStream_t st, const PermSegs& segs = PermSegs{}) {
  PermArgs pa = perm_args(ids, n, n_perm, chunk, w, ws);
  pa.seg_count = segs.count;
  pa.seg_stride = segs.stride;
  pa.seg_len = segs.len;
  pa.n_seg = segs.n;
  pa.wait = segs.wait;
  if (!cuda_ok(launch_permute(pa, st), "permute")) return LLMOC_ERR_CUDA;
  count_launch(1);
  return LLMOC_OK;
}

llmoc_status run_route(const llmoc_moe_layer* L, const uint16_t* X, int T, const WsLayout& w,
                       char* ws, cudaStream_t st, StageEvents* se = nullptr) {
  const int E = L->d.n_experts, H = L->d.hidden;
  float* logits = (float*)(ws + w.logits);
  if (se) se->mark(st);
  // the decode gate/up GEMM's fp16 rows: made by the router (its copy of the
  // tokens; the bf16 kernels, H % 256 == 0, T < 128) or else by the top-k warps
  const bool xh_router = w.xh && T < 128 && H % 256 == 0;
  XhOut xo{};
  if (xh_router) {
    xo.xh = ws + w.xh;
    xo.xsum = (float*)(ws + w.xsum);
    xo.xscale = (float*)(ws + w.xscale);
    xo.gs = L->d.group_size;
  }
  if (!cuda_ok(launch_router_logits(X, false, L->router_w, T, E + L->shared_gate, H, logits, st, xo), "router"))
    return LLMOC_ERR_CUDA;
  if (se) se->mark(st);
  TopkArgs ta{};
  ta.logits = logits;
  ta.bias = L->bias;
  ta.T = T;
  ta.E = E;
  ta.k = L->d.topk;
  ta.kk = L->kk;
  ta.router = L->d.router;
  ta.routed_scaling = L->d.routed_scaling;
  ta.shared_scale = L->d.shared_scale;
  ta.has_shared = L->d.has_shared;
  ta.ld = E + L->shared_gate;
  ta.shared_gate = L->shared_gate;
  ta.ids = (int*)(ws + w.ids);
  ta.weights = (float*)(ws + w.weights);
  if (w.xh && !xh_router) {  // decode-size forward: the top-k warps make the gate/up GEMM's fp16 rows
    ta.x = X;
    ta.H = H;
    ta.gs = L->d.group_size;
    ta.xh = ws + w.xh;
    ta.xsum = (float*)(ws + w.xsum);
    ta.xscale = (float*)(ws + w.xscale);
  }
  count_launch(1);
  if (T <= kFusedRouteMaxT && L->n_exp <= kMaxExpPerm) {  // one CTA: top-k + permutation
    const PermArgs pa = perm_args(ta.ids, T * L->kk, L->n_exp, chunk_rows(L, T), w, ws);
    if (!cuda_ok(launch_topk_permute(ta, pa, st), "topk+permute")) return LLMOC_ERR_CUDA;
    count_launch(1);
    if (se) se->mark(st);
    if (se) se->mark(st);
    return LLMOC_OK;
  }
  if (!cuda_ok(launch_topk(ta, st), "topk")) return LLMOC_ERR_CUDA;
  if (se) se->mark(st);
  count_launch(1);
  llmoc_status rc = run_permute(ta.ids, T * L->kk, L->n_exp, chunk_rows(L, T), w, ws, st);
  if (se) se->mark(st);
  return rc;
}

// Grouped expert FFN over R rows of X (kk slots per row, expert ids and weights
// in the workspace, already permuted): gather (tcgen05 path), gate/up +
// SiLU*mul, down; then, when Y is given, the weighted sum of each row's kk
// slots into Y (bf16; `weights` null = 1).
llmoc_status run_ffn(const llmoc_moe_layer* L, const uint16_t* X, int R, int kk, int chunk, const WsLayout& w,
                     char* ws, uint16_t* Y, const float* weights, cudaStream_t st, StageEvents* se = nullptr,
                     const uint16_t* residual = nullptr, int expect_pairs = 0, bool xh_ready = false) {
  const int H = L->d.hidden, I = L->d.inter;
  const bool awq = L->d.scheme == LLMOC_SCHEME_AWQ_SYM;
  // tensor cores when K of both GEMMs is a multiple of 128 and the group is
  // 32/64/128 wide (every BASELINE shape); the CUDA-core kernel otherwise
  const bool tc = tc_shapes(L);
  const int path = tc ? 0 : 2;
  const bool umma = use_umma_c(L, chunk);
  const int n_pairs = R * kk;
  // rows expected to be occupied (padded receive slots: fewer than R * kk)
  const int n_expect = expect_pairs > 0 ? std::min(expect_pairs, n_pairs) : n_pairs;
  const int n_groups = std::min(n_expect, L->n_exp);  // experts (groups) the pairs can reach
  const int grid_items = n_groups + (n_expect + chunk - 1) / chunk;  // work items expected
  if (umma) {
    if (!cuda_ok(launch_gather_rows(X, H, (const int*)(ws + w.sorted), kk, n_pairs,
                                    (const int*)(ws + w.offsets) + L->n_exp, ws + w.xs, st),
                 "gather"))
      return LLMOC_ERR_CUDA;
    count_launch(1);
  }
  const int ntiles = std::min(4, chunk / 8);
  GemmArgs a{};
  a.experts = L->table;
  a.M = I;
  a.K = H;
  a.Kc = L->gu.Kc;
  a.gs = L->d.group_size;
  a.ng = L->gu.ng;
  a.zp = L->d.awq_zp;
  a.B = X;
  a.ldb = H;
  a.gather = (const int*)(ws + w.sorted);
  a.kk = kk;
  a.work = (const WorkItem*)(ws + w.work);
  a.n_work = (const int*)(ws + w.n_work);
  a.out = ws + w.mid;
  a.ldo = I;
  a.out_bf16 = 1;
  a.err = (int*)(ws + w.err);
  a.wmaps = L->wmaps;
  a.ctr = (int*)(ws + w.err) + 1;
  if (umma) {  // B = the gathered rows, read by TMA
    a.B = ws + w.xs;
    a.gather = nullptr;
  } else if (path == 0) {
    // decode gate/up on fp16 rows: each row scaled by a power of two, rounded to
    // fp16, with its per-group sums -- made by the top-k warps of this forward
    // (xh_ready), else here (kk == 1: only the rows the permutation placed,
    // e.g. an expert-parallel owner's occupied receive slots)
    if (!xh_ready) {
      if (!cuda_ok(launch_prep_xh(X, R, H, L->d.group_size, kk == 1 ? (const int*)(ws + w.sorted) : nullptr,
                                  (const int*)(ws + w.offsets) + L->n_exp, ws + w.xh, (float*)(ws + w.xsum),
                                  (float*)(ws + w.xscale), st),
                   "fp16 rows"))
        return LLMOC_ERR_CUDA;
      count_launch(1);
    }
    a.B = ws + w.xh;
    a.bsum = (const float*)(ws + w.xsum);
    a.bscale = (const float*)(ws + w.xscale);
  }
  if (!cuda_ok(umma ? launch_gemm_umma(MODE_GATE_UP, a, w.max_work, awq, n_pairs, chunk, st)
                    : launch_gemm(MODE_GATE_UP, path, a, w.max_work, awq, ntiles, st, n_groups, grid_items),
               "gate/up"))
    return LLMOC_ERR_CUDA;
  if (se) se->mark(st);
  GemmArgs b = a;
  b.bsum = nullptr;  // the down GEMM reads mid (bf16) through its all-ones MMA
  b.bscale = nullptr;
  b.proj = 2;
  b.M = H;
  b.K = I;
  b.Kc = L->dn.Kc;
  b.ng = L->dn.ng;
  b.B = ws + w.mid;
  b.ldb = I;
  b.gather = nullptr;
  b.out = ws + w.partial;
  b.ldo = H;
  b.ctr = (int*)(ws + w.err) + 2;
  if (!cuda_ok(umma ? launch_gemm_umma(MODE_PLAIN_F32, b, w.max_work, awq, n_pairs, chunk, st)
                    : launch_gemm(MODE_PLAIN_F32, path, b, w.max_work, awq, ntiles, st, n_groups, grid_items),
               "down"))
    return LLMOC_ERR_CUDA;
  if (se) se->mark(st);
  count_launch(2);
  if (Y) {
    if (!cuda_ok(launch_combine((const float*)(ws + w.partial), (const int*)(ws + w.inverse), weights, R, kk, H, Y,
                                1, 0, st, residual),
                 "combine"))
      return LLMOC_ERR_CUDA;
    count_launch(1);
  }
  if (se) se->mark(st);
  return LLMOC_OK;
}

// The fused single-token kernel takes a whole-layer forward of one token when
// the layer has the decode GEMMs' shapes (tc_shapes), the router's rows are a
// multiple of 256 wide and the slots fit its work list.
bool decode1_ok(const llmoc_moe_layer* L) {
  return tc_shapes(L) && L->d.hidden % 256 == 0 && L->kk <= kDecode1MaxSlots && L->d.n_experts <= kMaxExperts;
}

// Distinct per launch of the fused kernel in this process (its barrier tags).
std::atomic<unsigned long long> g_decode1_epoch{0};

// One token through the layer in one launch (k_moe_decode1): the same
// routing outputs in the workspace as run_route, the same rows in mid /
// partial as run_ffn, y (+ the residual) as the combine.
llmoc_status run_decode1(const llmoc_moe_layer* L, const uint16_t* X, const uint16_t* R, uint16_t* Y,
                         const WsLayout& w, char* ws, cudaStream_t st, StageEvents* se) {
  const int E = L->d.n_experts, H = L->d.hidden, I = L->d.inter;
  Decode1Args a{};
  a.X = (const __nv_bfloat16*)X;
  a.Wr = L->router_w;
  a.rows = E + L->shared_gate;
  a.H = H;
  a.logits = (float*)(ws + w.logits);
  TopkArgs& ta = a.ta;
  ta.logits = a.logits;
  ta.bias = L->bias;
  ta.T = 1;
  ta.E = E;
  ta.k = L->d.topk;
  ta.kk = L->kk;
  ta.ld = E + L->shared_gate;
  ta.router = L->d.router;
  ta.routed_scaling = L->d.routed_scaling;
  ta.shared_scale = L->d.shared_scale;
  ta.has_shared = L->d.has_shared;
  ta.shared_gate = L->shared_gate;
  ta.ids = (int*)(ws + w.ids);
  ta.weights = (float*)(ws + w.weights);
  a.sig = L->d.router == LLMOC_ROUTER_SIGMOID_BIAS ? (float*)(ws + w.sig) : nullptr;
  ta.sig = a.sig;
  GemmArgs& g = a.gu;
  g.experts = L->table;
  g.proj = 0;
  g.M = I;
  g.K = H;
  g.Kc = L->gu.Kc;
  g.gs = L->d.group_size;
  g.ng = L->gu.ng;
  g.zp = L->d.awq_zp;
  g.B = X;  // the token's bf16 row (the kernel reads it for every slot)
  g.ldb = H;
  g.out = ws + w.mid;
  g.ldo = I;
  g.out_bf16 = 1;
  g.err = (int*)(ws + w.err);
  GemmArgs& d = a.dn;
  d = g;
  d.proj = 2;
  d.M = H;
  d.K = I;
  d.Kc = L->dn.Kc;
  d.ng = L->dn.ng;
  d.B = ws + w.mid;
  d.ldb = I;
  d.out = ws + w.partial;
  d.ldo = H;
  a.partial = (const float*)(ws + w.partial);
  a.Y = (__nv_bfloat16*)Y;
  a.R = (const __nv_bfloat16*)R;
  a.n_exp = L->n_exp;
  a.offsets = (int*)(ws + w.offsets);
  a.sorted = (int*)(ws + w.sorted);
  a.inverse = (int*)(ws + w.inverse);
  a.n_active = (int*)(ws + w.n_active);
  a.err = (int*)(ws + w.err);
  a.bar = (unsigned long long*)(ws + w.bar);
  a.epoch = ++g_decode1_epoch;
  a.budget = L->wait_cycles;
  // stage timing: the whole launch is reported as the gate/up stage
  for (int i = 0; i < 4; ++i)
    if (se) se->mark(st);
  const cudaError_t e = launch_decode1(a, L->d.scheme == LLMOC_SCHEME_AWQ_SYM, st);
  if (e == cudaErrorCooperativeLaunchTooLarge || e == cudaErrorNotSupported) {
    // the grid cannot be resident at once here (e.g. a client limited to part
    // of the GPU): nothing was launched, the caller runs the separate kernels
    (void)cudaGetLastError();
    return LLMOC_ERR_UNSUPPORTED;
  }
  if (!cuda_ok(e, "fused decode")) return LLMOC_ERR_CUDA;
  count_launch(1);
  for (int i = 0; i < 3; ++i)
    if (se) se->mark(st);
  return LLMOC_OK;
}

// Expert-parallel source-rank workspace (llmoc_moe_ep_dispatch, then
// llmoc_moe_ep_combine with the same workspace): routing of the T tokens over
// all n_experts (topk routed slots, no shared slot), the pairs ordered by
// (owner rank, owner-local expert, token, slot); then the shared expert's run
// over the T tokens.
struct EpSrcLayout {
  size_t logits, ids, weights, shw, key, offsets, sorted, inverse, work, n_work, n_active, err;
  size_t sh = 0;     // shared-expert grouped run (ws_layout_g with kk = 1)
  WsLayout shl{};
  int sh_chunk = 8;
  size_t total;
};
EpSrcLayout ep_src_layout(const llmoc_moe_layer* L, int T) {
  EpSrcLayout w{};
  const size_t n = (size_t)T * L->d.topk;
  const int E = L->d.n_experts;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes);
    return at;
  };
  const int max_work = (int)(std::min<size_t>((size_t)E, n) + (n + 7) / 8);
  w.logits = take((size_t)T * (E + L->shared_gate) * 4);
  w.ids = take(n * 4);
  w.weights = take(n * 4);
  w.shw = take((size_t)T * 4);  // per-token shared weights (shared gate)
  w.key = take(n * 4);
  w.offsets = take((size_t)(E + 1) * 4);
  w.sorted = take(n * 4);
  w.inverse = take(n * 4);
  w.work = take((size_t)std::max(1, max_work) * sizeof(WorkItem));
  w.n_work = take(4);
  w.n_active = take(4);
  w.err = take(4 * (1 + kGemmCounters));  // error word, then the GEMM unit counters
  if (L->d.has_shared) {
    w.sh_chunk = chunk_for_rows(T, 1);
    w.shl = ws_layout_g(L, T, 1, L->n_exp, w.sh_chunk, false);
    w.sh = take(w.shl.total);
  }
  w.total = o;
  return w;
}
// owner-rank workspace for `rows` received rows (the larger of the two item sizes)
size_t ep_owner_bytes(const llmoc_moe_layer* L, int rows) {
  size_t b = 0;
  for (int chunk : {8, kUmmaSmallRows, kUmmaRows}) b = std::max(b, ws_layout_g(L, rows, 1, L->n_exp, chunk, false).total);
  return b;
}

// Workspace of one NVLink expert-parallel step on a rank: the source side
// (routing, send rows, ids, counts) and the owner side (the grouped run over
// the padded receive slots), used in the same step.
struct EpP2PWs {
  size_t src, send_rows, send_expert, counts, own, total;
  EpSrcLayout sw;
};
EpP2PWs ep_p2p_ws(const llmoc_moe_layer* L, const llmoc_ep_transport* tr, int T);

}  // namespace

struct llmoc_ep_transport {
  int world = 1, rank = 0, device = 0, hidden = 0, max_tokens = 0, topk = 0;
  llmoc::EpP2PLayout lay{};
  char* base = nullptr;            // this rank's buffer (exported by CUDA IPC)
  std::vector<char*> peer;         // every rank's buffer as seen from here (own = base)
  std::vector<bool> opened;        // opened through CUDA IPC (closed at destroy)
  char** peers_dev = nullptr;      // device copy of `peer`
  int* ctr = nullptr;              // device: CTA counters of the two push kernels
  int* err = nullptr;              // device: bit 1 = a wait gave up
  long long wait_cycles = llmoc::kDefaultWaitCycles;  // budget of each bounded wait
  bool connected = false;
};

namespace {
EpP2PWs ep_p2p_ws(const llmoc_moe_layer* L, const llmoc_ep_transport* tr, int T) {
  EpP2PWs w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes);
    return at;
  };
  const size_t n = (size_t)T * L->d.topk, H = (size_t)L->d.hidden, slots = (size_t)tr->world * tr->lay.cap;
  w.sw = ep_src_layout(L, T);
  w.src = take(w.sw.total);
  w.send_rows = take(n * H * 2);
  w.send_expert = take(n * 4);
  w.counts = take((size_t)tr->world * 4);
  w.own = take(ep_owner_bytes(L, (int)slots));
  w.total = o;
  return w;
}
}  // namespace

// ===================================================================== ABI

extern "C" {

int llmoc_cuda_probe_available(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_probed) return g_available;
  g_probed = true;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    g_status = "no CUDA device";
    return 0;
  }
  cudaDeviceProp p{};
  if (cudaGetDeviceProperties(&p, 0) != cudaSuccess || p.major != 10) {
    g_status = "device 0 is not sm_100 (B200)";
    return 0;
  }
  g_ndev = n;
  g_available = true;
  g_status = std::string("available: ") + p.name;
  return 1;
}

int llmoc_cuda_enabled(void) { return g_enabled ? 1 : 0; }
const char* llmoc_cuda_status(void) { return g_status.c_str(); }
int llmoc_cuda_device_count(void) {
  llmoc_cuda_probe_available();
  return g_ndev;
}

int llmoc_cuda_enable(size_t vram_budget_bytes) {
  if (!llmoc_cuda_probe_available()) return fail(g_status);
  std::lock_guard<std::mutex> lk(g_mu);
  g_budget = vram_budget_bytes;
  if (g_enabled) return 1;
  if (!cuda_ok(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking), "stream create"))
    return 0;
  g_enabled = true;
  g_status = "enabled";
  return 1;
}

void llmoc_cuda_disable(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_enabled) return;
  cudaStreamSynchronize(g_stream);
  for (auto& kv : g_cache) free_resident(kv.second);
  g_cache.clear();
  g_used = 0;
  g_scratch.release();
  cudaStreamDestroy(g_stream);
  g_stream = nullptr;
  g_enabled = false;
  g_status = "disabled";
}

size_t llmoc_cuda_vram_used(void) { return g_used; }
size_t llmoc_cuda_vram_budget(void) { return g_budget; }
void llmoc_cuda_set_vram_budget(size_t bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_budget = bytes;
}
int llmoc_cuda_device_mem_info(size_t* free_bytes, size_t* total_bytes) {
  size_t f = 0, t = 0;
  if (cudaMemGetInfo(&f, &t) != cudaSuccess) {
    cudaGetLastError();
    return fail("cudaMemGetInfo failed");
  }
  if (free_bytes) *free_bytes = f;
  if (total_bytes) *total_bytes = t;
  return 1;
}
int llmoc_cuda_host_register(void* ptr, size_t bytes) {
  if (!ptr || !bytes) return fail("bad arguments");
  return cuda_ok(cudaHostRegister(ptr, bytes, cudaHostRegisterPortable), "cudaHostRegister") ? 1 : 0;
}
int llmoc_cuda_host_unregister(void* ptr) {
  if (!ptr) return fail("bad arguments");
  return cuda_ok(cudaHostUnregister(ptr), "cudaHostUnregister") ? 1 : 0;
}
const char* llmoc_last_error(void) { return t_err.c_str(); }

int llmoc_try_gemm_int4(const float* x, const llmoc_int4_view* W, float* y) {
  std::lock_guard<std::mutex> lk(g_mu);
  return dense_gemm_host(x, 1, W, y);
}

int llmoc_try_gemm_int4_argmax(const float* x, const llmoc_int4_view* W, int32_t* index, float* value) {
  if (!x || !W || !index || !value || W->M <= 0) return fail("bad arguments");
  std::lock_guard<std::mutex> lk(g_mu);
  const ArgmaxOut am{index, value};
  return dense_gemm_host(x, 1, W, nullptr, &am);
}

int llmoc_try_gemm_int4_batch(const float* X, int n, const llmoc_int4_view* W, float* Y) {
  std::lock_guard<std::mutex> lk(g_mu);
  return dense_gemm_host(X, n, W, Y);
}

int llmoc_try_gemm_int4_multi(const float* x, const llmoc_int4_view* const* Ws, float* const* ys,
                              int n) {
  if (!Ws || !ys || n < 1 || n > 4) return fail("try_gemm_int4_multi takes 1..4 weights");
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < n; ++i)
    if (!Ws[i] || Ws[i]->K != Ws[0]->K) return fail("weights must share K");
  for (int i = 0; i < n; ++i)
    if (!dense_gemm_host(x, 1, Ws[i], ys[i])) return 0;
  return 1;
}

int llmoc_try_gemm_int4_batch_multi(const float* X, int n, const llmoc_int4_view* const* Ws,
                                    float* const* Ys, int nW) {
  if (!Ws || !Ys || nW < 1 || nW > 4) return fail("try_gemm_int4_batch_multi takes 1..4 weights");
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < nW; ++i)
    if (!dense_gemm_host(X, n, Ws[i], Ys[i])) return 0;
  return 1;
}

int llmoc_prefetch_int4_weight(const llmoc_int4_view* W) {
  std::lock_guard<std::mutex> lk(g_mu);
  return ensure_resident(W) ? 1 : 0;
}

int llmoc_pin_int4_weight(const llmoc_int4_view* W) {
  std::lock_guard<std::mutex> lk(g_mu);
  Resident* r = ensure_resident(W);
  if (!r) return 0;
  r->pinned = true;
  return 1;
}

int llmoc_try_dequant_int4_matrix(const llmoc_int4_view* W, float* out) {
  if (!out) return fail("null out");
  std::lock_guard<std::mutex> lk(g_mu);
  Resident* r = ensure_resident(W);
  if (!r) return 0;
  const size_t bytes = (size_t)r->geo.M * r->geo.K * 4;
  if (!g_scratch.ensure(bytes)) return 0;
  if (!cuda_ok(launch_dequant(r->dev, r->geo.M, r->geo.K, r->geo.gs,
                              r->scheme == LLMOC_SCHEME_AWQ_SYM, r->zp, (float*)g_scratch.p, g_stream),
               "dequant"))
    return 0;
  count_launch();
  if (!cuda_ok(cudaMemcpyAsync(out, g_scratch.p, bytes, cudaMemcpyDeviceToHost, g_stream), "D2H") ||
      !cuda_ok(cudaStreamSynchronize(g_stream), "dequant"))
    return 0;
  return 1;
}

int llmoc_try_moe_ffn_int4(const float* x, int H, int I, const llmoc_moe_expert_int4* experts,
                           int n_experts, const llmoc_int4_view* shared_gate,
                           const llmoc_int4_view* shared_up, const llmoc_int4_view* shared_down,
                           float shared_scale, float* y) {
  if (!x || !y || !experts || n_experts <= 0 || H <= 0 || I <= 0) return fail("bad arguments");
  if (n_experts > 64) return fail("n_experts > 64");
  const bool has_shared = shared_gate && shared_up && shared_down && shared_gate->qweight &&
                          shared_up->qweight && shared_down->qweight && std::fabs(shared_scale) > 0.f;
  auto dims_ok = [&](const llmoc_int4_view* g, const llmoc_int4_view* u, const llmoc_int4_view* d) {
    return g && u && d && g->qweight && u->qweight && d->qweight && g->M == I && u->M == I &&
           d->M == H && g->K == H && u->K == H && d->K == I;
  };
  if (has_shared && !dims_ok(shared_gate, shared_up, shared_down))
    return fail("shared expert dims must be (I, H)");
  for (int i = 0; i < n_experts; ++i)
    if (!dims_ok(experts[i].gate, experts[i].up, experts[i].down)) return fail("expert dims mismatch");

  std::lock_guard<std::mutex> lk(g_mu);
  // pairs: experts with |w| >= 1e-12 (cuda_backend.cpp:5284), then the shared one
  std::vector<ExpertDev> tab;
  std::vector<float> wts;
  int scheme = -1, zp = 7, gs = 0;
  auto add = [&](const llmoc_int4_view* g, const llmoc_int4_view* u, const llmoc_int4_view* d,
                 float w) -> bool {
    Resident* rg = ensure_resident(g);
    Resident* ru = rg ? ensure_resident(u) : nullptr;
    Resident* rd = ru ? ensure_resident(d) : nullptr;
    if (!rd) return false;
    for (Resident* r : {rg, ru, rd}) {
      if (scheme < 0) {
        scheme = r->scheme;
        zp = r->zp;
        gs = r->geo.gs;
      } else if (r->scheme != scheme || r->zp != zp || r->geo.gs != gs) {
        t_err = "experts must share scheme, zero point and group size";
        return false;
      }
    }
    tab.push_back(ExpertDev{rg->dev, ru->dev, rd->dev});
    wts.push_back(w);
    return true;
  };
  for (int i = 0; i < n_experts; ++i) {
    if (std::fabs(experts[i].weight) < 1e-12f) continue;
    if (!add(experts[i].gate, experts[i].up, experts[i].down, experts[i].weight)) return 0;
  }
  if (has_shared && !add(shared_gate, shared_up, shared_down, shared_scale)) return 0;
  const int n = (int)tab.size();
  if (n == 0) {
    std::fill(y, y + H, 0.f);
    return 1;
  }
  const Geo gu = make_geo(I, H, gs, false), dn = make_geo(H, I, gs, false);
  // scratch: table | work | n_work | zeros(gather) | x | weights | inverse | mid | partial | y
  size_t o = 0;
  auto take = [&](size_t b) {
    size_t at = o;
    o += align256(b);
    return at;
  };
  const size_t o_tab = take(sizeof(ExpertDev) * n), o_work = take(sizeof(WorkItem) * n),
               o_nw = take(4), o_gat = take(4 * n), o_x = take((size_t)H * 4), o_w = take(4 * n),
               o_inv = take(4 * n), o_mid = take((size_t)n * I * 4), o_part = take((size_t)n * H * 4),
               o_y = take((size_t)H * 4);
  if (!g_scratch.ensure(o)) return 0;
  char* s = g_scratch.p;
  // host staging of the small tables in one pageable block, copied in order
  std::vector<char> host(o_x);
  memcpy(host.data() + o_tab, tab.data(), sizeof(ExpertDev) * n);
  WorkItem* wk = (WorkItem*)(host.data() + o_work);
  int* gat = (int*)(host.data() + o_gat);
  for (int i = 0; i < n; ++i) {
    wk[i] = WorkItem{i, i, 1, 0};
    gat[i] = 0;
  }
  memcpy(host.data() + o_nw, &n, 4);
  std::vector<int> inv(n);
  for (int i = 0; i < n; ++i) inv[i] = i;
  cudaStream_t st = g_stream;
  if (!cuda_ok(cudaMemcpyAsync(s, host.data(), o_x, cudaMemcpyHostToDevice, st), "H2D tables") ||
      !cuda_ok(cudaMemcpyAsync(s + o_x, x, (size_t)H * 4, cudaMemcpyHostToDevice, st), "H2D x") ||
      !cuda_ok(cudaMemcpyAsync(s + o_w, wts.data(), 4 * n, cudaMemcpyHostToDevice, st), "H2D w") ||
      !cuda_ok(cudaMemcpyAsync(s + o_inv, inv.data(), 4 * n, cudaMemcpyHostToDevice, st), "H2D inv"))
    return 0;
  GemmArgs a{};
  a.experts = (const ExpertDev*)(s + o_tab);
  a.M = I;
  a.K = H;
  a.Kc = gu.Kc;
  a.gs = gs;
  a.ng = gu.ng;
  a.zp = zp;
  a.B = s + o_x;
  a.ldb = H;
  a.gather = (const int*)(s + o_gat);
  a.kk = 1;
  a.work = (const WorkItem*)(s + o_work);
  a.n_work = (const int*)(s + o_nw);
  a.out = s + o_mid;
  a.ldo = I;
  a.out_bf16 = 0;
  const int awq = scheme == LLMOC_SCHEME_AWQ_SYM;
  if (!cuda_ok(launch_gemm(MODE_GATE_UP, 1, a, n, awq, 1, st), "gate/up")) return 0;
  GemmArgs b = a;
  b.proj = 2;
  b.M = H;
  b.K = I;
  b.Kc = dn.Kc;
  b.ng = dn.ng;
  b.B = s + o_mid;
  b.ldb = I;
  b.gather = nullptr;
  b.out = s + o_part;
  b.ldo = H;
  if (!cuda_ok(launch_gemm(MODE_PLAIN_F32, 1, b, n, awq, 1, st), "down")) return 0;
  if (!cuda_ok(launch_combine((const float*)(s + o_part), (const int*)(s + o_inv),
                              (const float*)(s + o_w), 1, n, H, s + o_y, 0, 0, st),
               "combine"))
    return 0;
  count_launch(3);
  if (!cuda_ok(cudaMemcpyAsync(y, s + o_y, (size_t)H * 4, cudaMemcpyDeviceToHost, st), "D2H y") ||
      !cuda_ok(cudaStreamSynchronize(st), "moe ffn"))
    return 0;
  return 1;
}

// ------------------------------------------------------------- layer API

llmoc_status llmoc_moe_layer_create(const llmoc_moe_layer_desc* desc, const uint16_t* router_w,
                                    const float* bias, const llmoc_int4_view* experts,
                                    const llmoc_int4_view* shared, int device,
                                    llmoc_moe_layer** out) {
  return layer_create(desc, router_w, bias, experts, shared, device, false, out);
}

llmoc_status llmoc_moe_layer_create_device(const llmoc_moe_layer_desc* desc,
                                           const uint16_t* router_w, const float* bias,
                                           const llmoc_int4_view* experts,
                                           const llmoc_int4_view* shared, int device,
                                           llmoc_moe_layer** out) {
  return layer_create(desc, router_w, bias, experts, shared, device, true, out);
}

llmoc_status llmoc_moe_layer_create_ep(const llmoc_moe_layer_desc* desc, const uint16_t* router_w,
                                       const float* bias, const llmoc_int4_view* experts,
                                       const llmoc_int4_view* shared, int device, int rank, int world,
                                       int on_device, llmoc_moe_layer** out) {
  return layer_create(desc, router_w, bias, experts, shared, device, on_device != 0, out, rank, world);
}

void llmoc_moe_layer_destroy(llmoc_moe_layer* L) {
  if (!L) return;
  DevGuard dg(L->device);
  llmoc_moe_set_stage_timing(L, 0);
  for (auto e : L->ev_pool) cudaEventDestroy(e);
  if (L->arena) cudaFree(L->arena);
  if (L->table) cudaFree(L->table);
  if (L->wmaps) cudaFree(L->wmaps);
  if (L->router_w) cudaFree(L->router_w);
  if (L->bias) cudaFree(L->bias);
  delete L;
}

size_t llmoc_moe_layer_weight_bytes(const llmoc_moe_layer* L) { return L ? L->weight_bytes : 0; }

size_t llmoc_expert_storage_bytes(int H, int I, int group_size, int has_zeros) {
  // qlwc_expert_bytes.h:43-48: gate[IxH] + up[IxH] + down[HxI], q + fp16 scales (+zeros)
  auto proj = [&](size_t M, size_t K) {
    const size_t gs = group_size > 0 ? (size_t)group_size : 128;
    const size_t ng = (K + gs - 1) / gs;
    return M * ((K + 1) / 2) + M * ng * 2 * (has_zeros ? 2 : 1);
  };
  return 2 * proj((size_t)I, (size_t)H) + proj((size_t)H, (size_t)I);
}

size_t llmoc_moe_workspace_bytes(const llmoc_moe_layer* L, int max_tokens) {
  if (!L || max_tokens < 0) return 0;
  return ws_layout(L, max_tokens).total;
}

llmoc_status llmoc_moe_route_views(const llmoc_moe_layer* L, int T, void* workspace,
                                   size_t workspace_bytes, llmoc_route_views* out) {
  if (!L || !out || T < 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  const WsLayout w = ws_layout(L, T);
  if (!workspace || workspace_bytes < w.total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  char* ws = (char*)workspace;
  out->logits = (float*)(ws + w.logits);
  out->ids = (int32_t*)(ws + w.ids);
  out->weights = (float*)(ws + w.weights);
  out->offsets = (int32_t*)(ws + w.offsets);
  out->sorted = (int32_t*)(ws + w.sorted);
  out->inverse = (int32_t*)(ws + w.inverse);
  out->n_active = (int32_t*)(ws + w.n_active);
  out->error_flag = (int32_t*)(ws + w.err);
  return LLMOC_OK;
}

llmoc_status llmoc_moe_route(const llmoc_moe_layer* L, const uint16_t* X, int T, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!L || T < 0 || (T > 0 && !X)) return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (L->ep_world > 1) return fails(LLMOC_ERR_INVALID, "expert-parallel layer: use llmoc_moe_ep_*");
  if (T == 0) return LLMOC_OK;
  const WsLayout w = ws_layout(L, T);
  if (!workspace || workspace_bytes < w.total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  DevGuard dg(L->device);
  return run_route(L, X, T, w, (char*)workspace, (cudaStream_t)stream);
}

namespace {
llmoc_status moe_forward(const llmoc_moe_layer* L, const uint16_t* X, int T, const uint16_t* R, uint16_t* Y,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!L || T < 0 || (T > 0 && (!X || !Y))) return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (L->ep_world > 1) return fails(LLMOC_ERR_INVALID, "expert-parallel layer: use llmoc_moe_ep_*");
  if (T == 0) return LLMOC_OK;
  const WsLayout w = ws_layout(L, T);
  if (!workspace || workspace_bytes < w.total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  DevGuard dg(L->device);
  cudaStream_t st = (cudaStream_t)stream;
  char* ws = (char*)workspace;
  StageEvents se(L);
  if (T == 1 && decode1_ok(L)) {
    const llmoc_status rc = run_decode1(L, X, R, Y, w, ws, st, &se);
    if (rc != LLMOC_ERR_UNSUPPORTED) {
      if (rc == LLMOC_OK) se.commit();
      return rc;
    }
    se.next = 0;  // the one-launch form was refused: the chain of separate kernels below
  }
  llmoc_status rc = run_route(L, X, T, w, ws, st, &se);
  if (rc != LLMOC_OK) return rc;
  rc = run_ffn(L, X, T, L->kk, chunk_rows(L, T), w, ws, Y, (const float*)(ws + w.weights), st, &se, R, 0,
               w.xh != 0);
  if (rc != LLMOC_OK) return rc;
  se.commit();
  return LLMOC_OK;
}
}  // namespace

llmoc_status llmoc_moe_forward(const llmoc_moe_layer* L, const uint16_t* X, int T, uint16_t* Y,
                               void* workspace, size_t workspace_bytes, void* stream) {
  return moe_forward(L, X, T, nullptr, Y, workspace, workspace_bytes, stream);
}

llmoc_status llmoc_moe_forward_residual(const llmoc_moe_layer* L, const uint16_t* X, int T, const uint16_t* R,
                                        uint16_t* Y, void* workspace, size_t workspace_bytes, void* stream) {
  if (T > 0 && !R) return fails(LLMOC_ERR_INVALID, "null residual");
  return moe_forward(L, X, T, R, Y, workspace, workspace_bytes, stream);
}

llmoc_status llmoc_moe_layer_set_shared_gate(llmoc_moe_layer* L, const uint16_t* gate_row, int on_device) {
  if (!L || !gate_row) return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (!L->d.has_shared) return fails(LLMOC_ERR_INVALID, "the layer has no shared expert");
  DevGuard dg(L->device);
  const size_t E = (size_t)L->d.n_experts, H = (size_t)L->d.hidden;
  uint16_t* nw = nullptr;
  if (!cuda_ok(cudaMalloc((void**)&nw, (E + 1) * H * 2), "router alloc")) return LLMOC_ERR_NO_MEMORY;
  if (!cuda_ok(cudaMemcpy(nw, L->router_w, E * H * 2, cudaMemcpyDeviceToDevice), "router copy") ||
      !cuda_ok(cudaMemcpy(nw + E * H, gate_row, H * 2, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice),
               "gate row")) {
    cudaFree(nw);
    return LLMOC_ERR_CUDA;
  }
  cudaFree(L->router_w);
  L->router_w = nw;
  L->shared_gate = 1;
  return LLMOC_OK;
}

llmoc_status llmoc_moe_dequant(const llmoc_moe_layer* L, int expert, int proj, float* out,
                               void* stream) {
  if (!L || !out || expert < 0 || expert >= L->n_exp || proj < 0 || proj > 2)
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  DevGuard dg(L->device);
  const ExpertDev& e = L->htable[expert];
  const ProjDev& P = proj == 0 ? e.gate : (proj == 1 ? e.up : e.down);
  const Geo& g = proj == 2 ? L->dn : L->gu;
  if (!cuda_ok(launch_dequant(P, g.M, g.K, g.gs, L->d.scheme == LLMOC_SCHEME_AWQ_SYM, L->d.awq_zp,
                              out, (cudaStream_t)stream),
               "dequant"))
    return LLMOC_ERR_CUDA;
  count_launch();
  return LLMOC_OK;
}

llmoc_status llmoc_quantize_awq_sym(const uint16_t* W, int M, int K, int group_size, int bf16_scale,
                                    uint8_t* q, uint16_t* scales, void* stream) {
  if (!W || !q || !scales || M <= 0 || K <= 0 || group_size <= 0 || K % group_size || group_size % 2)
    return fails(LLMOC_ERR_INVALID, "bad arguments (K % group_size must be 0)");
  if (!cuda_ok(launch_quant_awq_sym((const __nv_bfloat16*)W, M, K, group_size, bf16_scale, q,
                                    (__half*)scales, (cudaStream_t)stream),
               "quantize"))
    return LLMOC_ERR_CUDA;
  count_launch();
  return LLMOC_OK;
}

llmoc_status llmoc_moe_layer_set_wait_cycles(llmoc_moe_layer* L, long long cycles) {
  if (!L || cycles <= 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  L->wait_cycles = cycles;
  return LLMOC_OK;
}

llmoc_status llmoc_moe_set_stage_timing(llmoc_moe_layer* L, int enable) {
  if (!L) return fails(LLMOC_ERR_INVALID, "null layer");
  DevGuard dg(L->device);
  for (auto& call : L->ev_calls) {
    cudaEventSynchronize(call[6]);
    for (auto e : call) L->ev_pool.push_back(e);
  }
  L->ev_calls.clear();
  L->timing = enable != 0;
  return LLMOC_OK;
}

llmoc_status llmoc_moe_stage_times(llmoc_moe_layer* L, float* ms, int* calls) {
  if (!L || !ms) return fails(LLMOC_ERR_INVALID, "bad arguments");
  DevGuard dg(L->device);
  for (int i = 0; i < 6; ++i) ms[i] = 0.f;
  for (auto& call : L->ev_calls) {
    if (!cuda_ok(cudaEventSynchronize(call[6]), "stage events")) return LLMOC_ERR_CUDA;
    for (int i = 0; i < 6; ++i) {
      float t = 0.f;
      if (!cuda_ok(cudaEventElapsedTime(&t, call[i], call[i + 1]), "stage elapsed"))
        return LLMOC_ERR_CUDA;
      ms[i] += t;
    }
  }
  if (calls) *calls = (int)L->ev_calls.size();
  for (auto& call : L->ev_calls)
    for (auto e : call) L->ev_pool.push_back(e);
  L->ev_calls.clear();
  return LLMOC_OK;
}

uint64_t llmoc_kernel_launch_count(void) { return g_launches.load(); }

// ------------------------------------------------------ expert parallelism

size_t llmoc_moe_ep_source_workspace_bytes(const llmoc_moe_layer* L, int max_tokens) {
  if (!L || max_tokens < 0) return 0;
  return ep_src_layout(L, max_tokens).total;
}

size_t llmoc_moe_ep_owner_workspace_bytes(const llmoc_moe_layer* L, int max_rows) {
  if (!L || max_rows < 0) return 0;
  return ep_owner_bytes(L, max_rows);
}

namespace {
// gather: write send_rows (the C entry point); the NVLink send passes false,
// its push reads the tokens' rows through the sorted order instead
llmoc_status ep_dispatch(const llmoc_moe_layer* L, const uint16_t* X, int T, void* workspace,
                         size_t workspace_bytes, uint16_t* send_rows, int32_t* send_expert, int32_t* send_counts,
                         void* stream, bool gather) {
  if (!L || T < 0 || (T > 0 && (!X || (gather && !send_rows) || !send_expert)) || !send_counts)
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  const EpSrcLayout w = ep_src_layout(L, T);
  if (!workspace || workspace_bytes < w.total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  DevGuard dg(L->device);
  cudaStream_t st = (cudaStream_t)stream;
  char* ws = (char*)workspace;
  const int E = L->d.n_experts, H = L->d.hidden, k = L->d.topk, n = T * k;
  if (T == 0) {
    if (!cuda_ok(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * L->ep_world, st), "counts"))
      return LLMOC_ERR_CUDA;
    return LLMOC_OK;
  }
  float* logits = (float*)(ws + w.logits);
  if (!cuda_ok(launch_router_logits(X, false, L->router_w, T, E + L->shared_gate, H, logits, st), "router"))
    return LLMOC_ERR_CUDA;
  TopkArgs ta{};
  ta.logits = logits;
  ta.bias = L->bias;
  ta.T = T;
  ta.E = E;
  ta.k = k;
  ta.kk = k;  // routed slots only: the shared expert runs on the source rank
  ta.router = L->d.router;
  ta.routed_scaling = L->d.routed_scaling;
  ta.shared_scale = L->d.shared_scale;
  ta.has_shared = 0;
  ta.ld = E + L->shared_gate;
  ta.shared_gate = L->shared_gate;
  if (L->shared_gate) ta.shared_w = (float*)(ws + w.shw);  // for the combine at this source
  ta.ids = (int*)(ws + w.ids);
  ta.weights = (float*)(ws + w.weights);
  int* key = (int*)(ws + w.key);
  PermArgs pa{};
  pa.ids = key;
  pa.n = n;
  pa.n_exp = E;
  pa.offsets = (int*)(ws + w.offsets);
  pa.sorted = (int*)(ws + w.sorted);
  pa.inverse = (int*)(ws + w.inverse);
  pa.work = (WorkItem*)(ws + w.work);
  pa.n_work = (int*)(ws + w.n_work);
  pa.n_active = (int*)(ws + w.n_active);
  pa.err = (int*)(ws + w.err);
  pa.chunk = 8;
  if (T <= kFusedRouteMaxT && E <= kMaxExpPerm) {  // one CTA: top-k, owner keys, permutation, per-owner meta
    EpRouteArgs ea;
    ea.world = L->ep_world;
    ea.e_loc = L->e_loc;
    ea.key = key;
    ea.counts = send_counts;
    ea.send_expert = send_expert;
    if (!cuda_ok(launch_topk_permute(ta, pa, st, ea), "topk+permute")) return LLMOC_ERR_CUDA;
    count_launch(2);
  } else {  // top-k writing the owner keys too; the permutation with the per-owner tail
    ta.ep_key = key;
    ta.ep_world = L->ep_world;
    ta.ep_e_loc = L->e_loc;
    EpRouteArgs ea;
    ea.world = L->ep_world;
    ea.e_loc = L->e_loc;
    ea.key = key;
    ea.counts = send_counts;
    ea.send_expert = send_expert;
    if (!cuda_ok(launch_topk(ta, st), "topk") || !cuda_ok(launch_permute_ep(pa, ea, st), "permute"))
      return LLMOC_ERR_CUDA;
    count_launch(3);
  }
  if (gather) {
    if (!cuda_ok(launch_gather_rows(X, H, pa.sorted, k, n, nullptr, send_rows, st), "gather")) return LLMOC_ERR_CUDA;
    count_launch(1);
  }
  return LLMOC_OK;
}
}  // namespace

llmoc_status llmoc_moe_ep_dispatch(const llmoc_moe_layer* L, const uint16_t* X, int T, void* workspace,
                                   size_t workspace_bytes, uint16_t* send_rows, int32_t* send_expert,
                                   int32_t* send_counts, void* stream) {
  return ep_dispatch(L, X, T, workspace, workspace_bytes, send_rows, send_expert, send_counts, stream, true);
}

namespace {
// n rows (expert ids < 0: empty slots), about n_hint of them occupied (sets the kernel regime)
llmoc_status ep_experts(const llmoc_moe_layer* L, const uint16_t* rows, const int32_t* expert, int n, int n_hint,
                        uint16_t* out_rows, void* workspace, size_t workspace_bytes, void* stream,
                        const PermSegs& segs = PermSegs{}) {
  const int chunk = chunk_for_rows(n_hint, L->e_loc);
  const WsLayout w = ws_layout_g(L, n, 1, L->n_exp, chunk, false);
  if (!workspace || workspace_bytes < w.total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  DevGuard dg(L->device);
  cudaStream_t st = (cudaStream_t)stream;
  char* ws = (char*)workspace;
  llmoc_status rc = run_permute(expert, n, L->n_exp, chunk, w, ws, st, segs);
  if (rc != LLMOC_OK) return rc;
  return run_ffn(L, rows, n, 1, chunk, w, ws, out_rows, nullptr, st, nullptr, nullptr, n_hint);
}
}  // namespace

llmoc_status llmoc_moe_ep_experts(const llmoc_moe_layer* L, const uint16_t* rows, const int32_t* expert, int n,
                                  uint16_t* out_rows, void* workspace, size_t workspace_bytes, void* stream) {
  if (!L || n < 0 || (n > 0 && (!rows || !expert || !out_rows))) return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (n == 0) return LLMOC_OK;
  return ep_experts(L, rows, expert, n, n, out_rows, workspace, workspace_bytes, stream);
}

llmoc_status llmoc_moe_ep_experts_padded(const llmoc_moe_layer* L, const uint16_t* rows, const int32_t* expert,
                                         int n, int n_hint, uint16_t* out_rows, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  if (!L || n < 0 || n_hint < 0 || (n > 0 && (!rows || !expert || !out_rows)))
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (n == 0) return LLMOC_OK;
  // empty slots (ids outside [0, n_exp)) are skipped by the permutation; the
  // hint sizes the item regime and the GEMM grids by the occupied slots
  return ep_experts(L, rows, expert, n, std::max(1, std::min(n, n_hint)), out_rows, workspace, workspace_bytes,
                    stream);
}

namespace {
// The shared expert over the source rank's own T tokens, into the source
// workspace (no-op without a shared expert).
llmoc_status ep_shared(const llmoc_moe_layer* L, const uint16_t* X, int T, const EpSrcLayout& w, char* ws,
                       cudaStream_t st) {
  if (!L->d.has_shared || T == 0) return LLMOC_OK;
  char* s2 = ws + w.sh;
  int* ids = (int*)(s2 + w.shl.ids);
  if (!cuda_ok(launch_fill_i32(ids, T, L->e_loc, st), "fill")) return LLMOC_ERR_CUDA;
  count_launch(1);
  llmoc_status rc = run_permute(ids, T, L->n_exp, w.sh_chunk, w.shl, s2, st);
  if (rc == LLMOC_OK) rc = run_ffn(L, X, T, 1, w.sh_chunk, w.shl, s2, nullptr, nullptr, st);
  return rc;
}
// Y = the routed weights x the returned rows (slot order) + the shared expert's rows.
llmoc_status ep_combine_rows(const llmoc_moe_layer* L, int T, const uint16_t* ret_rows, uint16_t* Y,
                             const EpSrcLayout& w, char* ws, cudaStream_t st, const FlagWait& fw = FlagWait{}) {
  const float* sh = nullptr;
  const int* sh_inv = nullptr;
  if (L->d.has_shared) {
    sh = (const float*)(ws + w.sh + w.shl.partial);
    sh_inv = (const int*)(ws + w.sh + w.shl.inverse);
  }
  if (!cuda_ok(launch_combine_ep(ret_rows, (const int*)(ws + w.inverse), (const float*)(ws + w.weights), T,
                                 L->d.topk, L->d.hidden, sh, sh_inv, L->d.shared_scale,
                                 L->shared_gate ? (const float*)(ws + w.shw) : nullptr, Y, st, fw),
               "combine"))
    return LLMOC_ERR_CUDA;
  count_launch(1);
  return LLMOC_OK;
}
}  // namespace

llmoc_status llmoc_moe_ep_combine(const llmoc_moe_layer* L, const uint16_t* X, int T, const uint16_t* ret_rows,
                                  uint16_t* Y, void* workspace, size_t workspace_bytes, void* stream) {
  if (!L || T < 0 || (T > 0 && (!X || !ret_rows || !Y))) return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (T == 0) return LLMOC_OK;
  const EpSrcLayout w = ep_src_layout(L, T);
  if (!workspace || workspace_bytes < w.total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  DevGuard dg(L->device);
  cudaStream_t st = (cudaStream_t)stream;
  char* ws = (char*)workspace;
  llmoc_status rc = ep_shared(L, X, T, w, ws, st);
  if (rc != LLMOC_OK) return rc;
  return ep_combine_rows(L, T, ret_rows, Y, w, ws, st);
}

// ------------------------------------------------------- QLWC file loader
// The reference's INT4 container (src/weights/qlwc_format.h, .cpp:40-160):
// preface = magic "QLW1", u32 version, u64 catalog length, u64 FNV-1a 64 of
// the catalog; catalog (little-endian) = u32 scheme, u32 group size, u32 block
// alignment, u64 tensor count, then per tensor: string name (u32 length +
// bytes), u32 kind, u64 rank, rank x u64 dims, and for a passthrough tensor
// u32 dtype (1 bf16, 2 f16), u64 offset, u64 bytes; for an INT4 tensor u32
// group size, u64 q offset/bytes, u64 scales offset/bytes, u64 zeros
// offset/bytes.  Tensor names follow the reference's model loaders
// (src/model/qwen3_6_moe_int4_model.cpp:201, src/model/moe_model.cpp:308-364).

namespace {
struct QTensor {
  std::string name;
  uint32_t kind = 0, dtype = 0, gs = 0;
  std::vector<uint64_t> shape;
  uint64_t off = 0, nbytes = 0, q_off = 0, q_n = 0, s_off = 0, s_n = 0, z_off = 0, z_n = 0;
};
struct QFile {
  uint32_t scheme = 0, gs = 0;
  std::vector<QTensor> tensors;
  const QTensor* find(const std::string& n) const {
    for (const auto& t : tensors)
      if (t.name == n) return &t;
    return nullptr;
  }
};

bool qlwc_read_header(FILE* f, QFile* q) {
  unsigned char pre[24];
  if (fread(pre, 1, 24, f) != 24 || memcmp(pre, "QLW1", 4) != 0) return fails(LLMOC_ERR_INVALID, "not a QLWC v1 file"), false;
  uint32_t ver;
  uint64_t clen, crc;
  memcpy(&ver, pre + 4, 4);
  memcpy(&clen, pre + 8, 8);
  memcpy(&crc, pre + 16, 8);
  if (ver != 1 || clen > (1ull << 32)) return fails(LLMOC_ERR_INVALID, "QLWC version or catalog size"), false;
  std::vector<unsigned char> cat(clen);
  if (fread(cat.data(), 1, clen, f) != clen) return fails(LLMOC_ERR_INVALID, "QLWC catalog truncated"), false;
  uint64_t h = 14695981039346656037ull;
  for (unsigned char c : cat) h = (h ^ c) * 1099511628211ull;
  if (h != crc) return fails(LLMOC_ERR_INVALID, "QLWC catalog checksum"), false;
  size_t p = 0;
  bool ok = true;
  auto u32 = [&]() -> uint32_t {
    uint32_t v = 0;
    if (p + 4 > cat.size()) ok = false;
    else memcpy(&v, &cat[p], 4);
    p += 4;
    return v;
  };
  auto u64 = [&]() -> uint64_t {
    uint64_t v = 0;
    if (p + 8 > cat.size()) ok = false;
    else memcpy(&v, &cat[p], 8);
    p += 8;
    return v;
  };
  q->scheme = u32();
  q->gs = u32();
  u32();  // block alignment
  const uint64_t n = u64();
  for (uint64_t i = 0; ok && i < n; ++i) {
    QTensor t;
    const uint32_t len = u32();
    if (!ok || p + len > cat.size()) {
      ok = false;
      break;
    }
    t.name.assign(reinterpret_cast<const char*>(&cat[p]), len);
    p += len;
    t.kind = u32();
    const uint64_t rank = u64();
    for (uint64_t r = 0; ok && r < rank && r < 8; ++r) t.shape.push_back(u64());
    if (t.kind == 0) {
      t.dtype = u32();
      t.off = u64();
      t.nbytes = u64();
    } else {
      t.gs = u32();
      t.q_off = u64();
      t.q_n = u64();
      t.s_off = u64();
      t.s_n = u64();
      t.z_off = u64();
      t.z_n = u64();
    }
    q->tensors.push_back(std::move(t));
  }
  if (!ok) return fails(LLMOC_ERR_INVALID, "QLWC catalog malformed"), false;
  return true;
}

bool qlwc_read(FILE* f, uint64_t off, uint64_t n, void* dst) {
  if (n == 0) return true;
  if (fseeko(f, (off_t)off, SEEK_SET) != 0 || fread(dst, 1, n, f) != n)
    return fails(LLMOC_ERR_INVALID, "QLWC payload truncated"), false;
  return true;
}

struct QLayerNames {
  std::string base, shared, gate, bias, shared_gate;
};
QLayerNames qlwc_names(const char* prefix, int layer, const QFile& q) {
  QLayerNames n;
  n.base = std::string(prefix ? prefix : "") + "layers." + std::to_string(layer) + ".mlp.";
  n.gate = n.base + "gate.weight";
  n.bias = n.base + "gate.e_score_correction_bias";
  n.shared = q.find(n.base + "shared_expert.gate_proj.weight") ? n.base + "shared_expert."
                                                                 : n.base + "shared_experts.";
  n.shared_gate = n.base + "shared_expert_gate.weight";
  return n;
}

// An INT4 tensor's payloads must be exactly its packed nibbles (M x K/2
// bytes), M x K/gs fp16 scales and, for GPTQ, as many fp16 zeros.
bool qlwc_int4_sizes_ok(const QTensor& t, const QFile& q) {
  if (t.kind != 1 || t.shape.size() != 2) return false;
  const uint64_t M = t.shape[0], K = t.shape[1], gs = t.gs ? t.gs : q.gs;
  if (M == 0 || K == 0 || gs == 0 || M > (1u << 30) || K > (1u << 30)) return false;
  const uint64_t ng = (K + gs - 1) / gs;
  return t.q_n == M * ((K + 1) / 2) && t.s_n == M * ng * 2 &&
         t.z_n == (q.scheme == LLMOC_SCHEME_GPTQ_ASYM ? M * ng * 2 : 0);
}

llmoc_status qlwc_info(const QFile& q, const QLayerNames& nm, llmoc_qlwc_layer_info* out) {
  *out = llmoc_qlwc_layer_info{};
  const QTensor* g0 = q.find(nm.base + "experts.0.gate_proj.weight");
  const QTensor* d0 = q.find(nm.base + "experts.0.down_proj.weight");
  if (!g0 || !d0 || g0->kind != 1 || d0->kind != 1 || g0->shape.size() != 2)
    return fails(LLMOC_ERR_INVALID, "no INT4 experts for this layer in the QLWC file");
  int E = 0;
  while (q.find(nm.base + "experts." + std::to_string(E) + ".gate_proj.weight")) ++E;
  for (int e = 0; e <= E; ++e) {  // e == E: the shared expert, if any
    const std::string b = e < E ? nm.base + "experts." + std::to_string(e) + "." : nm.shared;
    if (e == E && !q.find(b + "gate_proj.weight")) break;
    for (const char* pn : {"gate_proj.weight", "up_proj.weight", "down_proj.weight"}) {
      const QTensor* t = q.find(b + pn);
      if (!t || !qlwc_int4_sizes_ok(*t, q)) return fails(LLMOC_ERR_INVALID, "QLWC tensor missing or malformed: " + b + pn);
    }
  }
  out->n_experts = E;
  out->inter = (int)g0->shape[0];
  out->hidden = (int)g0->shape[1];
  out->group_size = (int)(g0->gs ? g0->gs : q.gs);
  out->scheme = (int)q.scheme;
  out->has_shared = q.find(nm.shared + "gate_proj.weight") != nullptr;
  out->has_shared_gate = q.find(nm.shared_gate) != nullptr;
  out->has_bias = q.find(nm.bias) != nullptr;
  const QTensor* r = q.find(nm.gate);
  out->has_router = r && r->kind == 0 && r->dtype == 1;
  return LLMOC_OK;
}

float qlwc_half_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
}  // namespace

llmoc_status llmoc_qlwc_describe(const char* path, const char* prefix, int layer, llmoc_qlwc_layer_info* out) {
  if (!path || !out || layer < 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  FILE* f = fopen(path, "rb");
  if (!f) return fails(LLMOC_ERR_INVALID, "cannot open the QLWC file");
  QFile q;
  const bool ok = qlwc_read_header(f, &q);
  fclose(f);
  if (!ok) return LLMOC_ERR_INVALID;
  return qlwc_info(q, qlwc_names(prefix, layer, q), out);
}

int llmoc_qlwc_moe_layers(const char* path, const char* prefix, int32_t* layers, int max_layers) {
  if (!path || max_layers < 0 || (max_layers > 0 && !layers)) return fails(LLMOC_ERR_INVALID, "bad arguments"), -1;
  FILE* f = fopen(path, "rb");
  if (!f) return fails(LLMOC_ERR_INVALID, "cannot open the QLWC file"), -1;
  QFile q;
  const bool ok = qlwc_read_header(f, &q);
  fclose(f);
  if (!ok) return -1;
  // layers with an INT4 expert 0: "<prefix>layers.<n>.mlp.experts.0.gate_proj.weight"
  const std::string head = std::string(prefix ? prefix : "") + "layers.";
  const std::string tail = ".mlp.experts.0.gate_proj.weight";
  std::vector<int> found;
  for (const auto& t : q.tensors) {
    if (t.kind != 1 || t.name.size() <= head.size() + tail.size() || t.name.compare(0, head.size(), head) != 0 ||
        t.name.compare(t.name.size() - tail.size(), tail.size(), tail) != 0)
      continue;
    const std::string mid = t.name.substr(head.size(), t.name.size() - head.size() - tail.size());
    if (mid.empty() || mid.size() > 6 || mid.find_first_not_of("0123456789") != std::string::npos) continue;
    found.push_back(std::stoi(mid));
  }
  std::sort(found.begin(), found.end());
  found.erase(std::unique(found.begin(), found.end()), found.end());
  for (int i = 0; i < (int)found.size() && i < max_layers; ++i) layers[i] = found[i];
  return (int)found.size();
}

llmoc_status llmoc_moe_layer_create_qlwc(const char* path, const char* prefix, int layer,
                                         const llmoc_moe_layer_desc* desc, int device, llmoc_moe_layer** out) {
  if (!path || !desc || !out || layer < 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) return fails(LLMOC_ERR_INVALID, "cannot open the QLWC file");
  struct Closer {
    FILE* f;
    ~Closer() { fclose(f); }
  } closer{f};
  QFile q;
  if (!qlwc_read_header(f, &q)) return LLMOC_ERR_INVALID;
  const QLayerNames nm = qlwc_names(prefix, layer, q);
  llmoc_qlwc_layer_info info;
  llmoc_status rc = qlwc_info(q, nm, &info);
  if (rc != LLMOC_OK) return rc;
  if (!info.has_router) return fails(LLMOC_ERR_INVALID, "router (mlp.gate.weight, bf16) missing");
  if (desc->hidden != info.hidden || desc->inter != info.inter || desc->n_experts != info.n_experts ||
      desc->group_size != info.group_size || desc->scheme != info.scheme || desc->has_shared != info.has_shared)
    return fails(LLMOC_ERR_INVALID, "layer desc disagrees with the QLWC file");
  const int E = info.n_experts, H = info.hidden;
  // host copies of every tensor the layer needs; views point into them until the upload returns
  std::vector<std::vector<uint8_t>> blobs;
  blobs.reserve((size_t)3 * 3 * (E + 1) + 4);
  auto load = [&](uint64_t off, uint64_t n) -> const uint8_t* {
    blobs.emplace_back(n);
    if (!qlwc_read(f, off, n, blobs.back().data())) return nullptr;
    return blobs.back().data();
  };
  std::vector<llmoc_int4_view> views;
  auto add_view = [&](const std::string& name, std::vector<llmoc_int4_view>& dst) -> bool {
    const QTensor* t = q.find(name);
    if (!t || t->kind != 1 || t->shape.size() != 2) return fails(LLMOC_ERR_INVALID, "missing INT4 tensor " + name), false;
    llmoc_int4_view v{};
    v.M = (int)t->shape[0];
    v.K = (int)t->shape[1];
    v.group_size = (int)(t->gs ? t->gs : q.gs);
    if (!qlwc_int4_sizes_ok(*t, q)) return fails(LLMOC_ERR_INVALID, "QLWC payload sizes of " + name), false;
    v.scheme = q.scheme;
    v.awq_zp = q.scheme == LLMOC_SCHEME_AWQ_SYM ? 7 : 0;  // the reference's local AWQ zero point
    v.qweight = load(t->q_off, t->q_n);
    v.scales = (const uint16_t*)load(t->s_off, t->s_n);
    v.zeros = t->z_n ? (const uint16_t*)load(t->z_off, t->z_n) : nullptr;
    if (!v.qweight || !v.scales || (t->z_n && !v.zeros)) return false;
    dst.push_back(v);
    return true;
  };
  for (int e = 0; e < E; ++e)
    for (const char* pn : {"gate_proj.weight", "up_proj.weight", "down_proj.weight"})
      if (!add_view(nm.base + "experts." + std::to_string(e) + "." + pn, views)) return LLMOC_ERR_INVALID;
  std::vector<llmoc_int4_view> shared;
  if (info.has_shared)
    for (const char* pn : {"gate_proj.weight", "up_proj.weight", "down_proj.weight"})
      if (!add_view(nm.shared + pn, shared)) return LLMOC_ERR_INVALID;
  const QTensor* rt = q.find(nm.gate);
  if (rt->nbytes != (uint64_t)E * H * 2) return fails(LLMOC_ERR_INVALID, "router shape");
  const uint16_t* router = (const uint16_t*)load(rt->off, rt->nbytes);
  if (!router) return LLMOC_ERR_INVALID;
  std::vector<float> bias;
  if (info.has_bias) {  // selection bias (16-bit passthrough) -> fp32
    const QTensor* bt = q.find(nm.bias);
    if (bt->kind != 0 || bt->nbytes != (uint64_t)E * 2) return fails(LLMOC_ERR_INVALID, "bias shape");
    const uint16_t* b = (const uint16_t*)load(bt->off, bt->nbytes);
    if (!b) return LLMOC_ERR_INVALID;
    bias.resize(E);
    for (int e = 0; e < E; ++e) {
      if (bt->dtype == 2) {
        bias[e] = qlwc_half_to_f32(b[e]);
      } else {
        const uint32_t u = (uint32_t)b[e] << 16;
        memcpy(&bias[e], &u, 4);
      }
    }
  }
  llmoc_moe_layer* L = nullptr;
  rc = layer_create(desc, router, bias.empty() ? nullptr : bias.data(), views.data(),
                    info.has_shared ? shared.data() : nullptr, device, false, &L);
  if (rc != LLMOC_OK) return rc;
  if (info.has_shared && info.has_shared_gate) {
    const QTensor* gt = q.find(nm.shared_gate);
    const uint16_t* g = (gt->kind == 0 && gt->dtype == 1 && gt->nbytes == (uint64_t)H * 2)
                            ? (const uint16_t*)load(gt->off, gt->nbytes) : nullptr;
    rc = g ? llmoc_moe_layer_set_shared_gate(L, g, 0) : fails(LLMOC_ERR_INVALID, "shared expert gate shape");
    if (rc != LLMOC_OK) {
      llmoc_moe_layer_destroy(L);
      return rc;
    }
  }
  *out = L;
  return LLMOC_OK;
}

// ------------------------------------------- NVLink expert-parallel transport

size_t llmoc_ep_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

llmoc_status llmoc_ep_transport_create(int world, int rank, int hidden, int max_tokens, int topk, int device,
                                       llmoc_ep_transport** out, void* ipc_handle) {
  if (!out || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || hidden <= 0 || hidden % 8 ||
      max_tokens <= 0 || topk <= 0)
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  *out = nullptr;
  DevGuard dg(device);
  auto* tr = new llmoc_ep_transport();
  tr->world = world;
  tr->rank = rank;
  tr->device = device;
  tr->hidden = hidden;
  tr->max_tokens = max_tokens;
  tr->topk = topk;
  EpP2PLayout& l = tr->lay;
  l.world = world;
  l.cap = max_tokens * topk;  // a source sends at most this many rows (to one owner, in the worst case)
  l.row_bytes = hidden * 2;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes);
    return at;
  };
  l.flags = take((size_t)2 * world * 4);
  l.meta = take((size_t)2 * world * 8);
  l.recv_ids = take((size_t)2 * world * l.cap * 4);
  l.recv_rows = take((size_t)2 * world * l.cap * l.row_bytes);
  l.ret_rows = take((size_t)2 * l.cap * l.row_bytes);
  l.total = o;
  bool ok = cuda_ok(cudaMalloc((void**)&tr->base, l.total), "transport buffer") &&
            cuda_ok(cudaMemset(tr->base, 0, l.total), "transport memset") &&
            cuda_ok(cudaMalloc((void**)&tr->ctr, 64), "transport counters") &&
            cuda_ok(cudaMemset(tr->ctr, 0, 64), "transport memset") &&
            cuda_ok(cudaMalloc((void**)&tr->peers_dev, sizeof(char*) * world), "transport peers");
  tr->err = tr->ctr + 8;
  if (ok && ipc_handle) {
    cudaIpcMemHandle_t h;
    ok = cuda_ok(cudaIpcGetMemHandle(&h, tr->base), "ipc handle");
    if (ok) memcpy(ipc_handle, &h, sizeof(h));
  }
  tr->peer.assign(world, nullptr);
  tr->opened.assign(world, false);
  tr->peer[rank] = tr->base;
  if (!ok) {
    llmoc_ep_transport_destroy(tr);
    return LLMOC_ERR_CUDA;
  }
  *out = tr;
  return LLMOC_OK;
}

namespace {
llmoc_status upload_peers(llmoc_ep_transport* tr) {
  if (!cuda_ok(cudaMemcpy(tr->peers_dev, tr->peer.data(), sizeof(char*) * tr->world, cudaMemcpyHostToDevice),
               "peers"))
    return LLMOC_ERR_CUDA;
  tr->connected = true;
  return LLMOC_OK;
}
}  // namespace

llmoc_status llmoc_ep_transport_connect(llmoc_ep_transport* tr, const void* handles) {
  if (!tr || !handles) return fails(LLMOC_ERR_INVALID, "bad arguments");
  DevGuard dg(tr->device);
  const char* hb = static_cast<const char*>(handles);
  for (int r = 0; r < tr->world; ++r) {
    if (r == tr->rank || tr->opened[r]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (!cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc open")) return LLMOC_ERR_CUDA;
    tr->peer[r] = static_cast<char*>(p);
    tr->opened[r] = true;
  }
  return upload_peers(tr);
}

llmoc_status llmoc_ep_transport_connect_local(llmoc_ep_transport* tr, llmoc_ep_transport* const* all) {
  if (!tr || !all) return fails(LLMOC_ERR_INVALID, "bad arguments");
  for (int r = 0; r < tr->world; ++r) {
    if (!all[r] || all[r]->world != tr->world || all[r]->rank != r || all[r]->lay.total != tr->lay.total)
      return fails(LLMOC_ERR_INVALID, "transports of one world, in rank order");
    tr->peer[r] = all[r]->base;
  }
  DevGuard dg(tr->device);
  return upload_peers(tr);
}

void llmoc_ep_transport_destroy(llmoc_ep_transport* tr) {
  if (!tr) return;
  DevGuard dg(tr->device);
  for (int r = 0; r < tr->world; ++r)
    if (tr->opened[r]) cudaIpcCloseMemHandle(tr->peer[r]);
  if (tr->base) cudaFree(tr->base);
  if (tr->ctr) cudaFree(tr->ctr);
  if (tr->peers_dev) cudaFree(tr->peers_dev);
  delete tr;
}

llmoc_status llmoc_ep_transport_set_wait_cycles(llmoc_ep_transport* tr, long long cycles) {
  if (!tr || cycles <= 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  tr->wait_cycles = cycles;
  return LLMOC_OK;
}

int llmoc_ep_transport_error(llmoc_ep_transport* tr) {
  if (!tr) return -1;
  DevGuard dg(tr->device);
  int v = 0;
  if (!cuda_ok(cudaMemcpy(&v, tr->err, 4, cudaMemcpyDeviceToHost), "error word")) return -1;
  return v;
}

size_t llmoc_ep_p2p_workspace_bytes(const llmoc_moe_layer* L, const llmoc_ep_transport* tr, int max_tokens) {
  if (!L || !tr || max_tokens < 0) return 0;
  return ep_p2p_ws(L, tr, max_tokens).total;
}

namespace {
llmoc_status p2p_check(const llmoc_moe_layer* L, const llmoc_ep_transport* tr, int T, uint32_t seq,
                       size_t workspace_bytes, const void* workspace) {
  if (!L || !tr || T < 0 || T > tr->max_tokens || seq == 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (!tr->connected) return fails(LLMOC_ERR_INVALID, "transport not connected");
  if (L->ep_world != tr->world || L->ep_rank != tr->rank || L->d.hidden != tr->hidden || L->d.topk != tr->topk ||
      L->device != tr->device)
    return fails(LLMOC_ERR_INVALID, "shard and transport disagree");
  if (!workspace || workspace_bytes < ep_p2p_ws(L, tr, T).total) return fails(LLMOC_ERR_WORKSPACE, "workspace too small");
  return LLMOC_OK;
}
}  // namespace

llmoc_status llmoc_ep_p2p_send(const llmoc_moe_layer* L, llmoc_ep_transport* tr, const uint16_t* X, int T,
                               uint32_t seq, void* workspace, size_t workspace_bytes, void* stream) {
  llmoc_status rc = p2p_check(L, tr, T, seq, workspace_bytes, workspace);
  if (rc != LLMOC_OK) return rc;
  if (T > 0 && !X) return fails(LLMOC_ERR_INVALID, "bad arguments");
  const EpP2PWs w = ep_p2p_ws(L, tr, T);
  char* ws = (char*)workspace;
  rc = ep_dispatch(L, X, T, ws + w.src, w.sw.total, nullptr, (int32_t*)(ws + w.send_expert),
                   (int32_t*)(ws + w.counts), stream, false);
  if (rc != LLMOC_OK) return rc;
  DevGuard dg(L->device);
  // the push reads each routed pair's token row through the dispatch's sorted order
  if (!cuda_ok(launch_ep_push_dispatch(tr->lay, tr->peers_dev, nullptr, (const int*)(ws + w.send_expert),
                                       (const int*)(ws + w.counts), tr->rank, seq, tr->ctr, (cudaStream_t)stream, X,
                                       (const int*)(ws + w.src + w.sw.sorted), L->d.topk),
               "ep push"))
    return LLMOC_ERR_CUDA;
  count_launch(1);
  // the shared expert of this rank's tokens while the rows travel (finish only combines)
  return ep_shared(L, X, T, w.sw, ws + w.src, (cudaStream_t)stream);
}

llmoc_status llmoc_ep_p2p_serve(const llmoc_moe_layer* L, llmoc_ep_transport* tr, int T, uint32_t seq,
                                void* workspace, size_t workspace_bytes, void* stream) {
  llmoc_status rc = p2p_check(L, tr, T, seq, workspace_bytes, workspace);
  if (rc != LLMOC_OK) return rc;
  const EpP2PWs w = ep_p2p_ws(L, tr, T);
  char* ws = (char*)workspace;
  cudaStream_t st = (cudaStream_t)stream;
  DevGuard dg(L->device);
  const int parity = seq & 1, slots = tr->world * tr->lay.cap;
  const uint16_t* rows =
      (const uint16_t*)(tr->base + tr->lay.recv_rows + (size_t)parity * slots * tr->lay.row_bytes);
  const int32_t* ids = (const int32_t*)(tr->base + tr->lay.recv_ids + (size_t)parity * slots * 4);
  // the grouped FFN over the padded slots, without the output-row pass: the
  // return push reads the down GEMM's fp32 rows through the inverse map
  const int n_hint = std::max(1, T * L->d.topk);
  // the permutation reads only each source's occupied slots (its count in the meta)
  PermSegs segs;
  segs.count = (const int*)(tr->base + tr->lay.meta) + (size_t)parity * tr->world * 2;
  segs.stride = 2;
  segs.len = tr->lay.cap;
  segs.n = tr->world;
  // the wait for every source's dispatch flag runs inside the permutation kernel
  segs.wait.flags = (const uint32_t*)(tr->base + tr->lay.flags);
  segs.wait.n = tr->world;
  segs.wait.seq = seq;
  segs.wait.err = tr->err;
  segs.wait.budget = tr->wait_cycles;
  rc = ep_experts(L, rows, ids, slots, n_hint, nullptr, ws + w.own, ep_owner_bytes(L, slots), stream, segs);
  if (rc != LLMOC_OK) return rc;
  const WsLayout wo = ws_layout_g(L, slots, 1, L->n_exp, chunk_for_rows(n_hint, L->e_loc), false);
  if (!cuda_ok(launch_ep_push_return(tr->lay, tr->peers_dev, tr->base, (const float*)(ws + w.own + wo.partial),
                                     (const int*)(ws + w.own + wo.inverse), tr->rank, seq, tr->ctr + 1, st),
               "ep push back"))
    return LLMOC_ERR_CUDA;
  count_launch(1);
  return LLMOC_OK;
}

llmoc_status llmoc_ep_p2p_finish(const llmoc_moe_layer* L, llmoc_ep_transport* tr, const uint16_t* X, int T,
                                 uint16_t* Y, uint32_t seq, void* workspace, size_t workspace_bytes, void* stream) {
  llmoc_status rc = p2p_check(L, tr, T, seq, workspace_bytes, workspace);
  if (rc != LLMOC_OK) return rc;
  if (T > 0 && (!X || !Y)) return fails(LLMOC_ERR_INVALID, "bad arguments");
  const EpP2PWs w = ep_p2p_ws(L, tr, T);
  char* ws = (char*)workspace;
  DevGuard dg(L->device);
  const uint16_t* ret = (const uint16_t*)(tr->base + tr->lay.ret_rows + (size_t)(seq & 1) * tr->lay.cap * tr->lay.row_bytes);
  // the wait for every owner's return flag runs inside the combine kernel
  FlagWait fw;
  fw.flags = (const uint32_t*)(tr->base + tr->lay.flags) + tr->world;  // kind 1: returns
  fw.n = tr->world;
  fw.seq = seq;
  fw.err = tr->err;
  fw.budget = tr->wait_cycles;
  if (T == 0) {  // nothing to combine; the return flags are still waited for (the step's parity is reused)
    if (!cuda_ok(launch_ep_wait(tr->lay, tr->base, 1, seq, tr->err, tr->wait_cycles, (cudaStream_t)stream),
                 "ep wait back"))
      return LLMOC_ERR_CUDA;
    count_launch(1);
    return LLMOC_OK;
  }
  return ep_combine_rows(L, T, ret, Y, w.sw, ws + w.src, (cudaStream_t)stream, fw);
}

}  // extern "C"

namespace llmoc {
// Device a layer lives on (used by the allocation-free entry point in no_alloc.cu).
int layer_device(const llmoc_moe_layer* L) { return L ? L->device : -1; }
}  // namespace llmoc

namespace llmoc {
// Sets the text llmoc_last_error() returns on this thread.
void set_last_error(const std::string& msg) { t_err = msg; }
}  // namespace llmoc

// ------------------------------------------------------ NVLink collectives

struct llmoc_collective {
  int world = 1, rank = 0, device = 0;
  llmoc::CollLayout lay{};
  uint32_t seq = 0;                // steps started
  bool open_step = false;          // a start without its finish
  int open_op = 0, open_root = 0;  // the open step's operation, root and size (its finish must match)
  size_t open_bytes = 0;
  char* base = nullptr;            // this rank's buffer (exported by CUDA IPC)
  std::vector<char*> peer;         // every rank's buffer as seen from here
  std::vector<bool> opened;
  char** peers_dev = nullptr;
  int* ctr = nullptr;              // device: CTA counters of the push and consume kernels
  int* err = nullptr;              // device: bit 1 = a wait gave up
  long long wait_cycles = llmoc::kDefaultWaitCycles;  // budget of each bounded wait
  bool connected = false;
};

llmoc_status llmoc_collective_create(int world, int rank, size_t max_bytes, int device, llmoc_collective** out,
                                     void* ipc_handle) {
  if (!out || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || max_bytes == 0 ||
      max_bytes > ((size_t)1 << 34))
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  *out = nullptr;
  DevGuard dg(device);
  auto* c = new llmoc_collective();
  c->world = world;
  c->rank = rank;
  c->device = device;
  CollLayout& l = c->lay;
  l.world = world;
  l.slot = align256(max_bytes);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes);
    return at;
  };
  l.flags = take((size_t)world * 4);
  l.acks = take((size_t)world * 4);
  l.stage = take((size_t)2 * world * l.slot);
  l.total = o;
  bool ok = cuda_ok(cudaMalloc((void**)&c->base, l.total), "collective buffer") &&
            cuda_ok(cudaMemset(c->base, 0, l.total), "collective memset") &&
            cuda_ok(cudaMalloc((void**)&c->ctr, 64), "collective counters") &&
            cuda_ok(cudaMemset(c->ctr, 0, 64), "collective memset") &&
            cuda_ok(cudaMalloc((void**)&c->peers_dev, sizeof(char*) * world), "collective peers");
  c->err = c->ctr + 8;
  if (ok && ipc_handle) {
    cudaIpcMemHandle_t h;
    ok = cuda_ok(cudaIpcGetMemHandle(&h, c->base), "ipc handle");
    if (ok) memcpy(ipc_handle, &h, sizeof(h));
  }
  c->peer.assign(world, nullptr);
  c->opened.assign(world, false);
  c->peer[rank] = c->base;
  if (!ok) {
    llmoc_collective_destroy(c);
    return LLMOC_ERR_CUDA;
  }
  *out = c;
  return LLMOC_OK;
}

namespace {
llmoc_status coll_upload_peers(llmoc_collective* c) {
  if (!cuda_ok(cudaMemcpy(c->peers_dev, c->peer.data(), sizeof(char*) * c->world, cudaMemcpyHostToDevice),
               "collective peers"))
    return LLMOC_ERR_CUDA;
  c->connected = true;
  return LLMOC_OK;
}
}  // namespace

llmoc_status llmoc_collective_connect(llmoc_collective* c, const void* handles) {
  if (!c || !handles) return fails(LLMOC_ERR_INVALID, "bad arguments");
  DevGuard dg(c->device);
  const char* hb = static_cast<const char*>(handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->opened[r]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (!cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc open")) return LLMOC_ERR_CUDA;
    c->peer[r] = static_cast<char*>(p);
    c->opened[r] = true;
  }
  return coll_upload_peers(c);
}

llmoc_status llmoc_collective_connect_local(llmoc_collective* c, llmoc_collective* const* all) {
  if (!c || !all) return fails(LLMOC_ERR_INVALID, "bad arguments");
  for (int r = 0; r < c->world; ++r) {
    if (!all[r] || all[r]->world != c->world || all[r]->rank != r || all[r]->lay.total != c->lay.total)
      return fails(LLMOC_ERR_INVALID, "collectives of one world, in rank order");
    c->peer[r] = all[r]->base;
  }
  DevGuard dg(c->device);
  return coll_upload_peers(c);
}

void llmoc_collective_destroy(llmoc_collective* c) {
  if (!c) return;
  DevGuard dg(c->device);
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) cudaIpcCloseMemHandle(c->peer[r]);
  if (c->base) cudaFree(c->base);
  if (c->ctr) cudaFree(c->ctr);
  if (c->peers_dev) cudaFree(c->peers_dev);
  delete c;
}

int llmoc_collective_world_size(const llmoc_collective* c) { return c ? c->world : 0; }

llmoc_status llmoc_collective_set_wait_cycles(llmoc_collective* c, long long cycles) {
  if (!c || cycles <= 0) return fails(LLMOC_ERR_INVALID, "bad arguments");
  c->wait_cycles = cycles;
  return LLMOC_OK;
}

int llmoc_collective_error(llmoc_collective* c) {
  if (!c) return -1;
  DevGuard dg(c->device);
  int v = 0;
  if (!cuda_ok(cudaMemcpy(&v, c->err, 4, cudaMemcpyDeviceToHost), "error word")) return -1;
  return v;
}

namespace {
// whether (op, bytes, root, dtype) is a valid step for this collective
bool coll_shape(const llmoc_collective* c, int op, size_t bytes, int root, int dtype) {
  if (bytes == 0 || bytes > c->lay.slot) return false;
  if (op == LLMOC_COLL_ALLREDUCE_SUM) return (dtype == LLMOC_DTYPE_F32 && bytes % 4 == 0) ||
                                             (dtype == LLMOC_DTYPE_BF16 && bytes % 2 == 0);
  if (op == LLMOC_COLL_BROADCAST) return root >= 0 && root < c->world;
  return op == LLMOC_COLL_ALLTOALL;
}
}  // namespace

llmoc_status llmoc_collective_start(llmoc_collective* c, int op, const void* src, size_t bytes, int root,
                                    void* stream) {
  // start sees no dtype: the looser (bf16) size rule here, the exact one in finish
  if (!c || !src || c->open_step || !coll_shape(c, op, bytes, root, LLMOC_DTYPE_BF16))
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  if (!c->connected) return fails(LLMOC_ERR_INVALID, "collective not connected");
  DevGuard dg(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  const uint32_t seq = c->seq + 1;
  // staging parity seq & 1 was last used by step seq - 2: every rank must have consumed it
  if (seq > 2 && !cuda_ok(launch_coll_wait(c->lay, c->base, 1, seq - 2, c->err, c->wait_cycles, st), "collective wait acks"))
    return LLMOC_ERR_CUDA;
  const size_t n = op == LLMOC_COLL_BROADCAST && root != c->rank ? 0 : bytes;
  const size_t stride = op == LLMOC_COLL_ALLTOALL ? bytes : 0;
  if (!cuda_ok(launch_coll_push(c->lay, c->peers_dev, src, stride, n, c->rank, seq, c->ctr, st), "collective push"))
    return LLMOC_ERR_CUDA;
  count_launch(seq > 2 ? 2 : 1);
  c->seq = seq;
  c->open_step = true;
  c->open_op = op;
  c->open_bytes = bytes;
  c->open_root = op == LLMOC_COLL_BROADCAST ? root : 0;
  return LLMOC_OK;
}

llmoc_status llmoc_collective_finish(llmoc_collective* c, int op, void* dst, size_t bytes, int dtype, int root,
                                     void* stream) {
  if (!c || !dst || !c->open_step || !coll_shape(c, op, bytes, root, dtype))
    return fails(LLMOC_ERR_INVALID, "bad arguments");
  // the finish consumes what its start staged: same operation, size and root
  if (op != c->open_op || bytes != c->open_bytes || (op == LLMOC_COLL_BROADCAST && root != c->open_root))
    return fails(LLMOC_ERR_INVALID, "collective finish does not match its start (operation, bytes or root)");
  DevGuard dg(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  if (!cuda_ok(launch_coll_wait(c->lay, c->base, 0, c->seq, c->err, c->wait_cycles, st), "collective wait flags") ||
      !cuda_ok(launch_coll_consume(c->lay, c->base, c->peers_dev, op, dst, bytes, dtype, root, c->rank, c->seq,
                                   c->ctr + 1, st),
               "collective consume"))
    return LLMOC_ERR_CUDA;
  count_launch(2);
  c->open_step = false;
  return LLMOC_OK;
}

llmoc_status llmoc_collective_alltoall(llmoc_collective* c, const void* send, void* recv, size_t bytes,
                                       void* stream) {
  llmoc_status rc = llmoc_collective_start(c, LLMOC_COLL_ALLTOALL, send, bytes, 0, stream);
  return rc != LLMOC_OK ? rc : llmoc_collective_finish(c, LLMOC_COLL_ALLTOALL, recv, bytes, 0, 0, stream);
}

llmoc_status llmoc_collective_allreduce_sum(llmoc_collective* c, void* inout, size_t bytes, int dtype, void* stream) {
  llmoc_status rc = llmoc_collective_start(c, LLMOC_COLL_ALLREDUCE_SUM, inout, bytes, 0, stream);
  return rc != LLMOC_OK ? rc : llmoc_collective_finish(c, LLMOC_COLL_ALLREDUCE_SUM, inout, bytes, dtype, 0, stream);
}

llmoc_status llmoc_collective_broadcast(llmoc_collective* c, void* buf, size_t bytes, int root, void* stream) {
  llmoc_status rc = llmoc_collective_start(c, LLMOC_COLL_BROADCAST, buf, bytes, root, stream);
  return rc != LLMOC_OK ? rc : llmoc_collective_finish(c, LLMOC_COLL_BROADCAST, buf, bytes, 0, root, stream);
}
