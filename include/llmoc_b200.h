/*
 * llmoc_b200.h — C ABI of the B200 (sm_100a) INT4 weight-only MoE expert-FFN
 * library that replaces llm-on-cpu's hal::cuda INT4 / MoE entry points.
 *
 * Every entry point below names the reference interface it stands in for
 * (paths inside appolloqin/llm-on-cpu).  The plain structs are layout-
 * identical to the reference's C++ types, so the reference can pass its own
 * objects through a reinterpret_cast.
 *
 * Conventions
 *  - llmoc_try_* keep the reference's bool contract: 1 = done, 0 = not done
 *    (the caller may then run its own CPU path).  The reason for a 0 is in
 *    llmoc_last_error().  They take host fp32 pointers and are synchronous,
 *    like the reference (cuda_backend.cpp:2692-2728).
 *  - llmoc_moe_* (the batched device API) return llmoc_status; pointers are
 *    device pointers; work is enqueued on the given stream (cudaStream_t
 *    passed as void*, NULL = the legacy default stream) and is asynchronous.
 *  - INT4 layout: qweight [M, ceil(K/2)] bytes, low nibble = even k;
 *    scales/zeros [M, ceil(K/group_size)] fp16 bits, row-major
 *    (src/weights/qlwc_format.h:34-46).  Scheme 2 (AWQ sym): w = (q - zp) * s;
 *    scheme 1 (GPTQ asym): w = q * s + z (src/hal/int4_ops.cpp:640-662).
 */
#ifndef LLMOC_B200_H
#define LLMOC_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LLMOC_API __attribute__((visibility("default")))
#else
#define LLMOC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- types */

typedef enum llmoc_status {
  LLMOC_OK = 0,
  LLMOC_ERR_INVALID = 1,     /* bad argument or shape */
  LLMOC_ERR_NO_DEVICE = 2,   /* no CUDA device / not sm_100 */
  LLMOC_ERR_CUDA = 3,        /* a CUDA call failed */
  LLMOC_ERR_NO_MEMORY = 4,   /* allocation failed or VRAM budget exhausted */
  LLMOC_ERR_NOT_ENABLED = 5, /* llmoc_cuda_enable() not called */
  LLMOC_ERR_UNSUPPORTED = 6, /* shape or scheme this build does not handle */
  LLMOC_ERR_WORKSPACE = 7,   /* workspace too small */
  LLMOC_ERR_TIMEOUT = 8      /* a bounded device-side wait gave up */
} llmoc_status;

enum { LLMOC_SCHEME_GPTQ_ASYM = 1, LLMOC_SCHEME_AWQ_SYM = 2 };
enum { LLMOC_ROUTER_SOFTMAX = 0, LLMOC_ROUTER_SIGMOID_BIAS = 1 };

/* Layout-identical to qlwc::Int4View (src/weights/qlwc_store.h:17-27). */
typedef struct llmoc_int4_view {
  const uint8_t* qweight;
  const uint16_t* scales;
  const uint16_t* zeros;
  const float* scales_f32; /* ignored */
  int32_t M, K;
  int32_t group_size;
  uint32_t scheme; /* LLMOC_SCHEME_* (qlwc::Scheme) */
  int32_t awq_zp;  /* <= 0 means 7 */
} llmoc_int4_view;

/* Layout-identical to hal::cuda::MoeExpertInt4 (src/hal/cuda_backend.h:180-185). */
typedef struct llmoc_moe_expert_int4 {
  const llmoc_int4_view* gate;
  const llmoc_int4_view* up;
  const llmoc_int4_view* down;
  float weight;
} llmoc_moe_expert_int4;

/* ------------------------------------------------------------ lifecycle */

/* hal::cuda::probe_available (src/hal/cuda_backend.h:14; .cpp:733) */
LLMOC_API int llmoc_cuda_probe_available(void);
/* hal::cuda::enabled (cuda_backend.h:15) */
LLMOC_API int llmoc_cuda_enabled(void);
/* hal::cuda::status (cuda_backend.h:16) — also the last error text */
LLMOC_API const char* llmoc_cuda_status(void);
/* hal::cuda::device_count (cuda_backend.h:17) */
LLMOC_API int llmoc_cuda_device_count(void);
/* hal::cuda::enable (cuda_backend.h:21; .cpp:917).  Budget caps the resident
 * INT4 weight cache of the llmoc_try_* entry points (0 = unlimited). */
LLMOC_API int llmoc_cuda_enable(size_t vram_budget_bytes);
/* hal::cuda::disable (cuda_backend.h:22; .cpp:947): frees the weight cache. */
LLMOC_API void llmoc_cuda_disable(void);
/* hal::cuda::vram_used / vram_budget / set_vram_budget (cuda_backend.h:24-27) */
LLMOC_API size_t llmoc_cuda_vram_used(void);
LLMOC_API size_t llmoc_cuda_vram_budget(void);
LLMOC_API void llmoc_cuda_set_vram_budget(size_t bytes);
/* hal::cuda::device_mem_info (cuda_backend.h:29) */
LLMOC_API int llmoc_cuda_device_mem_info(size_t* free_bytes, size_t* total_bytes);
/* hal::cuda::host_register / host_unregister (cuda_backend.h:32-33) */
LLMOC_API int llmoc_cuda_host_register(void* ptr, size_t bytes);
LLMOC_API int llmoc_cuda_host_unregister(void* ptr);
/* Text of the last failure on the calling thread ("" if none). */
LLMOC_API const char* llmoc_last_error(void);

/* ------------------------------------------------- INT4 GEMM (host fp32) */

/* hal::cuda::try_gemm_int4 (cuda_backend.h:165; .cpp:2692): y[M] = W . x */
LLMOC_API int llmoc_try_gemm_int4(const float* x, const llmoc_int4_view* W, float* y);
/* hal::gemm_int4_argmax (int4_ops.h:13-19; .cpp:344-446): greedy decode over
 * an INT4 lm_head, argmax_m of (W . x)[m] without returning the logits.  Row
 * values as the reference sums them (within the GEMV tolerance); non-finite
 * rows count as -1e30; equal maxima -> the smallest row.  index/value are the
 * fields of hal::Int4ArgmaxResult.  1 = done, 0 = the caller runs its CPU path. */
LLMOC_API int llmoc_try_gemm_int4_argmax(const float* x, const llmoc_int4_view* W, int32_t* index, float* value);
/* hal::cuda::try_gemm_int4_batch (cuda_backend.h:166; .cpp:2858): Y[n,M] = X[n,K] . W^T */
LLMOC_API int llmoc_try_gemm_int4_batch(const float* X, int n, const llmoc_int4_view* W, float* Y);
/* hal::cuda::try_gemm_int4_multi (cuda_backend.h:172; .cpp:3048): 2..4 weights sharing x */
LLMOC_API int llmoc_try_gemm_int4_multi(const float* x, const llmoc_int4_view* const* Ws, float* const* ys,
                              int n);
/* hal::cuda::try_gemm_int4_batch_multi (cuda_backend.h:170-171) */
LLMOC_API int llmoc_try_gemm_int4_batch_multi(const float* X, int n, const llmoc_int4_view* const* Ws,
                                    float* const* Ys, int nW);
/* hal::cuda::prefetch_int4_weight / pin_int4_weight (cuda_backend.h:173-175; .cpp:5199-5215):
 * upload (repacked) into the resident cache keyed by W->qweight; pin exempts it from LRU. */
LLMOC_API int llmoc_prefetch_int4_weight(const llmoc_int4_view* W);
LLMOC_API int llmoc_pin_int4_weight(const llmoc_int4_view* W);
/* hal::dequant_int4_matrix (src/hal/int4_ops.h:27; int4_ops.cpp:664-668) run on
 * the GPU from the resident repacked copy: out[M*K] fp32 host, bit-exact. */
LLMOC_API int llmoc_try_dequant_int4_matrix(const llmoc_int4_view* W, float* out);

/* ---------------------------------------------------- fused MoE (1 token) */

/* hal::cuda::try_moe_ffn_int4 (src/hal/cuda_backend.h:186-188; .cpp:5217-5317):
 * y[H] = sum_i experts[i].weight * down_i(silu(gate_i x) * up_i x)
 *        + shared_scale * shared(x); y is overwritten; n_experts <= 64;
 * experts with |weight| < 1e-12 are skipped. */
LLMOC_API int llmoc_try_moe_ffn_int4(const float* x, int H, int I, const llmoc_moe_expert_int4* experts,
                           int n_experts, const llmoc_int4_view* shared_gate,
                           const llmoc_int4_view* shared_up, const llmoc_int4_view* shared_down,
                           float shared_scale, float* y);

/* ------------------------------------------- batched device-resident layer */

/* One MoE layer uploaded once into HBM in the kernels' repacked layout: the
 * replacement for the per-token moe_ffn_token loop
 * (src/model/qwen3_6_moe_int4_model.cpp:377-404, called per token from
 * src/model/qwen3_5_int4_model.cpp:1204-1208) and for the expert slot cache
 * (src/moe/offload_cache.h:24-91, src/moe/host_banks.h:54-111). */
typedef struct llmoc_moe_layer llmoc_moe_layer;

typedef struct llmoc_moe_layer_desc {
  int32_t hidden;         /* H */
  int32_t inter;          /* I (routed and shared experts) */
  int32_t n_experts;      /* E routed experts */
  int32_t topk;           /* k <= 64 (qwen3_6_moe_int4_model.cpp:384) */
  int32_t group_size;     /* INT4 group along K */
  int32_t scheme;         /* LLMOC_SCHEME_* (all experts) */
  int32_t awq_zp;         /* <= 0 means 7 */
  int32_t router;         /* LLMOC_ROUTER_* */
  float routed_scaling;   /* sigmoid router: weight multiplier */
  int32_t has_shared;     /* 1: one always-on shared expert */
  float shared_scale;     /* its combine weight */
} llmoc_moe_layer_desc;

/* Create from host QLWC views: router_w [E,H] bf16, bias [E] fp32 (sigmoid
 * router, else NULL), experts[3*E] = (gate, up, down) per expert, shared[3]
 * or NULL.  Uploads and repacks on `device`.  The host buffers are not kept. */
LLMOC_API llmoc_status llmoc_moe_layer_create(const llmoc_moe_layer_desc* desc, const uint16_t* router_w,
                                    const float* bias, const llmoc_int4_view* experts,
                                    const llmoc_int4_view* shared, int device,
                                    llmoc_moe_layer** out);
/* Same, but every pointer (router_w, bias, and the views' qweight/scales/zeros)
 * is a device pointer on `device` (no host staging; used to build large layers
 * directly in HBM). */
LLMOC_API llmoc_status llmoc_moe_layer_create_device(const llmoc_moe_layer_desc* desc,
                                           const uint16_t* router_w, const float* bias,
                                           const llmoc_int4_view* experts,
                                           const llmoc_int4_view* shared, int device,
                                           llmoc_moe_layer** out);
LLMOC_API void llmoc_moe_layer_destroy(llmoc_moe_layer* layer);
/* Bytes of resident expert weights (packed q + fp16 scales/zeros), router excluded. */
LLMOC_API size_t llmoc_moe_layer_weight_bytes(const llmoc_moe_layer* layer);
/* Bytes one expert streams per forward (src/moe/qlwc_expert_bytes.h:43-60). */
LLMOC_API size_t llmoc_expert_storage_bytes(int H, int I, int group_size, int has_zeros);

/* Per-token weight of the shared expert: sigmoid(gate_row . x) instead of the
 * constant shared_scale (Qwen3.6-style shared_expert_gate, bf16 [hidden],
 * host or device memory): the reference's `gemm_opt(normed,
 * lp.shared_expert_gate)` + `sigmoid`
 * (src/model/qwen3_6_moe_int4_model.cpp:365-371, :29).  The gate row joins the
 * router GEMV (same summation order); the layer must have a shared expert.
 * Works for single-GPU layers and expert-parallel shards. */
LLMOC_API llmoc_status llmoc_moe_layer_set_shared_gate(llmoc_moe_layer* layer, const uint16_t* gate_row,
                                                       int on_device);

/* A layer straight from a QLWC v1 file, the reference's INT4 container
 * (src/weights/qlwc_format.h; written by tools/quantize_int4.py): tensors
 * `<prefix>layers.<layer>.mlp.experts.<e>.{gate,up,down}_proj.weight` (INT4),
 * `.mlp.gate.weight` (bf16 router), optional `.mlp.shared_expert(s).*_proj`,
 * `.mlp.shared_expert_gate.weight` and `.mlp.gate.e_score_correction_bias`
 * (the names of src/model/qwen3_6_moe_int4_model.cpp:201 and
 * src/model/moe_model.cpp:308-364).  Replaces the host-bank fill of
 * QlwcExpertHostBanks::fill_from_qlwc (src/moe/host_banks.cpp:165-261): the
 * experts are read once and uploaded to HBM, repacked. */
typedef struct llmoc_qlwc_layer_info {
  int32_t hidden, inter, n_experts, group_size, scheme;
  int32_t has_router, has_shared, has_shared_gate, has_bias;
} llmoc_qlwc_layer_info;
LLMOC_API llmoc_status llmoc_qlwc_describe(const char* path, const char* prefix, int layer,
                                           llmoc_qlwc_layer_info* out);
/* The layer numbers n of the file's MoE layers (those holding an INT4
 * "<prefix>layers.<n>.mlp.experts.0.gate_proj.weight"), ascending: writes up to
 * max_layers of them and returns how many there are, or -1 (bad file). */
LLMOC_API int llmoc_qlwc_moe_layers(const char* path, const char* prefix, int32_t* layers, int max_layers);
/* desc gives what the file does not hold (topk, router kind, routed scaling,
 * shared scale) and must agree with it on the rest (llmoc_qlwc_describe). */
LLMOC_API llmoc_status llmoc_moe_layer_create_qlwc(const char* path, const char* prefix, int layer,
                                                   const llmoc_moe_layer_desc* desc, int device,
                                                   llmoc_moe_layer** out);

/* Workspace (device memory the caller provides) for up to max_tokens tokens. */
LLMOC_API size_t llmoc_moe_workspace_bytes(const llmoc_moe_layer* layer, int max_tokens);

/* Y[T,H] bf16 = MoE(X[T,H] bf16): router GEMV (fp32, the reference's
 * summation order), softmax or sigmoid+bias top-k, renormalise, canonical
 * permutation, grouped INT4 gate/up + SiLU*mul, down, weighted combine (+ the
 * shared expert).  T may be 0 (no work).  Asynchronous on `stream`. */
LLMOC_API llmoc_status llmoc_moe_forward(const llmoc_moe_layer* layer, const uint16_t* X, int T, uint16_t* Y,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Y = R + MoE(X): the forward above with the decoder's residual add fused
 * into the weighted combine (y = bf16(float(r) + sum), one rounding), so the
 * residual stream stays on the device.  Replaces the per-token
 * `down_acc` + caller-side add of src/model/qwen3_5_int4_model.cpp:1204-1208
 * for a batch.  R may alias Y (in-place residual) and both may alias X. */
LLMOC_API llmoc_status llmoc_moe_forward_residual(const llmoc_moe_layer* layer, const uint16_t* X, int T,
                                                  const uint16_t* R, uint16_t* Y, void* workspace,
                                                  size_t workspace_bytes, void* stream);

/* Routing results inside a workspace after llmoc_moe_forward / llmoc_moe_route
 * (device pointers; kk = topk + has_shared slots per token):
 *   logits [T,E] fp32 ([T,E+1] with a shared gate: its logit last); ids [T,kk] int32; weights [T,kk] fp32;
 *   offsets [E+has_shared+1] int32; sorted [T*kk] int32 (= t*kk + j);
 *   inverse [T*kk] int32; n_active: number of experts with >= 1 pair;
 *   error_flag: 0, or bit 0 set when a bounded device-side wait gave up
 *   (the outputs of that forward are then not valid). */
typedef struct llmoc_route_views {
  float* logits;
  int32_t* ids;
  float* weights;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* inverse;
  int32_t* n_active;
  int32_t* error_flag;
} llmoc_route_views;
LLMOC_API llmoc_status llmoc_moe_route_views(const llmoc_moe_layer* layer, int T, void* workspace,
                                   size_t workspace_bytes, llmoc_route_views* out);
/* Routing and permutation only (no expert FFN). */
LLMOC_API llmoc_status llmoc_moe_route(const llmoc_moe_layer* layer, const uint16_t* X, int T,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Dequantise one resident projection (proj 0 gate, 1 up, 2 down; expert ==
 * n_experts selects the shared expert) from the repacked layout into
 * out[M*K] fp32 (device), bit-exact with hal::dequant_int4_matrix. */
LLMOC_API llmoc_status llmoc_moe_dequant(const llmoc_moe_layer* layer, int expert, int proj, float* out,
                               void* stream);

/* Budget, in SM clocks, of each grid-wide barrier wait inside the fused
 * single-token forward (T = 1: the router, top-k, both GEMMs and the combine
 * in one launch).  A wait that runs out sets bit 2 (value 4) of the
 * workspace's error word (llmoc_route_views.error_flag) and the launch goes
 * on, its outputs then invalid; the next forward starts clean.  Default 2^31
 * (about a second).  No reference counterpart (its decode is host-driven). */
LLMOC_API llmoc_status llmoc_moe_layer_set_wait_cycles(llmoc_moe_layer* layer, long long cycles);

/* Per-stage CUDA-event timing of llmoc_moe_forward (the reference only keeps
 * wall-clock accumulators, src/hal/cuda_backend.cpp:285-288, :5347-5357).
 * While enabled, every forward records events around its six stages on its
 * stream: 0 router GEMV, 1 top-k, 2 permutation, 3 gate/up + SiLU*mul,
 * 4 down, 5 combine (a forward of one token runs as one launch, reported
 * under stage 3).  llmoc_moe_stage_times synchronizes on the recorded
 * events, writes the summed milliseconds per stage into ms[6] and the number
 * of timed calls into *calls, and clears the record.  Disabling also clears. */
LLMOC_API llmoc_status llmoc_moe_set_stage_timing(llmoc_moe_layer* layer, int enable);
LLMOC_API llmoc_status llmoc_moe_stage_times(llmoc_moe_layer* layer, float* ms, int* calls);

/* Allocation-free forward (no counterpart in the reference).  For callers
 * that cannot provide device memory for a workspace — their device memory is
 * owned by another allocator, or their serving loop must not call
 * cudaMalloc/cudaFree (which synchronize the device), or they reach this
 * library through an FFI without a device allocator — this runs
 * llmoc_moe_forward with its workspace in a fixed file-scope device array of
 * llmoc_moe_noalloc_capacity() bytes (8 MiB) that every GPU loading the
 * library holds until the process exits.  It allocates nothing.  The first
 * call on a device looks up the array's device address; make that first call
 * before any stream capture on the device.  Returns LLMOC_ERR_WORKSPACE when
 * llmoc_moe_workspace_bytes(layer, T) exceeds the capacity.  All calls on a
 * device share the array: calls whose work overlaps on the GPU race and must
 * be serialized by the caller.  The cached address belongs to the device's
 * context: after cudaDeviceReset it is stale, so a process that resets a
 * device must not call this entry point again. */
LLMOC_API llmoc_status llmoc_moe_forward_noalloc(const llmoc_moe_layer* layer, const uint16_t* X,
                                                 int T, uint16_t* Y, void* stream);
LLMOC_API size_t llmoc_moe_noalloc_capacity(void);
/* Synchronizes `stream`, then reads the device error word that the last
 * llmoc_moe_forward_noalloc call of T tokens on the layer's device left in
 * the static array (the caller has no workspace pointer to read it through):
 * LLMOC_ERR_TIMEOUT when one of that forward's bounded device-side waits gave
 * up (its outputs are then not valid), LLMOC_OK otherwise. */
LLMOC_API llmoc_status llmoc_moe_noalloc_status(const llmoc_moe_layer* layer, int T, void* stream);

/* ------------------------------------------------- expert parallelism (EP)
 * The reference gives only the contracts: expert e is owned by rank
 * e % world (DeviceMesh::owner_rank with EpShard::kMod,
 * src/contracts/device_mesh.h:63-72) and the transport is an all-to-all
 * (ICollective::alltoall, src/contracts/collective.h:13).  A layer shard
 * created with llmoc_moe_layer_create_ep holds the routed experts e with
 * e % world == rank (owner-local id e / world), the replicated router and the
 * shared expert.  One forward of T tokens on every rank is:
 *   1. llmoc_moe_ep_dispatch: route the rank's T tokens over all n_experts,
 *      order the T*topk routed pairs by (owner rank, owner-local expert,
 *      token, slot), write their bf16 rows to send_rows [T*topk][hidden], the
 *      owner-local expert ids to send_expert, and per-rank pair counts to
 *      send_counts [world] (all device memory);
 *   2. the caller exchanges counts, rows and expert ids with an all-to-all;
 *   3. llmoc_moe_ep_experts on the received rows (any order; expert ids
 *      owner-local) writes each row's expert output (bf16) to out_rows in the
 *      same order;
 *   4. the caller returns out_rows with the inverse all-to-all, so the source
 *      gets its rows back in send order (ret_rows);
 *   5. llmoc_moe_ep_combine (same workspace as step 1): the routed weights
 *      times ret_rows, in slot order, plus the shared expert run locally,
 *      into Y [T][hidden] (bf16).
 * n_experts % world == 0.  llmoc_moe_forward / llmoc_moe_route refuse a shard
 * with world > 1. */
LLMOC_API llmoc_status llmoc_moe_layer_create_ep(const llmoc_moe_layer_desc* desc, const uint16_t* router_w,
                                                 const float* bias, const llmoc_int4_view* experts,
                                                 const llmoc_int4_view* shared, int device, int rank,
                                                 int world, int on_device, llmoc_moe_layer** out);
LLMOC_API size_t llmoc_moe_ep_source_workspace_bytes(const llmoc_moe_layer* layer, int max_tokens);
LLMOC_API size_t llmoc_moe_ep_owner_workspace_bytes(const llmoc_moe_layer* layer, int max_rows);
LLMOC_API llmoc_status llmoc_moe_ep_dispatch(const llmoc_moe_layer* layer, const uint16_t* X, int T,
                                             void* workspace, size_t workspace_bytes, uint16_t* send_rows,
                                             int32_t* send_expert, int32_t* send_counts, void* stream);
LLMOC_API llmoc_status llmoc_moe_ep_experts(const llmoc_moe_layer* layer, const uint16_t* rows,
                                            const int32_t* expert, int n, uint16_t* out_rows, void* workspace,
                                            size_t workspace_bytes, void* stream);
LLMOC_API llmoc_status llmoc_moe_ep_combine(const llmoc_moe_layer* layer, const uint16_t* X, int T,
                                            const uint16_t* ret_rows, uint16_t* Y, void* workspace,
                                            size_t workspace_bytes, void* stream);
/* Step 3 over a fixed-capacity receive layout, for an all-to-all whose split
 * sizes the host never reads (equal splits of world x capacity slots, the
 * transport ICollective::alltoall, src/contracts/collective.h:13, declares):
 * slots whose owner-local expert id lies outside [0, experts of the shard)
 * are empty -- not computed, their out_rows left as they were.  n_hint is
 * the number of occupied slots expected (e.g. the T * topk pairs a source
 * sends); it sizes the work items and the GEMM grids, not the result.  The
 * workspace is llmoc_moe_ep_owner_workspace_bytes(layer, n). */
LLMOC_API llmoc_status llmoc_moe_ep_experts_padded(const llmoc_moe_layer* layer, const uint16_t* rows,
                                                   const int32_t* expert, int n, int n_hint, uint16_t* out_rows,
                                                   void* workspace, size_t workspace_bytes, void* stream);

/* -------------------------- expert-parallel transport over NVLink peer memory
 *
 * The all-to-all of the step above (the reference only declares it:
 * ICollective::alltoall, src/contracts/collective.h:13) done by the library's
 * own kernels: each rank stores its routed rows straight into the owners'
 * receive buffers (CUDA IPC peer pointers, plain stores over NVLink), raises
 * a per-source sequence flag there, and the owners push the expert outputs
 * back the same way.  The step needs no host synchronisation and no library
 * collective:
 *   llmoc_ep_p2p_send    dispatch (as llmoc_moe_ep_dispatch) + push the rows,
 *                        then the shared expert of the rank's tokens
 *   llmoc_ep_p2p_serve   wait for every source, grouped expert FFN over the
 *                        received rows, push the outputs back
 *   llmoc_ep_p2p_finish  wait for every owner, combine (+ the shared expert's rows)
 * all asynchronous on `stream`; every rank calls the three in this order with
 * the same seq = 1, 2, 3, ... (one per layer step).  Waits are bounded
 * (~1 s): a wait that gives up sets bit 1 of llmoc_ep_transport_error and the
 * step's outputs are invalid.  One transport per (shard shape, max_tokens);
 * T <= max_tokens on every call. */
typedef struct llmoc_ep_transport llmoc_ep_transport;
LLMOC_API size_t llmoc_ep_ipc_handle_bytes(void);
/* Allocates this rank's buffers on `device` and writes its CUDA IPC handle
 * (llmoc_ep_ipc_handle_bytes() bytes) to ipc_handle (may be null when every
 * rank lives in this process: llmoc_ep_transport_connect_local). */
LLMOC_API llmoc_status llmoc_ep_transport_create(int world, int rank, int hidden, int max_tokens, int topk,
                                                 int device, llmoc_ep_transport** out, void* ipc_handle);
/* handles: every rank's IPC handle in rank order (world x handle bytes). */
LLMOC_API llmoc_status llmoc_ep_transport_connect(llmoc_ep_transport* tr, const void* handles);
/* All ranks in this process (tests): the world's transports in rank order. */
LLMOC_API llmoc_status llmoc_ep_transport_connect_local(llmoc_ep_transport* tr, llmoc_ep_transport* const* all);
LLMOC_API void llmoc_ep_transport_destroy(llmoc_ep_transport* tr);
/* Reads (synchronously) the device error word: 0, or bit 1 when a wait gave up. */
LLMOC_API int llmoc_ep_transport_error(llmoc_ep_transport* tr);
/* SM clock cycles each of the transport's bounded waits spins before it gives
 * up (default 2^31, about 1.1 s at 1.965 GHz); applies to later calls. */
LLMOC_API llmoc_status llmoc_ep_transport_set_wait_cycles(llmoc_ep_transport* tr, long long cycles);
LLMOC_API size_t llmoc_ep_p2p_workspace_bytes(const llmoc_moe_layer* shard, const llmoc_ep_transport* tr,
                                              int max_tokens);
LLMOC_API llmoc_status llmoc_ep_p2p_send(const llmoc_moe_layer* shard, llmoc_ep_transport* tr, const uint16_t* X,
                                         int T, uint32_t seq, void* workspace, size_t workspace_bytes, void* stream);
LLMOC_API llmoc_status llmoc_ep_p2p_serve(const llmoc_moe_layer* shard, llmoc_ep_transport* tr, int T, uint32_t seq,
                                          void* workspace, size_t workspace_bytes, void* stream);
LLMOC_API llmoc_status llmoc_ep_p2p_finish(const llmoc_moe_layer* shard, llmoc_ep_transport* tr, const uint16_t* X,
                                           int T, uint16_t* Y, uint32_t seq, void* workspace,
                                           size_t workspace_bytes, void* stream);

/* --------------------------------------------------- NVLink collectives */

/* contracts::ICollective (src/contracts/collective.h:9-15) between the ranks
 * of one box, one process (or one ranks' object) per GPU, over peer memory
 * opened with CUDA IPC -- the implementation that exec/mesh_nccl.cpp:85-134
 * leaves as stubs.  Every rank makes the same calls in the same order; each
 * call is a step (numbered inside the object).  Operations (op):
 *   LLMOC_COLL_ALLTOALL       send = world chunks of `bytes`; chunk d goes to
 *                             rank d, which receives it as its chunk `rank`
 *   LLMOC_COLL_ALLREDUCE_SUM  elementwise sum over ranks of a buffer of
 *                             `bytes` (dtype fp32 or bf16; fp32 accumulation
 *                             in rank order, so every rank gets the same bits)
 *   LLMOC_COLL_BROADCAST      root's buffer of `bytes` to every rank
 * bytes <= the max_bytes given at creation; a finish must repeat its start's
 * op, bytes and root (else LLMOC_ERR_INVALID).  Asynchronous on `stream`; a wait
 * that gives up (~1 s) sets bit 1 of llmoc_collective_error and the step's
 * result is invalid.  start / finish split a step in two (the first pushes,
 * the second waits and consumes) so that several ranks' objects can share
 * one stream in one process; the op calls are start + finish. */
enum { LLMOC_COLL_ALLTOALL = 0, LLMOC_COLL_ALLREDUCE_SUM = 1, LLMOC_COLL_BROADCAST = 2 };
enum { LLMOC_DTYPE_F32 = 0, LLMOC_DTYPE_BF16 = 1 };
typedef struct llmoc_collective llmoc_collective;
/* Allocates this rank's buffer (2 x world x max_bytes of staging) and writes
 * its IPC handle (llmoc_ep_ipc_handle_bytes() bytes; may be null for
 * llmoc_collective_connect_local). */
LLMOC_API llmoc_status llmoc_collective_create(int world, int rank, size_t max_bytes, int device,
                                               llmoc_collective** out, void* ipc_handle);
LLMOC_API llmoc_status llmoc_collective_connect(llmoc_collective* c, const void* handles);
LLMOC_API llmoc_status llmoc_collective_connect_local(llmoc_collective* c, llmoc_collective* const* all);
LLMOC_API void llmoc_collective_destroy(llmoc_collective* c);
LLMOC_API int llmoc_collective_world_size(const llmoc_collective* c);
LLMOC_API int llmoc_collective_error(llmoc_collective* c);
/* SM clock cycles each bounded wait spins before it gives up (default 2^31). */
LLMOC_API llmoc_status llmoc_collective_set_wait_cycles(llmoc_collective* c, long long cycles);
LLMOC_API llmoc_status llmoc_collective_start(llmoc_collective* c, int op, const void* src, size_t bytes, int root,
                                              void* stream);
LLMOC_API llmoc_status llmoc_collective_finish(llmoc_collective* c, int op, void* dst, size_t bytes, int dtype,
                                               int root, void* stream);
LLMOC_API llmoc_status llmoc_collective_alltoall(llmoc_collective* c, const void* send, void* recv, size_t bytes,
                                                 void* stream);
LLMOC_API llmoc_status llmoc_collective_allreduce_sum(llmoc_collective* c, void* inout, size_t bytes, int dtype,
                                                      void* stream);
LLMOC_API llmoc_status llmoc_collective_broadcast(llmoc_collective* c, void* buf, size_t bytes, int root,
                                                  void* stream);

/* ------------------------------------------------------------ utilities */

/* quant_awq_sym (tools/quantize_int4.py:150-166) on the device: W [M,K] bf16
 * -> q [M,K/2], scales [M,K/gs] fp16.  bf16_scale rounds each scale to bf16
 * first.  Requires K % gs == 0.  Used to build synthetic layers in HBM. */
LLMOC_API llmoc_status llmoc_quantize_awq_sym(const uint16_t* W, int M, int K, int group_size,
                                    int bf16_scale, uint8_t* q, uint16_t* scales, void* stream);

/* Number of this library's kernels launched since load (all devices). */
LLMOC_API uint64_t llmoc_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* LLMOC_B200_H */
