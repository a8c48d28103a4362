// cuda_backend_b200.cpp — the reference's hal::cuda INT4 / MoE entry points
// (src/hal/cuda_backend.h:14-33, :159-188) implemented on libllmoc_b200.so.
//
// A maintainer compiles this file instead of the INT4/MoE part of
// src/hal/cuda_backend.cpp when the B200 backend is selected; it includes the
// reference's own headers, so the reference passes its qlwc::Int4View and
// hal::cuda::MoeExpertInt4 objects through unchanged.  The static_asserts
// below pin that the library's C structs (include/llmoc_b200.h) have the
// same size and member offsets as those reference types: if either side
// drifts, this file stops compiling.
#include <cstddef>

#include "hal/cuda_backend.h"
#include "hal/int4_ops.h"
#include "llmoc_b200.h"

namespace llmoc::hal::cuda {

static_assert(sizeof(qlwc::Int4View) == sizeof(llmoc_int4_view), "Int4View size");
static_assert(offsetof(qlwc::Int4View, qweight) == offsetof(llmoc_int4_view, qweight), "qweight");
static_assert(offsetof(qlwc::Int4View, scales) == offsetof(llmoc_int4_view, scales), "scales");
static_assert(offsetof(qlwc::Int4View, zeros) == offsetof(llmoc_int4_view, zeros), "zeros");
static_assert(offsetof(qlwc::Int4View, scales_f32) == offsetof(llmoc_int4_view, scales_f32), "scales_f32");
static_assert(offsetof(qlwc::Int4View, M) == offsetof(llmoc_int4_view, M), "M");
static_assert(offsetof(qlwc::Int4View, K) == offsetof(llmoc_int4_view, K), "K");
static_assert(offsetof(qlwc::Int4View, group_size) == offsetof(llmoc_int4_view, group_size), "group_size");
static_assert(offsetof(qlwc::Int4View, scheme) == offsetof(llmoc_int4_view, scheme), "scheme");
static_assert(sizeof(qlwc::Int4View::scheme) == sizeof(llmoc_int4_view::scheme), "scheme width");
static_assert(offsetof(qlwc::Int4View, awq_zp) == offsetof(llmoc_int4_view, awq_zp), "awq_zp");
static_assert(static_cast<int>(qlwc::Scheme::kAwqSym) == LLMOC_SCHEME_AWQ_SYM, "AWQ scheme value");
static_assert(static_cast<int>(qlwc::Scheme::kGptqAsym) == LLMOC_SCHEME_GPTQ_ASYM, "GPTQ scheme value");
static_assert(sizeof(MoeExpertInt4) == sizeof(llmoc_moe_expert_int4), "MoeExpertInt4 size");
static_assert(offsetof(MoeExpertInt4, gate) == offsetof(llmoc_moe_expert_int4, gate), "gate");
static_assert(offsetof(MoeExpertInt4, up) == offsetof(llmoc_moe_expert_int4, up), "up");
static_assert(offsetof(MoeExpertInt4, down) == offsetof(llmoc_moe_expert_int4, down), "down");
static_assert(offsetof(MoeExpertInt4, weight) == offsetof(llmoc_moe_expert_int4, weight), "weight");
static_assert(sizeof(Int4ArgmaxResult::index) == sizeof(int32_t), "argmax index");

static const llmoc_int4_view* V(const qlwc::Int4View& W) { return reinterpret_cast<const llmoc_int4_view*>(&W); }
static const llmoc_int4_view* VP(const qlwc::Int4View* W) { return W ? V(*W) : nullptr; }

bool probe_available() { return llmoc_cuda_probe_available() != 0; }
bool enabled() { return llmoc_cuda_enabled() != 0; }
const char* status() { return llmoc_cuda_status(); }
int device_count() { return llmoc_cuda_device_count(); }
bool enable(size_t vram_budget_bytes) { return llmoc_cuda_enable(vram_budget_bytes) != 0; }
void disable() { llmoc_cuda_disable(); }
size_t vram_used() { return llmoc_cuda_vram_used(); }
size_t vram_budget() { return llmoc_cuda_vram_budget(); }
void set_vram_budget(size_t bytes) { llmoc_cuda_set_vram_budget(bytes); }
bool device_mem_info(size_t* free_bytes, size_t* total_bytes) {
  return llmoc_cuda_device_mem_info(free_bytes, total_bytes) != 0;
}
bool host_register(void* ptr, size_t bytes) { return llmoc_cuda_host_register(ptr, bytes) != 0; }
bool host_unregister(void* ptr) { return llmoc_cuda_host_unregister(ptr) != 0; }

bool try_gemm_int4(const float* x, const qlwc::Int4View& W, float* y) { return llmoc_try_gemm_int4(x, V(W), y) != 0; }
bool try_gemm_int4_batch(const float* X, int n, const qlwc::Int4View& W, float* Y) {
  return llmoc_try_gemm_int4_batch(X, n, V(W), Y) != 0;
}
bool try_gemm_int4_batch_multi(const float* X, int n, const qlwc::Int4View* const* Ws, float* const* Ys, int nW) {
  return llmoc_try_gemm_int4_batch_multi(X, n, reinterpret_cast<const llmoc_int4_view* const*>(Ws), Ys, nW) != 0;
}
bool try_gemm_int4_multi(const float* x, const qlwc::Int4View* const* Ws, float* const* ys, int n) {
  return llmoc_try_gemm_int4_multi(x, reinterpret_cast<const llmoc_int4_view* const*>(Ws), ys, n) != 0;
}
bool prefetch_int4_weight(const qlwc::Int4View& W) { return llmoc_prefetch_int4_weight(V(W)) != 0; }
bool pin_int4_weight(const qlwc::Int4View& W) { return llmoc_pin_int4_weight(V(W)) != 0; }

bool try_moe_ffn_int4(const float* x, int H, int I, const MoeExpertInt4* experts, int n_experts,
                      const qlwc::Int4View* shared_gate, const qlwc::Int4View* shared_up,
                      const qlwc::Int4View* shared_down, float shared_scale, float* y) {
  return llmoc_try_moe_ffn_int4(x, H, I, reinterpret_cast<const llmoc_moe_expert_int4*>(experts), n_experts,
                                VP(shared_gate), VP(shared_up), VP(shared_down), shared_scale, y) != 0;
}

// hal::gemm_int4_argmax (greedy decode over an INT4 lm_head, called at
// src/model/qwen3_5_int4_model.cpp:1848): on the device when it can run,
// else the reference's CPU operator.
Int4ArgmaxResult gemm_int4_argmax_b200(const float* x, const qlwc::Int4View& W) {
  Int4ArgmaxResult r;
  if (llmoc_try_gemm_int4_argmax(x, V(W), &r.index, &r.value)) return r;
  return hal::gemm_int4_argmax(x, W);
}

}  // namespace llmoc::hal::cuda
