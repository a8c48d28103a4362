// ref_shim.cpp — C entry points over the reference's own CPU operators.
//
// TEST INFRASTRUCTURE ONLY.  Linked with the reference's unmodified sources
// src/hal/{int4_ops,cpu_ops,cpu_ops_attn,gated_delta_chunk}.cpp (compiled in
// place from the reference tree by oracle/Makefile) into oracle/_ref/libllmoc_ref.so.
// It is used to pin the plain-C oracle (oracle/moe_oracle.c) bit-for-bit and,
// in bench.py's reference arm, as the timed CPU baseline.  Nothing in the
// CUDA library links it.
//
// The reference's CUDA backend is not built: the two hooks cpu_ops.cpp calls
// (hal::cuda::try_gemm_w16 / try_gemm_w16_batch, src/hal/cuda_backend.h:159-161)
// report "no GPU", which is what the reference does when hal::cuda::enable()
// was never called, so the AVX2/OpenMP CPU path runs.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <numeric>
#include <vector>

#include "hal/cpu_ops.h"
#include "hal/int4_ops.h"

#if defined(_OPENMP)
#include <omp.h>
#endif

namespace llmoc::hal::cuda {
bool try_gemm_w16(const float*, const uint16_t*, float*, int, int, bool) { return false; }
bool try_gemm_w16_batch(const float*, int, const uint16_t*, float*, int, int, bool) {
  return false;
}
}  // namespace llmoc::hal::cuda

using namespace llmoc;

extern "C" {

// Same field order as orc_int4_view in moe_oracle.c.
struct ref_int4_view {
  const uint8_t* qweight;
  const uint16_t* scales;
  const uint16_t* zeros;
  int M, K, group_size;
  int scheme;  // 1 = GPTQ asym, 2 = AWQ sym (qlwc_format.h:22)
  int awq_zp;
};

struct ref_expert {
  ref_int4_view gate, up, down;
};

struct ref_layer {
  int H, I, E, topk;
  int router;  // 0 softmax, 1 sigmoid+bias
  const uint16_t* router_w;
  const float* bias;
  float routed_scaling;
  const ref_expert* experts;
  const ref_expert* shared;
  float shared_scale;
  const uint16_t* shared_gate_w;  // null, or bf16 [H]: per-token scale sigmoid(gate . x)
};

// the reference's float sigmoid (qwen3_6_moe_int4_model.cpp:29)
static float ref_sigmoid(float x) { return 1.f / (1.f + std::exp(-x)); }

static qlwc::Int4View to_view(const ref_int4_view& v) {
  qlwc::Int4View W;
  W.qweight = v.qweight;
  W.scales = v.scales;
  W.zeros = v.zeros;
  W.scales_f32 = nullptr;
  W.M = v.M;
  W.K = v.K;
  W.group_size = v.group_size;
  W.scheme = v.scheme == 1 ? qlwc::Scheme::kGptqAsym : qlwc::Scheme::kAwqSym;
  W.awq_zp = v.awq_zp > 0 ? v.awq_zp : qlwc::kLocalAwqSymZero;
  return W;
}

__attribute__((visibility("default"))) void ref_gemm_int4(const float* x, const ref_int4_view* W,
                                                          float* y) {
  hal::gemm_int4(x, to_view(*W), y);
}

__attribute__((visibility("default"))) void ref_gemm_int4_argmax(const float* x, const ref_int4_view* W,
                                                                 int32_t* index, float* value) {
  const hal::Int4ArgmaxResult r = hal::gemm_int4_argmax(x, to_view(*W));
  *index = r.index;
  *value = r.value;
}

__attribute__((visibility("default"))) void ref_gemm_int4_batch(const float* X, int n,
                                                                const ref_int4_view* W, float* Y) {
  hal::gemm_int4_batch(X, n, to_view(*W), Y);
}

__attribute__((visibility("default"))) int ref_dequant_int4_row(const ref_int4_view* W, int row,
                                                               float* out) {
  try {
    hal::dequant_int4_row(to_view(*W), row, out);
  } catch (...) {
    return -1;
  }
  return 0;
}

__attribute__((visibility("default"))) void ref_gemm_bias_free(const float* x, const uint16_t* W,
                                                               float* y, int M, int K,
                                                               int w_is_f16) {
  hal::gemm_bias_free(x, W, y, M, K, w_is_f16 ? hal::WDtype::kF16 : hal::WDtype::kBF16,
                      /*allow_gpu=*/false);
}

__attribute__((visibility("default"))) void ref_silu_and_mul(const float* g, const float* u,
                                                             float* out, int n) {
  hal::silu_and_mul(g, u, out, n);
}

__attribute__((visibility("default"))) int ref_max_threads() {
#if defined(_OPENMP)
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// One token of Qwen36MoeInt4Model::moe_ffn_token on the CPU (no offload cache):
// router GEMV, softmax, partial_sort top-k, renormalise
// (src/model/qwen3_6_moe_int4_model.cpp:386-402), then moe_cpu_experts (:184-232:
// OpenMP over the selected experts, thread-local accumulators merged under a
// critical section) and the INT4 shared expert (:352-374).  The sigmoid+bias
// router has no reference counterpart; it is the oracle's specification.
static void moe_token(const ref_layer& L, const float* x, float* down_acc, int* ids_out,
                      float* w_out) {
  const int H = L.H, I = L.I, E = L.E, K = L.topk;
  std::vector<float> logits(static_cast<size_t>(E));
  hal::gemm_bias_free(x, L.router_w, logits.data(), E, H, hal::WDtype::kBF16, false);
  std::vector<int> order(static_cast<size_t>(E));
  std::vector<float> wts(static_cast<size_t>(K));
  if (L.router == 0) {
    float m = *std::max_element(logits.begin(), logits.end());
    double s = 0.0;
    for (int i = 0; i < E; ++i) {
      logits[i] = std::exp(logits[i] - m);
      s += logits[i];
    }
    for (int i = 0; i < E; ++i) logits[i] = static_cast<float>(logits[i] / s);
    std::iota(order.begin(), order.end(), 0);
    std::partial_sort(order.begin(), order.begin() + K, order.end(),
                      [&](int a, int b) { return logits[a] > logits[b]; });
    double wsum = 0.0;
    for (int i = 0; i < K; ++i) wsum += logits[order[i]];
    if (wsum < 1e-12) wsum = 1.0;
    for (int i = 0; i < K; ++i)
      wts[i] = static_cast<float>(logits[static_cast<size_t>(order[i])] / wsum);
  } else {
    std::vector<float> s(static_cast<size_t>(E)), sel(static_cast<size_t>(E));
    for (int e = 0; e < E; ++e) {
      s[e] = static_cast<float>(1.0 / (1.0 + std::exp(-static_cast<double>(logits[e]))));
      sel[e] = s[e] + L.bias[e];
    }
    std::iota(order.begin(), order.end(), 0);
    std::partial_sort(order.begin(), order.begin() + K, order.end(), [&](int a, int b) {
      return sel[a] > sel[b] || (sel[a] == sel[b] && a < b);
    });
    double wsum = 0.0;
    for (int i = 0; i < K; ++i) wsum += s[order[i]];
    if (wsum < 1e-20) wsum = 1.0;
    for (int i = 0; i < K; ++i)
      wts[i] = static_cast<float>(static_cast<double>(s[order[i]]) / wsum) * L.routed_scaling;
  }
  for (int i = 0; i < K; ++i) {
    ids_out[i] = order[i];
    w_out[i] = wts[i];
  }
  std::fill(down_acc, down_acc + H, 0.f);

  auto run_one = [&](const ref_expert& ex, float ww, float* local) {
    std::vector<float> g(static_cast<size_t>(I)), u(static_cast<size_t>(I)),
        mid(static_cast<size_t>(I)), down(static_cast<size_t>(H));
    hal::gemm_int4(x, to_view(ex.gate), g.data());
    hal::gemm_int4(x, to_view(ex.up), u.data());
    hal::silu_and_mul(g.data(), u.data(), mid.data(), I);
    hal::gemm_int4(mid.data(), to_view(ex.down), down.data());
    for (int d = 0; d < H; ++d) local[d] += ww * down[static_cast<size_t>(d)];
  };
#if defined(_OPENMP)
#pragma omp parallel
  {
    std::vector<float> local(static_cast<size_t>(H), 0.f);
#pragma omp for schedule(static)
    for (int i = 0; i < K; ++i) run_one(L.experts[order[i]], wts[i], local.data());
#pragma omp critical
    for (int d = 0; d < H; ++d) down_acc[d] += local[static_cast<size_t>(d)];
  }
#else
  std::vector<float> local(static_cast<size_t>(H), 0.f);
  for (int i = 0; i < K; ++i) run_one(L.experts[order[i]], wts[i], local.data());
  for (int d = 0; d < H; ++d) down_acc[d] += local[static_cast<size_t>(d)];
#endif
  if (L.shared) {
    std::vector<float> g(static_cast<size_t>(I)), u(static_cast<size_t>(I)),
        mid(static_cast<size_t>(I)), down(static_cast<size_t>(H));
    hal::gemm_int4(x, to_view(L.shared->gate), g.data());
    hal::gemm_int4(x, to_view(L.shared->up), u.data());
    hal::silu_and_mul(g.data(), u.data(), mid.data(), I);
    hal::gemm_int4(mid.data(), to_view(L.shared->down), down.data());
    float scale = L.shared_scale;
    if (L.shared_gate_w) {  // qwen3_6_moe_int4_model.cpp:365-371
      float gate_logit = 0.f;
      hal::gemm_bias_free(x, L.shared_gate_w, &gate_logit, 1, H, hal::WDtype::kBF16, false);
      scale = ref_sigmoid(gate_logit);
    }
    for (int d = 0; d < H; ++d) down_acc[d] += scale * down[static_cast<size_t>(d)];
  }
}

// The reference's per-token loop over a batch (qwen3_5_int4_model.cpp:1204-1208
// calls moe_ffn_token once per token).
__attribute__((visibility("default"))) void ref_moe_layer_forward(const ref_layer* L,
                                                                  const float* X, int T, float* Y,
                                                                  int* ids, float* weights) {
  for (int t = 0; t < T; ++t)
    moe_token(*L, X + static_cast<size_t>(t) * L->H, Y + static_cast<size_t>(t) * L->H,
              ids + static_cast<size_t>(t) * L->topk, weights + static_cast<size_t>(t) * L->topk);
}

}  // extern "C"
