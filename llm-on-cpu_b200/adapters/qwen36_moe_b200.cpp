// qwen36_moe_b200.cpp — see qwen36_moe_b200.h.
#include "qwen36_moe_b200.h"

#include <cmath>
#include <cstring>

namespace llmoc::model {

namespace {
uint16_t f32_to_bf16(float f) {  // round to nearest even (NaN stays NaN)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
float bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
}  // namespace

Qwen36MoeB200Model::~Qwen36MoeB200Model() {
  for (llmoc_moe_layer* l : dev_)
    if (l) llmoc_moe_layer_destroy(l);
  if (ws_) cudaFree(ws_);
  if (dx_) cudaFree(dx_);
  if (dy_) cudaFree(dy_);
  if (st_) cudaStreamDestroy(st_);
}

bool Qwen36MoeB200Model::init_b200(const std::string& qlwc_path, const std::string& prefix, int device,
                                   int max_tokens) {
  if (!cfg_.is_moe || max_tokens <= 0 || !llmoc_cuda_probe_available()) return false;
  H_ = cfg_.hidden;
  max_tokens_ = max_tokens;
  device_ = device;
  std::vector<int32_t> moe(llmoc_qlwc_moe_layers(qlwc_path.c_str(), prefix.c_str(), nullptr, 0) > 0
                               ? llmoc_qlwc_moe_layers(qlwc_path.c_str(), prefix.c_str(), nullptr, 0)
                               : 0);
  if (moe.empty()) return false;
  llmoc_qlwc_moe_layers(qlwc_path.c_str(), prefix.c_str(), moe.data(), (int)moe.size());
  dev_.assign(cfg_.layers, nullptr);
  for (int32_t l : moe) {
    if (l < 0 || l >= cfg_.layers) return false;
    llmoc_qlwc_layer_info info{};
    if (llmoc_qlwc_describe(qlwc_path.c_str(), prefix.c_str(), l, &info) != LLMOC_OK) return false;
    // the router of qwen3_6_moe_int4_model.cpp:386-402: softmax, top-k, renormalise;
    // the shared expert weighted by its sigmoid gate when the file holds one
    llmoc_moe_layer_desc d{info.hidden, info.inter, info.n_experts, cfg_.topk, info.group_size, info.scheme,
                           qlwc::kLocalAwqSymZero, LLMOC_ROUTER_SOFTMAX, 1.0f, info.has_shared, 1.0f};
    if (llmoc_moe_layer_create_qlwc(qlwc_path.c_str(), prefix.c_str(), l, &d, device, &dev_[l]) != LLMOC_OK)
      return false;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  for (llmoc_moe_layer* l : dev_)
    if (l) ws_bytes_ = std::max(ws_bytes_, llmoc_moe_workspace_bytes(l, max_tokens));
  const size_t rows = (size_t)max_tokens * H_ * sizeof(uint16_t);
  const bool ok = cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaMalloc(&ws_, ws_bytes_) == cudaSuccess &&
                  cudaMalloc(reinterpret_cast<void**>(&dx_), rows) == cudaSuccess &&
                  cudaMalloc(reinterpret_cast<void**>(&dy_), rows) == cudaSuccess;
  cudaSetDevice(prev);
  hx_.resize((size_t)max_tokens * H_);
  hy_.resize((size_t)max_tokens * H_);
  return ok;
}

bool Qwen36MoeB200Model::moe_ffn_rows(int layer, const float* normed, int n_tok, float* down) {
  if (layer < 0 || layer >= (int)dev_.size() || !dev_[layer] || n_tok <= 0 || n_tok > max_tokens_) return false;
  const size_t n = (size_t)n_tok * H_;
  for (size_t i = 0; i < n; ++i) hx_[i] = f32_to_bf16(normed[i]);
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device_);
  bool ok = cudaMemcpyAsync(dx_, hx_.data(), n * 2, cudaMemcpyHostToDevice, st_) == cudaSuccess &&
            llmoc_moe_forward(dev_[layer], dx_, n_tok, dy_, ws_, ws_bytes_, st_) == LLMOC_OK &&
            cudaMemcpyAsync(hy_.data(), dy_, n * 2, cudaMemcpyDeviceToHost, st_) == cudaSuccess &&
            cudaStreamSynchronize(st_) == cudaSuccess;
  cudaSetDevice(prev);
  if (!ok) return false;
  for (size_t i = 0; i < n; ++i) down[i] = bf16_to_f32(hy_[i]);
  return true;
}

void Qwen36MoeB200Model::moe_ffn_token(int layer, const float* normed, float* down_acc) {
  if (!moe_ffn_rows(layer, normed, 1, down_acc)) Qwen36MoeInt4Model::moe_ffn_token(layer, normed, down_acc);
}

}  // namespace llmoc::model
