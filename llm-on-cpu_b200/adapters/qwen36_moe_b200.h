// qwen36_moe_b200.h — the reference's Qwen3.6 MoE INT4 model with its expert
// FFN on the B200 library.
//
// Qwen36MoeInt4Model::moe_ffn_token (src/model/qwen3_6_moe_int4_model.h:41;
// .cpp:377-404) routes one token on the host and runs its experts from the
// slot cache.  This subclass keeps the reference's model code and its call
// site (layer_forward calls moe_ffn_token per token,
// src/model/qwen3_5_int4_model.cpp:1204-1208) and replaces the body: the
// token's normed row goes to the device layer (uploaded once by init_b200),
// which routes, groups and runs the experts and the shared expert, and the
// expert output comes back into down_acc (overwritten, as the reference
// does).  moe_ffn_rows is the batched hook: one device forward for all the
// rows of a prefill chunk, what the loop at qwen3_5_int4_model.cpp:1204-1208
// calls once per layer instead of once per token when it is patched to.
// When the device path cannot run, the reference's own CPU path runs.
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "llmoc_b200.h"
#include "model/qwen3_6_moe_int4_model.h"

namespace llmoc::model {

class Qwen36MoeB200Model : public Qwen36MoeInt4Model {
 public:
  ~Qwen36MoeB200Model() override;
  // After load(): every MoE layer of the QLWC file the model was loaded from
  // (the tensors named as in moe_model.cpp:308-364) into HBM on `device`,
  // repacked; max_tokens bounds moe_ffn_rows.  False leaves the CPU path on.
  bool init_b200(const std::string& qlwc_path, const std::string& prefix, int device, int max_tokens);
  // down[n_tok][H] = MoE(normed[n_tok][H]) on the device (fp32 host rows).
  bool moe_ffn_rows(int layer, const float* normed, int n_tok, float* down);

 protected:
  void moe_ffn_token(int layer, const float* normed, float* down_acc) override;

 private:
  std::vector<llmoc_moe_layer*> dev_;  // per model layer (null: not a MoE layer)
  int H_ = 0, max_tokens_ = 0, device_ = 0;
  cudaStream_t st_ = nullptr;
  void* ws_ = nullptr;
  size_t ws_bytes_ = 0;
  uint16_t *dx_ = nullptr, *dy_ = nullptr;  // device bf16 rows
  std::vector<uint16_t> hx_, hy_;             // host bf16 staging
};

}  // namespace llmoc::model
