// contracts_b200.cpp — see contracts_b200.h.
#include "contracts_b200.h"

#include <algorithm>

namespace llmoc::b200 {

// ------------------------------------------------------------ ICollective

CollectiveB200::~CollectiveB200() { llmoc_collective_destroy(c_); }
int CollectiveB200::world_size() const { return llmoc_collective_world_size(c_); }

void CollectiveB200::allreduce_sum(contracts::TensorView t) {
  const int dt = t.dtype == contracts::DType::kBF16 ? LLMOC_DTYPE_BF16 : LLMOC_DTYPE_F32;
  const llmoc_status s = llmoc_collective_allreduce_sum(c_, t.ptr, t.nbytes(), dt, st_);
  if (s != LLMOC_OK && !err_) err_ = s;
}
void CollectiveB200::alltoall(contracts::TensorView send, contracts::TensorView recv) {
  const llmoc_status s =
      llmoc_collective_alltoall(c_, send.ptr, recv.ptr, send.nbytes() / (size_t)world_size(), st_);
  if (s != LLMOC_OK && !err_) err_ = s;
}
void CollectiveB200::broadcast(contracts::TensorView buf, int root) {
  const llmoc_status s = llmoc_collective_broadcast(c_, buf.ptr, buf.nbytes(), root, st_);
  if (s != LLMOC_OK && !err_) err_ = s;
}

// --------------------------------------------------------- IExpertRuntime

ExpertRuntimeB200::ExpertRuntimeB200(std::vector<const llmoc_moe_layer*> shards, int rank, int world, int device,
                                     size_t expert_bytes, int max_rows, cudaStream_t st)
    : shards_(std::move(shards)), rank_(rank), world_(world), device_(device), expert_bytes_(expert_bytes),
      max_rows_(max_rows), st_(st) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device_);
  for (const llmoc_moe_layer* s : shards_)
    ws_bytes_ = std::max(ws_bytes_, llmoc_moe_ep_owner_workspace_bytes(s, max_rows_));
  if (cudaMalloc(reinterpret_cast<void**>(&ids_), sizeof(int32_t) * std::max(1, max_rows_)) != cudaSuccess ||
      cudaMalloc(&ws_, std::max<size_t>(ws_bytes_, 256)) != cudaSuccess)
    err_ = LLMOC_ERR_NO_MEMORY;
  ids_host_.resize(std::max(1, max_rows_));
  cudaSetDevice(prev);
}

ExpertRuntimeB200::~ExpertRuntimeB200() {
  cudaStreamSynchronize(st_);
  if (ids_) cudaFree(ids_);
  if (ws_) cudaFree(ws_);
}

void ExpertRuntimeB200::prefetch(int, const contracts::ExpertId*, int) {}  // every owned expert is resident

void ExpertRuntimeB200::pin(int layer, const contracts::ExpertId* ids, int n, contracts::BlockHandle* out) {
  const bool ok = layer >= 0 && layer < (int)shards_.size();
  for (int i = 0; i < n; ++i) {
    out[i].id = ids[i];
    const bool mine = ok && ids[i].layer == layer && shards_[layer] && owns(ids[i]);
    out[i].ptr = mine ? const_cast<llmoc_moe_layer*>(shards_[layer]) : nullptr;  // the shard holding it
    out[i].device_ordinal = mine ? device_ : -1;
    out[i].nbytes = mine ? expert_bytes_ : 0;  // a handle of an expert another rank owns is not valid()
  }
}

void ExpertRuntimeB200::gemm_swiglu(const contracts::BlockHandle& h, const contracts::TensorView& x,
                                    contracts::TensorView& y) {
  const int n = static_cast<int>(x.shape[0]);
  if (!h.valid() || !owns(h.id) || h.id.layer < 0 || h.id.layer >= (int)shards_.size() || n < 0 ||
      n > max_rows_ || x.dtype != contracts::DType::kBF16 || y.dtype != contracts::DType::kBF16) {
    if (!err_) err_ = LLMOC_ERR_INVALID;
    return;
  }
  if (n == 0) return;
  std::fill(ids_host_.begin(), ids_host_.begin() + n, h.id.expert / world_);  // owner-local id
  if (cudaMemcpyAsync(ids_, ids_host_.data(), sizeof(int32_t) * n, cudaMemcpyHostToDevice, st_) != cudaSuccess) {
    if (!err_) err_ = LLMOC_ERR_CUDA;
    return;
  }
  const llmoc_status s = llmoc_moe_ep_experts(shards_[h.id.layer], static_cast<const uint16_t*>(x.ptr), ids_, n,
                                              static_cast<uint16_t*>(y.ptr), ws_, ws_bytes_, st_);
  if (s != LLMOC_OK && !err_) err_ = s;
  // ids_host_ is reused by the next call: the copy must have read it
  cudaStreamSynchronize(st_);
}

void ExpertRuntimeB200::release(const contracts::BlockHandle*, int) {}  // nothing was moved

bool ExpertRuntimeB200::owns(contracts::ExpertId id) const { return id.expert % world_ == rank_; }

}  // namespace llmoc::b200

// ---- C entry for the library's tests (the Python tests reach the classes
// through it; a C++ caller uses the classes directly)
extern "C" __attribute__((visibility("default"))) int llmoc_adapter_expert_runtime_run(
    const llmoc_moe_layer* shard, int rank, int world, int device, size_t expert_bytes, int layer_of_shard,
    int expert, const void* x, int n, int hidden, void* y, void* stream, int* owns_out, int* valid_out) {
  using namespace llmoc;
  std::vector<const llmoc_moe_layer*> shards(layer_of_shard + 1, nullptr);
  shards[layer_of_shard] = shard;
  b200::ExpertRuntimeB200 rt(shards, rank, world, device, expert_bytes, std::max(1, n),
                             static_cast<cudaStream_t>(stream));
  contracts::ExpertId id{layer_of_shard, expert};
  *owns_out = rt.owns(id) ? 1 : 0;
  contracts::BlockHandle h;
  rt.prefetch(layer_of_shard, &id, 1);
  rt.pin(layer_of_shard, &id, 1, &h);
  *valid_out = h.valid() ? 1 : 0;
  if (!h.valid()) return 0;  // another rank's expert: nothing to run here
  contracts::TensorView xv, yv;
  xv.ptr = const_cast<void*>(x);
  xv.device_ordinal = device;
  xv.dtype = contracts::DType::kBF16;
  xv.numel = (int64_t)n * hidden;
  xv.rank = 2;
  xv.shape[0] = n;
  xv.shape[1] = hidden;
  yv = xv;
  yv.ptr = y;
  rt.gemm_swiglu(h, xv, yv);
  rt.release(&h, 1);
  return rt.error();
}
