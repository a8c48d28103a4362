// contracts_b200.h — the reference's contracts::ICollective
// (src/contracts/collective.h:9-15) and contracts::IExpertRuntime
// (src/contracts/expert_runtime.h:9-17) implemented on libllmoc_b200.so.
//
// CollectiveB200: the NVLink collectives of one rank (llmoc_collective_*),
// the implementation that src/exec/mesh_nccl.cpp:85-134 leaves as stubs.
//
// ExpertRuntimeB200: the experts of one expert-parallel shard per layer
// (llmoc_moe_layer_create_ep: routed experts e with e % world == rank, owner
// id e / world).  They are resident in HBM, so prefetch, pin and release move
// nothing: pin fills the handles (the shard that holds the expert, its device
// and bytes) and gemm_swiglu runs down(silu(gate x) * up x) for the rows of x
// on one expert through llmoc_moe_ep_experts.  owns(id) is the reference's
// DeviceMesh::owner_rank with EpShard::kMod (src/contracts/device_mesh.h:63-72).
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "contracts/collective.h"
#include "contracts/expert_runtime.h"
#include "llmoc_b200.h"

namespace llmoc::b200 {

class CollectiveB200 final : public contracts::ICollective {
 public:
  // c: a connected llmoc_collective (owned from here on); st: the stream every call is ordered on
  CollectiveB200(llmoc_collective* c, cudaStream_t st) : c_(c), st_(st) {}
  ~CollectiveB200() override;
  int world_size() const override;
  void allreduce_sum(contracts::TensorView inout) override;  // device fp32 or bf16
  void alltoall(contracts::TensorView send, contracts::TensorView recv) override;  // world equal chunks
  void broadcast(contracts::TensorView buf, int root) override;
  // 0, or nonzero when a call failed or a bounded device-side wait gave up
  int error() const { return err_; }

 private:
  llmoc_collective* c_;
  cudaStream_t st_;
  int err_ = 0;
};

class ExpertRuntimeB200 final : public contracts::IExpertRuntime {
 public:
  // shards[l]: this rank's shard of layer l (not owned); expert_bytes: one
  // expert's three projections as stored (llmoc_expert_storage_bytes);
  // max_rows: the most rows one gemm_swiglu call takes
  ExpertRuntimeB200(std::vector<const llmoc_moe_layer*> shards, int rank, int world, int device,
                    size_t expert_bytes, int max_rows, cudaStream_t st);
  ~ExpertRuntimeB200() override;
  void prefetch(int layer, const contracts::ExpertId* ids, int n) override;
  void pin(int layer, const contracts::ExpertId* ids, int n, contracts::BlockHandle* out) override;
  // x, y: device bf16 [n, hidden] (y may not alias x); the expert is h.id
  void gemm_swiglu(const contracts::BlockHandle& h, const contracts::TensorView& x,
                   contracts::TensorView& y) override;
  void release(const contracts::BlockHandle* hs, int n) override;
  bool owns(contracts::ExpertId id) const override;
  // 0, or the llmoc_status / cudaError of the first call that failed
  int error() const { return err_; }

 private:
  std::vector<const llmoc_moe_layer*> shards_;
  int rank_, world_, device_;
  size_t expert_bytes_;
  int max_rows_;
  cudaStream_t st_;
  int32_t* ids_ = nullptr;       // device [max_rows]: the owner-local expert of each row
  std::vector<int32_t> ids_host_;
  void* ws_ = nullptr;           // device workspace of llmoc_moe_ep_experts
  size_t ws_bytes_ = 0;
  int err_ = 0;
};

}  // namespace llmoc::b200
