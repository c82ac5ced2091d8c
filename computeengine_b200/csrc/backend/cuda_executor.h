// Graph execution on the GPU with device-resident values: the CUDA
// counterpart of the reference Executor (src/core/runtime/executor.h:19-33,
// executor.cpp:12-109), which runs each node on host tensors.
//
// run() uploads the graph inputs once, runs every node in graph order on one
// CUDA stream with the ops of the given registry (register_cuda_ops) in
// device mode (ExecutionContext::device = CUDA: inputs and outputs stay in
// device memory, no per-node copy or synchronize), and copies the graph
// outputs back into host tensors from `host_allocator`.  Flatten is a
// zero-copy reshape.  One op instance per node is kept across runs of the
// same graph object, so device copies of the weights are uploaded once.
// Nodes without a CUDA op (BatchNorm, a Relu / Add that was not fused, ...)
// return Unsupported: run ConvBnReluFusionPass on the graph first.  A device
// error (a bounded wait that timed out) returns Runtime.
#pragma once

#include <cstddef>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "cuda_conv_ops.h"
#include "ie_op_iface.h"

namespace ie_b200 {

// cudaMalloc / cudaFree behind the engine's Allocator interface
// (src/core/memory/allocator.h:10-22), for device-resident tensors.
class CudaDeviceAllocator final : public ie::Allocator {
 public:
  ie::Result<ie::BufferHandle> alloc(std::size_t bytes, ie::MemoryKind kind) override;
  void free(ie::BufferHandle handle) override;
  std::size_t available(ie::MemoryKind kind) const override;
};

class CudaExecutor {
 public:
  using OpFactory = std::function<ie::Result<std::unique_ptr<ie::Op>>(ie::OpType)>;
  // Ops from a registry with register_cuda_ops applied (the standalone build's
  // registry, or the reference singleton) or from the CUDA backend's own table.
  explicit CudaExecutor(ie::OpRegistry& registry)
      : create_([&registry](ie::OpType t) { return registry.create(t); }) {}
  explicit CudaExecutor(CudaOpTable& table)
      : create_([&table](ie::OpType t) { return table.create(t); }) {}
  ie::Result<std::vector<ie::Tensor>> run(const ie::Graph& graph,
                                          const std::unordered_map<std::string, ie::Tensor>& inputs,
                                          std::shared_ptr<ie::Allocator> host_allocator,
                                          void* stream = nullptr);

 private:
  OpFactory create_;
  std::shared_ptr<CudaDeviceAllocator> device_alloc_ = std::make_shared<CudaDeviceAllocator>();
  const ie::Graph* graph_ = nullptr;
  std::vector<std::unique_ptr<ie::Op>> ops_;  // one per node of graph_
};

}  // namespace ie_b200
