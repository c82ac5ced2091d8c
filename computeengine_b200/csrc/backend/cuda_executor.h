// Graph execution on the GPU with device-resident values: the CUDA
// counterpart of the reference Executor (src/core/runtime/executor.h:19-33,
// executor.cpp:12-109), which runs each node on host tensors.
//
// run() uploads the graph inputs once, runs every node in graph order on one
// CUDA stream with the ops of the given registry (register_cuda_ops) in
// device mode (ExecutionContext::device = CUDA: inputs and outputs stay in
// device memory, no per-node copy or synchronize), and copies the graph
// outputs back into host tensors from `host_allocator`.  Flatten is a
// zero-copy reshape.  Each intermediate value is released right after the
// last node that reads it (stream-ordered, so the next node's output may
// reuse its memory), so a run holds the live set of the graph, not the sum
// of its values.  One op instance per node is kept across runs of the same
// graph object, so device copies of the weights are uploaded once.
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

// Device-resident tensors behind the engine's Allocator interface
// (src/core/memory/allocator.h:10-22): stream-ordered allocations
// (cudaMallocFromPoolAsync / cudaFreeAsync on the executor's stream) from a
// memory pool of its own that keeps freed memory reserved, so after the first
// run of a graph its activations cost no driver allocation at all.  The pool
// is created on the current device at the first allocation and destroyed with
// the allocator (memory still in use is released when its last tensor is).
class CudaDeviceAllocator final : public ie::Allocator {
 public:
  CudaDeviceAllocator() = default;
  CudaDeviceAllocator(const CudaDeviceAllocator&) = delete;
  CudaDeviceAllocator& operator=(const CudaDeviceAllocator&) = delete;
  ~CudaDeviceAllocator() override;
  ie::Result<ie::BufferHandle> alloc(std::size_t bytes, ie::MemoryKind kind) override;
  void free(ie::BufferHandle handle) override;
  std::size_t available(ie::MemoryKind kind) const override;
  // the stream that orders allocations and frees (a cudaStream_t)
  void set_stream(void* stream) { stream_ = stream; }
  // bytes the pool holds from the device (in use + kept for reuse)
  std::size_t reserved_bytes() const;

 private:
  void* pool_ = nullptr;    // cudaMemPool_t
  void* stream_ = nullptr;  // cudaStream_t
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
  // device memory the executor's pool holds (the peak live set of the runs)
  std::size_t reserved_device_bytes() const { return device_alloc_->reserved_bytes(); }

 private:
  OpFactory create_;
  std::shared_ptr<CudaDeviceAllocator> device_alloc_ = std::make_shared<CudaDeviceAllocator>();
  const ie::Graph* graph_ = nullptr;
  std::vector<std::unique_ptr<ie::Op>> ops_;  // one per node of graph_
};

}  // namespace ie_b200
