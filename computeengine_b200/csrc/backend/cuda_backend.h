// The CUDA backend of the reference engine (src/core/backend/backend.h:23-52)
// and the engine-level entry points that reach it.
//
//   CudaBackend            ie::Backend on one B200: compile() copies the
//                          graph and runs ConvBnReluFusionPass on it;
//                          execute_async() runs it with CudaExecutor (every
//                          intermediate value in device memory, the CUDA ops
//                          of this backend's own CudaOpTable); alloc / copy
//                          map to cudaMalloc / cudaMemcpy on the backend's
//                          stream.
//   register_cuda_backend  BackendRegistry::register_backend(BackendKind::CUDA,
//                          ...) (backend_registry.h:23-32); AlreadyExists when
//                          CUDA is taken.
//   BackendEngine          the reference Engine's load / infer contract
//                          (core/runtime/engine.h) with the backend chosen by
//                          EngineConfig::gpu_backend: GpuBackend::CUDA takes
//                          the CUDA backend from the BackendRegistry
//                          (registering it when absent), anything else the CPU
//                          backend exactly as ie::Engine does.  The reference
//                          Engine always creates the CPU backend
//                          (engine.cpp:22-27); this is that constructor with
//                          the selection added.
//   CudaTraditionalEngine  TraditionalEngine (engine/traditional/
//                          traditional_engine.h) on the CUDA backend: ONNX
//                          load through the reference loader, infer(), and an
//                          infer_batch() that stacks the samples along the
//                          batch dimension and runs them as one batch instead
//                          of one Engine::infer per sample
//                          (traditional_engine.cpp:79-91).
//
// These types implement interfaces that exist only in the reference tree, so
// this file compiles only with IE_B200_REFERENCE_HEADERS (the reference's src/
// on the include path): dropped into src/backends/cuda/ it builds with the
// engine; the standalone build of this package leaves it out.
#pragma once

#ifdef IE_B200_REFERENCE_HEADERS

#include <chrono>
#include <memory>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "core/backend/backend.h"
#include "core/backend/backend_registry.h"
#include "core/backend/engine_config.h"
#include "core/memory/malloc_allocator.h"
#include "core/config/model_format.h"
#include "cuda_conv_ops.h"
#include "cuda_executor.h"

namespace ie_b200 {

class CudaBackend final : public ie::Backend {
 public:
  CudaBackend() = default;
  ~CudaBackend() override;

  ie::Status init() override;
  ie::Status shutdown() override;
  ie::Device device() const override { return ie::Device::CUDA; }

  ie::Result<ie::BufferHandle> alloc(std::size_t bytes) override;
  void free(ie::BufferHandle handle) override;
  ie::Status copy_to_device(ie::BufferHandle dst, const void* src, std::size_t bytes) override;
  ie::Status copy_to_host(void* dst, ie::BufferHandle src, std::size_t bytes) override;
  ie::Status copy_d2d(ie::BufferHandle dst, ie::BufferHandle src, std::size_t bytes) override;

  // Keeps a copy of the graph with Conv + BatchNorm (+ Add) + Relu chains
  // fused (ConvBnReluFusionPass), so no BatchNorm / Relu node reaches the
  // executor.
  ie::Status compile(ie::Graph& graph) override;
  // Runs the compiled graph on context.inputs (host or device tensors) and
  // leaves host tensors from context.allocator (a MallocAllocator when null)
  // in context.outputs.  The outputs are complete when it returns.
  ie::Status execute_async(const ie::BatchPlan& plan, ie::ExecutionContext& context) override;
  ie::Status wait(ie::Timeout timeout) override;
  bool is_idle() const override;

  ie::BackendCaps caps() const override;
  ie::PluginMeta meta() const override;
  ie::Result<ie::HardwareProfile> hardware_profile() const override;
  ie::Result<ie::MemoryPolicy> memory_policy() const override;

  // Fusions of the last compile() (for tests and logs).
  int folded_batch_norms() const { return folded_; }
  int fused_activations() const { return fused_act_; }

 private:
  bool initialized_ = false;
  int device_ = 0;
  void* stream_ = nullptr;  // cudaStream_t
  CudaOpTable ops_;
  std::unique_ptr<ie::Graph> graph_;
  std::unique_ptr<CudaExecutor> executor_;
  std::shared_ptr<ie::MallocAllocator> host_alloc_ = std::make_shared<ie::MallocAllocator>();
  int folded_ = 0, fused_act_ = 0;
};

ie::Status register_cuda_backend(ie::BackendRegistry& registry = ie::BackendRegistry::instance());

class BackendEngine {
 public:
  explicit BackendEngine(ie::EngineConfig config);
  ~BackendEngine();
  ie::Status load(const ie::Graph& graph);
  ie::Result<std::vector<ie::Tensor>> infer(const std::unordered_map<std::string, ie::Tensor>& inputs);
  ie::Backend* backend() { return backend_.get(); }

 private:
  ie::EngineConfig config_;
  std::optional<ie::Error> error_;
  std::optional<ie::Graph> graph_;
  std::shared_ptr<ie::MallocAllocator> allocator_;
  std::unique_ptr<ie::Backend> backend_;
  bool loaded_ = false;
};

class CudaTraditionalEngine {
 public:
  ie::Status load_model(const std::string& path, ie::ModelFormat format);
  ie::Result<ie::Tensor> infer(const std::vector<ie::Tensor>& inputs);
  // All samples in one batch: every sample must give each input the same
  // shape, which is stacked along dimension 0; the first output is split
  // back along dimension 0 (its size must be the stacked batch).  Results
  // equal per-sample infer() bit for bit (the kernels' sums do not depend on
  // the batch size).
  ie::Result<std::vector<ie::Tensor>> infer_batch(const std::vector<std::vector<ie::Tensor>>& batches);

 private:
  std::unique_ptr<BackendEngine> engine_;
  std::vector<std::string> input_names_;
};

}  // namespace ie_b200

#endif  // IE_B200_REFERENCE_HEADERS
