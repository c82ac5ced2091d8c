// The CUDA backend inside the reference engine (see cuda_backend.h).  Built
// only against the reference's headers (IE_B200_REFERENCE_HEADERS).
#include "cuda_backend.h"

#ifdef IE_B200_REFERENCE_HEADERS

#include <cuda_runtime.h>

#include <cstring>
#include <thread>
#include <utility>

#include "backends/cpu/cpu_backend.h"
#include "core/runtime/execution_context.h"
#include "core/scheduler/plan.h"
#include "graph_passes.h"
#include "models/traditional/onnx/onnx_loader.h"

namespace ie_b200 {
namespace {

ie::Status cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return {};
  cudaGetLastError();
  if (e == cudaErrorMemoryAllocation) {
    return ie::Error::out_of_memory(std::string(what) + ": " + cudaGetErrorString(e));
  }
  return ie::Error::runtime(std::string(what) + ": " + cudaGetErrorString(e));
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

// ------------------------------------------------------------ CudaBackend

CudaBackend::~CudaBackend() { (void)shutdown(); }

ie::Status CudaBackend::init() {
  if (initialized_) return {};
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return ie::Error::runtime("no CUDA device: the CUDA backend has no CPU fallback");
  }
  if (auto st = cuda_ok(cudaGetDevice(&device_), "cudaGetDevice"); !st.has_value()) return st;
  cudaStream_t s = nullptr;
  if (auto st = cuda_ok(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
      !st.has_value()) {
    return st;
  }
  stream_ = s;
  if (ops_.list().empty()) {
    if (auto st = register_cuda_ops(ops_); !st.has_value()) return st;
  }
  initialized_ = true;
  return {};
}

ie::Status CudaBackend::shutdown() {
  executor_.reset();  // drops the ops and their device weights
  graph_.reset();
  if (stream_ != nullptr) {
    cudaStreamSynchronize(as_stream(stream_));
    cudaStreamDestroy(as_stream(stream_));
    stream_ = nullptr;
  }
  initialized_ = false;
  return {};
}

ie::Result<ie::BufferHandle> CudaBackend::alloc(std::size_t bytes) {
  if (!initialized_) return ie::Error::invalid_argument("cuda backend is not initialized");
  void* p = nullptr;
  if (auto st = cuda_ok(cudaMalloc(&p, bytes == 0 ? 256 : bytes), "cudaMalloc"); !st.has_value()) {
    return st.error();
  }
  return p;
}

void CudaBackend::free(ie::BufferHandle handle) {
  if (handle != nullptr) cudaFree(handle);
}

ie::Status CudaBackend::copy_to_device(ie::BufferHandle dst, const void* src, std::size_t bytes) {
  if (bytes == 0) return {};
  if (dst == nullptr || src == nullptr) return ie::Error::invalid_argument("null copy buffer");
  if (auto st = cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream_)),
                        "cudaMemcpyAsync H2D");
      !st.has_value()) {
    return st;
  }
  return cuda_ok(cudaStreamSynchronize(as_stream(stream_)), "cudaStreamSynchronize");
}

ie::Status CudaBackend::copy_to_host(void* dst, ie::BufferHandle src, std::size_t bytes) {
  if (bytes == 0) return {};
  if (dst == nullptr || src == nullptr) return ie::Error::invalid_argument("null copy buffer");
  if (auto st = cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream_)),
                        "cudaMemcpyAsync D2H");
      !st.has_value()) {
    return st;
  }
  return cuda_ok(cudaStreamSynchronize(as_stream(stream_)), "cudaStreamSynchronize");
}

ie::Status CudaBackend::copy_d2d(ie::BufferHandle dst, ie::BufferHandle src, std::size_t bytes) {
  if (bytes == 0) return {};
  if (dst == nullptr || src == nullptr) return ie::Error::invalid_argument("null copy buffer");
  if (auto st = cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, as_stream(stream_)),
                        "cudaMemcpyAsync D2D");
      !st.has_value()) {
    return st;
  }
  return cuda_ok(cudaStreamSynchronize(as_stream(stream_)), "cudaStreamSynchronize");
}

ie::Status CudaBackend::compile(ie::Graph& graph) {
  auto g = std::make_unique<ie::Graph>(graph);
  ConvBnReluFusionPass pass(true);
  ie::PassContext ctx;
  if (auto st = pass.run(*g, ctx); !st.has_value()) return st;
  folded_ = pass.folded_batch_norms();
  fused_act_ = pass.fused_activations();
  graph_ = std::move(g);
  executor_ = std::make_unique<CudaExecutor>(ops_);
  return {};
}

ie::Status CudaBackend::execute_async(const ie::BatchPlan& /*plan*/, ie::ExecutionContext& context) {
  if (!initialized_) return ie::Error::invalid_argument("cuda backend is not initialized");
  if (!graph_ || !executor_) return ie::Error::invalid_argument("cuda backend has no compiled graph");
  std::shared_ptr<ie::Allocator> host =
      context.allocator ? context.allocator : std::static_pointer_cast<ie::Allocator>(host_alloc_);
  auto out = executor_->run(*graph_, context.inputs, std::move(host), stream_);
  if (!out.has_value()) return out.error();
  context.outputs = std::move(*out);
  return {};
}

ie::Status CudaBackend::wait(ie::Timeout timeout) {
  if (stream_ == nullptr) return {};
  const auto deadline = std::chrono::steady_clock::now() + timeout;
  for (;;) {
    const cudaError_t e = cudaStreamQuery(as_stream(stream_));
    if (e == cudaSuccess) return {};
    if (e != cudaErrorNotReady) return cuda_ok(e, "cudaStreamQuery");
    if (std::chrono::steady_clock::now() >= deadline) {
      return ie::Error::runtime("cuda backend: work still running after the wait timeout");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

bool CudaBackend::is_idle() const {
  return stream_ == nullptr || cudaStreamQuery(as_stream(stream_)) == cudaSuccess;
}

ie::BackendCaps CudaBackend::caps() const {
  ie::BackendCaps c;
  c.supports_async = false;  // execute_async returns with the outputs on the host
  c.supports_deterministic_kernels = true;
  c.supports_batch_invariant = true;  // per-output sums do not depend on the batch
  return c;
}

ie::PluginMeta CudaBackend::meta() const {
  return ie::PluginMeta{"cuda", "0.2.0", "0.1", {"backend", "cuda", "sm_100a"},
                        "B200 backend: tcgen05 implicit-GEMM convolutions, device-resident graphs"};
}

ie::Result<ie::HardwareProfile> CudaBackend::hardware_profile() const {
  cudaDeviceProp prop{};
  if (auto st = cuda_ok(cudaGetDeviceProperties(&prop, device_), "cudaGetDeviceProperties");
      !st.has_value()) {
    return st.error();
  }
  ie::HardwareProfile p;
  p.vendor = "NVIDIA";
  p.device_name = prop.name;
  p.cu.num_cores = prop.multiProcessorCount;
  p.cu.max_threads_per_core = prop.maxThreadsPerMultiProcessor;
  p.cu.shared_memory_per_core = prop.sharedMemPerMultiprocessor;
  p.cu.l2_cache_size = static_cast<std::size_t>(prop.l2CacheSize);
  p.matrix.has_matrix_unit = p.matrix.has_tensor_core = true;
  p.matrix.supports_fp16_mma = p.matrix.supports_bf16_mma = p.matrix.supports_int8_mma = true;
  p.mem.vram_total = prop.totalGlobalMem;
  p.mem.type = "HBM3e";
  p.dma.supports_async_copy = p.dma.supports_bulk_tensor_copy = true;
  p.exec.supports_workgroup_cluster = p.exec.supports_distributed_shared_mem = true;
  p.exec.supports_warp_specialization = p.exec.supports_async_pipeline = true;
  return p;
}

ie::Result<ie::MemoryPolicy> CudaBackend::memory_policy() const { return ie::MemoryPolicy{}; }

ie::Status register_cuda_backend(ie::BackendRegistry& registry) {
  return registry.register_backend(ie::BackendKind::CUDA,
                                   [] { return std::make_unique<CudaBackend>(); });
}

// ---------------------------------------------------------- BackendEngine

BackendEngine::BackendEngine(ie::EngineConfig config)
    : config_(std::move(config)), allocator_(std::make_shared<ie::MallocAllocator>()) {
  if (auto valid = ie::validate(config_); !valid.has_value()) {
    error_ = valid.error();
    return;
  }
  auto& registry = ie::BackendRegistry::instance();
  ie::BackendKind kind = ie::BackendKind::CPU;
  if (config_.gpu_backend == ie::GpuBackend::CUDA) {
    kind = ie::BackendKind::CUDA;
    if (!registry.contains(kind)) (void)register_cuda_backend(registry);
  } else if (config_.gpu_backend == ie::GpuBackend::VULKAN) {
    error_ = ie::Error::unsupported("no Vulkan backend");
    return;
  } else if (!registry.contains(kind)) {
    (void)registry.register_backend(kind, [] { return std::make_unique<ie::CpuBackend>(); });
  }
  auto backend = registry.create(kind);
  if (!backend.has_value()) {
    error_ = backend.error();
    return;
  }
  backend_ = std::move(*backend);
  if (auto st = backend_->init(); !st.has_value()) {
    error_ = st.error();
    backend_.reset();
  }
}

BackendEngine::~BackendEngine() {
  if (backend_) (void)backend_->shutdown();
}

ie::Status BackendEngine::load(const ie::Graph& graph) {
  if (error_.has_value()) return *error_;
  if (!backend_) return ie::Error::invalid_argument("no backend available");
  graph_ = graph;
  if (auto st = backend_->compile(*graph_); !st.has_value()) return st;
  loaded_ = true;
  return {};
}

ie::Result<std::vector<ie::Tensor>> BackendEngine::infer(
    const std::unordered_map<std::string, ie::Tensor>& inputs) {
  if (error_.has_value()) return *error_;
  if (!loaded_ || !graph_.has_value()) return ie::Error::invalid_argument("engine has no loaded graph");
  ie::ExecutionContext context;
  context.allocator = allocator_;
  context.inputs = inputs;
  ie::BatchPlan plan;
  ie::PrefillItem item;
  item.request = 0;
  plan.prefills.push_back(std::move(item));
  for (const auto& kv : inputs) plan.token_budget += static_cast<std::size_t>(kv.second.numel());
  if (auto st = backend_->execute_async(plan, context); !st.has_value()) return st.error();
  if (auto st = backend_->wait(std::chrono::milliseconds(60000)); !st.has_value()) return st.error();
  return std::move(context.outputs);
}

// -------------------------------------------------- CudaTraditionalEngine

ie::Status CudaTraditionalEngine::load_model(const std::string& path, ie::ModelFormat format) {
  if (format != ie::ModelFormat::ONNX) {
    return ie::Error::unsupported("traditional engine only loads ONNX models");
  }
  auto graph = ie::load_onnx_model(path);
  if (!graph.has_value()) return graph.error();
  std::vector<std::string> names;
  for (const ie::Value& v : graph->values) {
    if (v.is_input) names.push_back(v.name);
  }
  ie::EngineConfig config;
  config.gpu_backend = ie::GpuBackend::CUDA;
  auto engine = std::make_unique<BackendEngine>(config);
  if (auto st = engine->load(*graph); !st.has_value()) return st;
  engine_ = std::move(engine);
  input_names_ = std::move(names);
  return {};
}

ie::Result<ie::Tensor> CudaTraditionalEngine::infer(const std::vector<ie::Tensor>& inputs) {
  if (!engine_) return ie::Error::invalid_argument("traditional engine has no loaded model");
  if (inputs.size() != input_names_.size()) {
    return ie::Error::invalid_argument("traditional engine expected " +
                                       std::to_string(input_names_.size()) + " inputs, got " +
                                       std::to_string(inputs.size()));
  }
  std::unordered_map<std::string, ie::Tensor> named;
  for (size_t i = 0; i < inputs.size(); ++i) named.emplace(input_names_[i], inputs[i]);
  auto outputs = engine_->infer(named);
  if (!outputs.has_value()) return outputs.error();
  if (outputs->empty()) return ie::Error::invalid_argument("traditional model produced no outputs");
  return std::move(outputs->front());
}

ie::Result<std::vector<ie::Tensor>> CudaTraditionalEngine::infer_batch(
    const std::vector<std::vector<ie::Tensor>>& batches) {
  std::vector<ie::Tensor> results;
  if (batches.empty()) return results;
  if (!engine_) return ie::Error::invalid_argument("traditional engine has no loaded model");
  const size_t n_in = input_names_.size();
  for (const auto& sample : batches) {
    if (sample.size() != n_in) {
      return ie::Error::invalid_argument("traditional engine expected " + std::to_string(n_in) +
                                         " inputs per sample, got " + std::to_string(sample.size()));
    }
  }
  // stack every input along dimension 0
  auto host = std::make_shared<ie::MallocAllocator>();
  std::vector<int64_t> rows;  // samples' dim-0 sizes of the first input
  std::unordered_map<std::string, ie::Tensor> named;
  for (size_t k = 0; k < n_in; ++k) {
    const ie::Tensor& first = batches[0][k];
    if (first.shape.dims.empty() || first.buffer == nullptr || first.device != ie::Device::CPU) {
      return ie::Error::invalid_argument("batched inputs must be host tensors with a batch dimension");
    }
    int64_t total = 0;
    for (const auto& sample : batches) {
      const ie::Tensor& t = sample[k];
      if (t.dtype != first.dtype || t.shape.dims.size() != first.shape.dims.size() ||
          !std::equal(t.shape.dims.begin() + 1, t.shape.dims.end(), first.shape.dims.begin() + 1) ||
          t.buffer == nullptr || t.device != ie::Device::CPU) {
        return ie::Error::invalid_argument("samples must agree in dtype and in every input shape "
                                           "past the batch dimension");
      }
      total += t.shape.dims[0];
      if (k == 0) rows.push_back(t.shape.dims[0]);
    }
    ie::Shape shape = first.shape;
    shape.dims[0] = total;
    auto stacked = ie::Tensor::allocate(shape, first.dtype, host);
    if (!stacked.has_value()) return stacked.error();
    uint8_t* dst = static_cast<uint8_t*>(stacked->buffer);
    for (const auto& sample : batches) {
      std::memcpy(dst, sample[k].buffer, sample[k].bytes());
      dst += sample[k].bytes();
    }
    named.emplace(input_names_[k], std::move(*stacked));
  }
  auto outputs = engine_->infer(named);
  if (!outputs.has_value()) return outputs.error();
  if (outputs->empty()) return ie::Error::invalid_argument("traditional model produced no outputs");
  const ie::Tensor& y = outputs->front();
  int64_t total_rows = 0;
  for (int64_t r : rows) total_rows += r;
  if (y.shape.dims.empty() || y.shape.dims[0] != total_rows) {
    return ie::Error::unsupported("the model's first output has no batch dimension to split");
  }
  const size_t row_bytes = y.bytes() / static_cast<size_t>(total_rows);
  const uint8_t* src = static_cast<const uint8_t*>(y.buffer);
  for (int64_t r : rows) {
    ie::Shape shape = y.shape;
    shape.dims[0] = r;
    auto part = ie::Tensor::allocate(shape, y.dtype, host);
    if (!part.has_value()) return part.error();
    std::memcpy(part->buffer, src, row_bytes * static_cast<size_t>(r));
    src += row_bytes * static_cast<size_t>(r);
    results.push_back(std::move(*part));
  }
  return results;
}

}  // namespace ie_b200

#endif  // IE_B200_REFERENCE_HEADERS
