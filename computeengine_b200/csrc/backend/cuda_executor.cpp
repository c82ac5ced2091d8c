// Device-resident graph execution (see cuda_executor.h).
#include "cuda_executor.h"

#include <cuda_runtime.h>

#include <cstring>
#include <optional>
#include <utility>

#include "ie_cuda_conv.h"

namespace ie_b200 {
namespace {

ie::Status cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return {};
  if (e == cudaErrorMemoryAllocation) {
    return ie::Error::out_of_memory(std::string(what) + ": " + cudaGetErrorString(e));
  }
  return ie::Error::runtime(std::string(what) + ": " + cudaGetErrorString(e));
}

// Flatten (layout_ops.cpp:47-110): [prod(dims[:axis]), prod(dims[axis:])].
ie::Result<ie::Tensor> flatten(const ie::Tensor& x, const ie::Attrs& attrs) {
  int64_t axis = 1;
  auto it = attrs.find("axis");
  if (it != attrs.end()) {
    if (const auto* v = std::get_if<int64_t>(&it->second)) {
      axis = *v;
    } else {
      return ie::Error::invalid_argument("attribute 'axis' must be an int");
    }
  }
  const int64_t rank = static_cast<int64_t>(x.shape.dims.size());
  if (axis < 0) axis += rank;
  if (axis < 0 || axis > rank) return ie::Error::invalid_argument("Flatten axis out of range");
  int64_t outer = 1, inner = 1;
  for (int64_t i = 0; i < rank; ++i) (i < axis ? outer : inner) *= x.shape.dims[static_cast<size_t>(i)];
  ie::Tensor y = x;  // shares the buffer and its owner
  y.shape = ie::Shape{{outer, inner}};
  return y;
}

}  // namespace

CudaDeviceAllocator::~CudaDeviceAllocator() {
  if (pool_ != nullptr) cudaMemPoolDestroy(static_cast<cudaMemPool_t>(pool_));
}

ie::Result<ie::BufferHandle> CudaDeviceAllocator::alloc(std::size_t bytes, ie::MemoryKind) {
  if (pool_ == nullptr) {
    int dev = 0;
    if (auto st = cuda_check(cudaGetDevice(&dev), "cudaGetDevice"); !st.has_value()) {
      cudaGetLastError();
      return st.error();
    }
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (auto st = cuda_check(cudaMemPoolCreate(&pool, &props), "cudaMemPoolCreate"); !st.has_value()) {
      cudaGetLastError();
      return st.error();
    }
    // keep freed memory in the pool across synchronizations
    uint64_t keep = ~uint64_t{0};
    if (auto st = cuda_check(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep),
                             "cudaMemPoolSetAttribute");
        !st.has_value()) {
      cudaGetLastError();
      cudaMemPoolDestroy(pool);
      return st.error();
    }
    pool_ = pool;
  }
  void* p = nullptr;
  if (auto st = cuda_check(cudaMallocFromPoolAsync(&p, bytes == 0 ? 256 : bytes,
                                                   static_cast<cudaMemPool_t>(pool_),
                                                   static_cast<cudaStream_t>(stream_)),
                           "cudaMallocFromPoolAsync");
      !st.has_value()) {
    cudaGetLastError();
    return st.error();
  }
  return p;
}

void CudaDeviceAllocator::free(ie::BufferHandle handle) {
  if (handle != nullptr) cudaFreeAsync(handle, static_cast<cudaStream_t>(stream_));
}

std::size_t CudaDeviceAllocator::reserved_bytes() const {
  if (pool_ == nullptr) return 0;
  uint64_t v = 0;
  if (cudaMemPoolGetAttribute(static_cast<cudaMemPool_t>(pool_), cudaMemPoolAttrReservedMemCurrent, &v) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return static_cast<std::size_t>(v);
}

std::size_t CudaDeviceAllocator::available(ie::MemoryKind) const {
  size_t free_b = 0, total = 0;
  if (cudaMemGetInfo(&free_b, &total) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return free_b;
}

ie::Result<std::vector<ie::Tensor>> CudaExecutor::run(
    const ie::Graph& graph, const std::unordered_map<std::string, ie::Tensor>& inputs,
    std::shared_ptr<ie::Allocator> host_allocator, void* stream) {
  if (!host_allocator) return ie::Error::invalid_argument("executor requires an allocator");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return ie::Error::runtime("no CUDA device: the CUDA executor has no CPU fallback");
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  device_alloc_->set_stream(stream);
  if (graph_ != &graph || ops_.size() != graph.nodes.size()) {
    ops_.clear();
    for (const ie::Node& node : graph.nodes) {
      if (node.op == ie::OpType::Flatten) {
        ops_.push_back(nullptr);
        continue;
      }
      auto op = create_(node.op);
      if (!op.has_value()) {
        return ie::Error::unsupported("no CUDA op for a node of this graph (run the fusion pass first)");
      }
      if (auto s = (*op)->configure(node.attrs); !s.has_value()) return s.error();
      ops_.push_back(std::move(*op));
    }
    graph_ = &graph;
  }
  std::unordered_map<ie::ValueId, ie::Tensor> values;
  // constants stay host tensors: the ops keep device copies per host buffer
  for (const auto& [name, tensor] : graph.weights) {
    const ie::Value* v = nullptr;
    for (const ie::Value& cand : graph.values) {
      if (cand.name == name) v = &cand;
    }
    if (v == nullptr) return ie::Error::invalid_argument("weight has no graph value: " + name);
    if (!v->is_input) values.emplace(v->id, tensor);
  }
  for (const ie::Value& v : graph.values) {
    if (!v.is_input) continue;
    auto it = inputs.find(v.name);
    if (it == inputs.end()) return ie::Error::invalid_argument("missing input: " + v.name);
    const ie::Tensor& t = it->second;
    if (t.buffer == nullptr) return ie::Error::invalid_argument("input has no buffer: " + v.name);
    if (t.device == ie::Device::CUDA) {
      values.emplace(v.id, t);
      continue;
    }
    auto d = ie::Tensor::allocate(t.shape, t.dtype, device_alloc_);
    if (!d.has_value()) return d.error();
    d->device = ie::Device::CUDA;
    if (auto s = cuda_check(cudaMemcpyAsync(d->buffer, t.buffer, t.bytes(), cudaMemcpyHostToDevice, st),
                            "cudaMemcpyAsync H2D");
        !s.has_value()) {
      return s.error();
    }
    values.emplace(v.id, std::move(*d));
  }
  // the last node that reads each value; graph outputs are kept to the end
  std::unordered_map<ie::ValueId, size_t> last_use;
  for (size_t i = 0; i < graph.nodes.size(); ++i) {
    for (ie::ValueId id : graph.nodes[i].inputs) last_use[id] = i;
  }
  for (const ie::Value& v : graph.values) {
    if (v.is_output) last_use[v.id] = graph.nodes.size();
  }
  auto release_after = [&](size_t i, ie::ValueId id) {
    auto it = last_use.find(id);
    if (it == last_use.end() || it->second == i) values.erase(id);
  };
  ie::ExecutionContext ctx;
  ctx.device = ie::Device::CUDA;
  ctx.allocator = device_alloc_;
  ctx.stream = stream;
  for (size_t i = 0; i < graph.nodes.size(); ++i) {
    const ie::Node& node = graph.nodes[i];
    std::vector<ie::Tensor*> in_ptrs;
    for (ie::ValueId id : node.inputs) {
      auto it = values.find(id);
      if (it == values.end()) return ie::Error::invalid_argument("missing node input value");
      in_ptrs.push_back(&it->second);
    }
    if (node.op == ie::OpType::Flatten) {
      if (in_ptrs.size() != 1 || node.outputs.size() != 1) {
        return ie::Error::invalid_argument("Flatten expects one input and one output");
      }
      auto y = flatten(*in_ptrs[0], node.attrs);
      if (!y.has_value()) return y.error();
      values.emplace(node.outputs[0], std::move(*y));
      for (ie::ValueId id : node.inputs) release_after(i, id);
      release_after(i, node.outputs[0]);
      continue;
    }
    std::vector<ie::Tensor> out_storage(node.outputs.size());
    std::vector<ie::Tensor*> out_ptrs;
    for (ie::Tensor& t : out_storage) out_ptrs.push_back(&t);
    if (auto s = ops_[i]->forward(in_ptrs, out_ptrs, ctx); !s.has_value()) return s.error();
    for (size_t k = 0; k < node.outputs.size(); ++k) {
      values.emplace(node.outputs[k], std::move(out_storage[k]));
    }
    // stream-ordered frees: the memory is reused only by work queued later
    for (ie::ValueId id : node.inputs) release_after(i, id);
    for (ie::ValueId id : node.outputs) release_after(i, id);
  }
  std::vector<ie::Tensor> outputs;
  for (const ie::Value& v : graph.values) {
    if (!v.is_output) continue;
    auto it = values.find(v.id);
    if (it == values.end()) return ie::Error::invalid_argument("output value was not produced");
    const ie::Tensor* t = &it->second;
    // an int8 activation in the backend's NHWC layout goes back to NCHW first
    std::optional<ie::Tensor> nchw;
    if (t->layout == ie::Layout::NHWC && t->device == ie::Device::CUDA &&
        (t->dtype == ie::DType::U8 || t->dtype == ie::DType::I8) && t->shape.dims.size() == 4) {
      auto d = ie::Tensor::allocate(t->shape, t->dtype, device_alloc_);
      if (!d.has_value()) return d.error();
      d->device = ie::Device::CUDA;
      const auto& dims = t->shape.dims;
      const int rc = ie_cuda_q8_unpack_output(t->buffer, d->buffer, dims[0], dims[1], dims[2], dims[3],
                                              (dims[1] + 15) / 16 * 16, stream);
      if (rc != IE_OK) return ie::Error::runtime(std::string("unpack int8 output: ") + ie_cuda_last_error());
      nchw = std::move(*d);
      t = &*nchw;
    }
    auto h = ie::Tensor::allocate(t->shape, t->dtype, host_allocator);
    if (!h.has_value()) return h.error();
    const cudaMemcpyKind kind = t->device == ie::Device::CUDA ? cudaMemcpyDeviceToHost
                                                              : cudaMemcpyHostToHost;
    if (auto s = cuda_check(cudaMemcpyAsync(h->buffer, t->buffer, t->bytes(), kind, st), "cudaMemcpyAsync D2H");
        !s.has_value()) {
      return s.error();
    }
    outputs.push_back(std::move(*h));
  }
  if (outputs.empty()) return ie::Error::invalid_argument("graph has no outputs");
  if (auto s = cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize"); !s.has_value()) {
    return s.error();
  }
  uint32_t code = 0;
  if (ie_cuda_take_device_error(&code) != IE_OK || code != 0) {
    return ie::Error::runtime("device-side wait timed out (site 0x" + std::to_string(code) + ")");
  }
  return outputs;
}

}  // namespace ie_b200
