// Engine-side interface the CUDA convolution ops implement.
//
// By default this header restates the subset of the reference engine's
// interface the ops use, with the same names, members and semantics:
//   Error / Status / Result       src/core/base/error.h:9-80
//   DType, Device, Layout         src/core/base/types.h:8-26
//   Shape                         src/core/base/shape.h:9-16
//   MemoryKind, Allocator         src/core/memory/memory_kind.h, allocator.h:10-22
//   Tensor (+ Tensor::allocate)   src/core/memory/tensor.h:21-103
//   AttrValue / Attrs             src/core/ir/attr.h:12-15
//   ExecutionContext              src/core/runtime/execution_context.h:17-27
//   Op                            src/core/ops/op.h:27-54
//   OpType (the kinds used here)  src/core/ir/op_type.h
//   OpRegistry                    src/core/ops/op_registry.h:15-30, op_registry.cpp:23-50
//   NodeId / ValueId, Value, Node, Edge, Graph (nodes, values, edges,
//     weights, find_value)        src/core/ir/ids.h, graph.h:27-101
//   ModelKind, PassContext, Pass  src/core/ir/model_kind.h, pass.h:14-25
//   PluginMeta                    src/core/plugin/plugin_meta.h:8-14
//   QuantConfig / QuantPlugin     src/core/plugin/quant_plugin.h:11-28
// Built inside the reference tree with IE_B200_REFERENCE_HEADERS defined (and
// the reference's src/ on the include path), it includes the reference's own
// headers instead and the ops compile against the real types unchanged.
#pragma once

#ifdef IE_B200_REFERENCE_HEADERS

#include "core/ir/op_type.h"
#include "core/ops/op.h"
#include "core/ops/op_registry.h"
#include "core/ir/pass.h"
#include "core/plugin/quant_plugin.h"

#else

#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <functional>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <unordered_map>
#include <utility>
#include <variant>
#include <vector>

namespace ie {

struct Error {
  enum class Code { InvalidArgument, Unsupported, NotFound, AlreadyExists, OutOfMemory, Runtime };
  Code code{Code::Runtime};
  std::string message;
  static Error invalid_argument(std::string m) { return {Code::InvalidArgument, std::move(m)}; }
  static Error unsupported(std::string m) { return {Code::Unsupported, std::move(m)}; }
  static Error not_found(std::string m) { return {Code::NotFound, std::move(m)}; }
  static Error already_exists(std::string m) { return {Code::AlreadyExists, std::move(m)}; }
  static Error out_of_memory(std::string m) { return {Code::OutOfMemory, std::move(m)}; }
  static Error runtime(std::string m) { return {Code::Runtime, std::move(m)}; }
};

class Status {
 public:
  Status() = default;
  Status(Error error) : error_(std::move(error)) {}
  bool has_value() const { return !error_.has_value(); }
  explicit operator bool() const { return has_value(); }
  Error& error() { return *error_; }
  const Error& error() const { return *error_; }

 private:
  std::optional<Error> error_;
};

template <class T>
class Result {
 public:
  Result(T value) : value_(std::move(value)) {}
  Result(Error error) : error_(std::move(error)) {}
  bool has_value() const { return value_.has_value(); }
  explicit operator bool() const { return has_value(); }
  T& operator*() { return *value_; }
  const T& operator*() const { return *value_; }
  T* operator->() { return &*value_; }
  const T* operator->() const { return &*value_; }
  T& value() { return *value_; }
  const T& value() const { return *value_; }
  Error& error() { return error_; }
  const Error& error() const { return error_; }

 private:
  std::optional<T> value_;
  Error error_{};
};

enum class Device { CPU, CUDA, VULKAN };
enum class DType { F32, F16, BF16, I8, I4, U8, FP8_E4M3, FP8_E5M2, MXFP4, MXFP6, BOOL };
enum class Layout { ROW_MAJOR, COL_MAJOR, BLOCKED, NHWC, NCHW };

inline std::size_t dtype_size(DType dtype) {
  switch (dtype) {
    case DType::F32: return 4;
    case DType::F16:
    case DType::BF16: return 2;
    case DType::I8:
    case DType::U8:
    case DType::FP8_E4M3:
    case DType::FP8_E5M2:
    case DType::BOOL: return 1;
    default: return 1;  // sub-byte types are not used by these ops
  }
}

struct Shape {
  std::vector<int64_t> dims;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
  }
  bool is_concrete() const {
    for (int64_t d : dims) {
      if (d < 0) return false;
    }
    return true;
  }
};

enum class MemoryKind {
  HOST, DEVICE, PINNED, UNIFIED, MANAGED, GRADIENT, OPTIMIZER_STATE, ACTIVATION, WEIGHT_CONST,
  KV_CACHE,
};

using BufferHandle = void*;

class Allocator {
 public:
  virtual ~Allocator() = default;
  virtual Result<BufferHandle> alloc(std::size_t bytes, MemoryKind kind) = 0;
  virtual void free(BufferHandle handle) = 0;
  virtual std::size_t available(MemoryKind kind) const = 0;
};

class Tensor {
 public:
  Shape shape;
  DType dtype{DType::F32};
  Device device{Device::CPU};
  Layout layout{Layout::ROW_MAJOR};
  BufferHandle buffer{nullptr};

  int64_t numel() const { return shape.numel(); }
  std::size_t bytes() const { return static_cast<std::size_t>(numel()) * dtype_size(dtype); }
  template <class T>
  T* data() { return static_cast<T*>(buffer); }
  template <class T>
  const T* data() const { return static_cast<const T*>(buffer); }

  static Result<Tensor> allocate(const Shape& shape, DType dtype,
                                 std::shared_ptr<Allocator> allocator,
                                 MemoryKind kind = MemoryKind::ACTIVATION) {
    if (!allocator) return Error::invalid_argument("Tensor::allocate requires allocator");
    if (!shape.is_concrete()) {
      return Error::invalid_argument("Tensor::allocate requires concrete shape");
    }
    auto handle = allocator->alloc(static_cast<std::size_t>(shape.numel()) * dtype_size(dtype), kind);
    if (!handle.has_value()) return handle.error();
    Tensor t;
    t.shape = shape;
    t.dtype = dtype;
    t.device = Device::CPU;
    t.layout = Layout::ROW_MAJOR;
    t.buffer = *handle;
    t.owner_ = std::shared_ptr<void>(*handle, [allocator](void* p) { allocator->free(p); });
    return t;
  }

 private:
  std::shared_ptr<void> owner_;
};

using AttrValue = std::variant<int64_t, double, bool, std::string, std::vector<int64_t>,
                               std::vector<double>>;
using Attrs = std::unordered_map<std::string, AttrValue>;

struct ExecutionContext {
  Device device{Device::CPU};
  std::shared_ptr<Allocator> allocator;
  std::unordered_map<std::string, Tensor> inputs;
  std::vector<Tensor> outputs;
  void* stream{nullptr};
};

class Op {
 public:
  virtual ~Op() = default;
  virtual Status configure(const Attrs& /*attrs*/) { return {}; }
  virtual Status forward(const std::vector<Tensor*>& inputs, std::vector<Tensor*>& outputs,
                         ExecutionContext& context) = 0;
};

enum class OpType {
  Add, Relu, Reshape, Conv2D, DepthwiseConv2D, MaxPool2D, AvgPool2D, GlobalAvgPool, BatchNorm,
  Clip, Gemm, Flatten
};

using NodeId = uint32_t;
using ValueId = uint32_t;
inline constexpr ValueId kInvalidValue = 0xFFFFFFFFu;
inline constexpr NodeId kInvalidNode = 0xFFFFFFFFu;

enum class ModelKind { TRADITIONAL, TRANSFORMER, HYBRID, RULE, UNKNOWN };

struct Value {
  ValueId id{kInvalidValue};
  std::string name;
  Shape shape;
  DType dtype{DType::F32};
  bool is_input{false};
  bool is_output{false};
};

struct Node {
  NodeId id{kInvalidNode};
  OpType op{OpType::Add};
  std::vector<ValueId> inputs;
  std::vector<ValueId> outputs;
  Attrs attrs;
  std::optional<Device> placed_device;
  ModelKind kind{ModelKind::UNKNOWN};
};

struct Edge {
  ValueId value{kInvalidValue};
  std::optional<NodeId> from;
  std::optional<NodeId> to;
};

// The slice of the reference Graph a compiler pass over traditional nodes
// uses: nodes in execution order, values, edges and the constant tensors
// keyed by value name.
class Graph {
 public:
  std::vector<Node> nodes;
  std::vector<Value> values;
  std::vector<Edge> edges;
  std::unordered_map<std::string, Tensor> weights;

  const Value* find_value(ValueId id) const {
    for (const Value& v : values) {
      if (v.id == id) return &v;
    }
    return nullptr;
  }
  const Value* find_value(const std::string& name) const {
    for (const Value& v : values) {
      if (v.name == name) return &v;
    }
    return nullptr;
  }
};

struct HardwareProfile {};

struct PassContext {
  HardwareProfile hardware;
  ModelKind model_kind{ModelKind::UNKNOWN};
};

class Pass {
 public:
  virtual ~Pass() = default;
  virtual std::string name() const = 0;
  virtual Status run(Graph& graph, PassContext& context) = 0;
};

// The reference registry is a process singleton with a private constructor;
// here instances can also be made directly, which is what a backend-private
// registry handed to the executor needs.
class OpRegistry {
 public:
  using Creator = std::function<std::unique_ptr<Op>()>;
  OpRegistry() = default;
  static OpRegistry& instance() {
    static OpRegistry registry;
    return registry;
  }
  Status register_op(OpType op, Creator creator) {
    if (!creator) return Error::invalid_argument("empty op creator");
    std::lock_guard<std::mutex> lock(mutex_);
    if (creators_.find(op) != creators_.end()) return Error::already_exists("op already registered");
    creators_.emplace(op, std::move(creator));
    return {};
  }
  Result<std::unique_ptr<Op>> create(OpType op) {
    Creator creator;
    {
      std::lock_guard<std::mutex> lock(mutex_);
      auto it = creators_.find(op);
      if (it == creators_.end()) return Error::not_found("no kernel for op");
      creator = it->second;
    }
    auto instance = creator();
    if (!instance) return Error::runtime("op factory returned null");
    return instance;
  }

 private:
  mutable std::mutex mutex_;
  std::unordered_map<OpType, Creator> creators_;
};

struct PluginMeta {
  std::string name;
  std::string version;
  std::string api_version;
  std::vector<std::string> tags;
  std::string description;
};

struct QuantConfig {
  std::string format;
  int bits{8};
  bool symmetric{true};
};

class QuantPlugin {
 public:
  virtual ~QuantPlugin() = default;
  virtual PluginMeta meta() const = 0;
  virtual Result<Tensor> quantize(const Tensor& tensor, const QuantConfig& config) = 0;
  virtual Result<Tensor> dequantize(const Tensor& tensor, const QuantConfig& config) = 0;
};

// Host allocator (malloc/free), the engine's default for CPU tensors.
class MallocAllocator final : public Allocator {
 public:
  Result<BufferHandle> alloc(std::size_t bytes, MemoryKind) override {
    void* p = std::malloc(bytes == 0 ? 1 : bytes);
    if (p == nullptr) return Error::out_of_memory("malloc failed");
    return p;
  }
  void free(BufferHandle h) override { std::free(h); }
  std::size_t available(MemoryKind) const override { return SIZE_MAX; }
};

}  // namespace ie

#endif  // IE_B200_REFERENCE_HEADERS
