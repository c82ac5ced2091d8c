// CUDA convolution ops for the reference engine's Op interface; see
// cuda_conv_ops.h for the contract.
#include "cuda_conv_ops.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <optional>
#include <string>
#include <utility>

namespace ie_b200 {
namespace {

// ------------------------------------------------ attribute readers
// Same names, accepted alternatives and messages as attrs_util.h:31-107.

struct IntListAttr {
  bool found = false;
  std::vector<int64_t> values;
};

ie::Status read_int_list(const ie::Attrs& attrs, const char* key, IntListAttr& out) {
  out = IntListAttr{};
  const auto it = attrs.find(key);
  if (it == attrs.end()) return {};
  const auto* values = std::get_if<std::vector<int64_t>>(&it->second);
  if (values == nullptr) {
    return ie::Error::invalid_argument(std::string("attribute '") + key + "' must be an int list");
  }
  out.found = true;
  out.values = *values;
  return {};
}

ie::Status read_int(const ie::Attrs& attrs, const char* key, bool* found, int64_t* value) {
  *found = false;
  const auto it = attrs.find(key);
  if (it == attrs.end()) return {};
  if (const auto* v = std::get_if<int64_t>(&it->second)) {
    *found = true;
    *value = *v;
    return {};
  }
  if (const auto* v = std::get_if<bool>(&it->second)) {
    *found = true;
    *value = *v ? 1 : 0;
    return {};
  }
  return ie::Error::invalid_argument(std::string("attribute '") + key + "' must be an int");
}

ie::Status read_double(const ie::Attrs& attrs, const char* key, bool* found, double* value) {
  *found = false;
  const auto it = attrs.find(key);
  if (it == attrs.end()) return {};
  if (const auto* v = std::get_if<double>(&it->second)) {
    *found = true;
    *value = *v;
    return {};
  }
  if (const auto* v = std::get_if<int64_t>(&it->second)) {
    *found = true;
    *value = static_cast<double>(*v);
    return {};
  }
  return ie::Error::invalid_argument(std::string("attribute '") + key + "' must be numeric");
}

ie::Status read_double_list(const ie::Attrs& attrs, const char* key, bool* found,
                            std::vector<double>* out) {
  *found = false;
  const auto it = attrs.find(key);
  if (it == attrs.end()) return {};
  if (const auto* v = std::get_if<std::vector<double>>(&it->second)) {
    *found = true;
    *out = *v;
    return {};
  }
  if (const auto* v = std::get_if<std::vector<int64_t>>(&it->second)) {
    *found = true;
    out->assign(v->begin(), v->end());
    return {};
  }
  return ie::Error::invalid_argument(std::string("attribute '") + key + "' must be a float list");
}

ie::Status read_pair(const ie::Attrs& attrs, const char* key, std::array<int64_t, 2>& out) {
  IntListAttr value;
  if (auto st = read_int_list(attrs, key, value); !st.has_value()) return st;
  if (!value.found) return {};
  if (value.values.size() != 2) {
    return ie::Error::invalid_argument(std::string(key) + " must contain 2 values");
  }
  if (value.values[0] <= 0 || value.values[1] <= 0) {
    return ie::Error::invalid_argument(std::string(key) + " values must be positive");
  }
  out = {value.values[0], value.values[1]};
  return {};
}

ie::Status read_pads(const ie::Attrs& attrs, std::array<int64_t, 4>& pads) {
  pads = {0, 0, 0, 0};
  IntListAttr value;
  if (auto st = read_int_list(attrs, "pads", value); !st.has_value()) return st;
  if (!value.found || value.values.empty()) return {};
  if (value.values.size() == 2) {
    pads = {value.values[0], value.values[1], value.values[0], value.values[1]};
  } else if (value.values.size() == 4) {
    pads = {value.values[0], value.values[1], value.values[2], value.values[3]};
  } else {
    return ie::Error::invalid_argument("pads must contain 2 or 4 values");
  }
  for (int64_t p : pads) {
    if (p < 0) return ie::Error::invalid_argument("pads must be non-negative");
  }
  return {};
}

ie::Status read_auto_pad(const ie::Attrs& attrs, AutoPad& out) {
  out = AutoPad::NotSet;
  const auto it = attrs.find("auto_pad");
  if (it == attrs.end()) return {};
  const auto* value = std::get_if<std::string>(&it->second);
  if (value == nullptr) return ie::Error::invalid_argument("attribute 'auto_pad' must be a string");
  if (value->empty() || *value == "NOTSET") return {};
  if (*value == "VALID") {
    out = AutoPad::Valid;
  } else if (*value == "SAME_UPPER") {
    out = AutoPad::SameUpper;
  } else if (*value == "SAME_LOWER") {
    out = AutoPad::SameLower;
  } else {
    return ie::Error::invalid_argument("unsupported auto_pad: " + *value);
  }
  return {};
}

// ------------------------------------------------ forward helpers

ie::Status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return {};
  if (e == cudaErrorMemoryAllocation) {
    return ie::Error::out_of_memory(std::string(what) + ": " + cudaGetErrorString(e));
  }
  return ie::Error::runtime(std::string(what) + ": " + cudaGetErrorString(e));
}

ie::Status require_device() {
  int count = 0;
  const cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();  // clear the sticky "no device" error
    return ie::Error::runtime("no CUDA device: the CUDA convolution ops have no CPU fallback");
  }
  return {};
}

// Validation shared by the fp32 and int8 ops, in the reference's order
// (conv2d_op.cpp:77-123): argument counts, allocator, null tensors, dtypes,
// ranks, kernel_shape; the remaining shape rules run in ie_conv2d_resolve.
ie::Status validate(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                    const ie::ExecutionContext& context, size_t min_in, size_t max_in,
                    const char* name) {
  if (inputs.size() < min_in || inputs.size() > max_in || outputs.size() != 1 ||
      outputs[0] == nullptr) {
    return ie::Error::invalid_argument(std::string(name) +
                                       (max_in == 3 ? " expects two or three inputs and one output"
                                                    : " expects two inputs and one output"));
  }
  if (context.allocator == nullptr) {
    return ie::Error::invalid_argument(std::string(name) + " requires an allocator");
  }
  for (const ie::Tensor* t : inputs) {
    if (t == nullptr || t->buffer == nullptr) return ie::Error::invalid_argument("null tensor or buffer");
  }
  return {};
}

ie::Status check_ranks(const ie::Tensor& x, const ie::Tensor& w, const ConvConfig& cfg,
                       const char* name) {
  if (x.shape.dims.size() != 4 || w.shape.dims.size() != 4) {
    return ie::Error::invalid_argument(std::string(name) + " expects 4D NCHW tensors");
  }
  if (cfg.has_kernel_shape &&
      (cfg.kernel_shape[0] != w.shape.dims[2] || cfg.kernel_shape[1] != w.shape.dims[3])) {
    return ie::Error::invalid_argument("kernel_shape does not match the weight tensor");
  }
  return {};
}

ie_conv2d_desc make_desc(const ConvConfig& cfg, const ie::Tensor& x, const ie::Tensor& w,
                         bool depthwise) {
  ie_conv2d_desc d;
  std::memset(&d, 0, sizeof(d));
  d.n = x.shape.dims[0];
  d.c = x.shape.dims[1];
  d.h = x.shape.dims[2];
  d.w = x.shape.dims[3];
  d.m = w.shape.dims[0];
  d.kh = w.shape.dims[2];
  d.kw = w.shape.dims[3];
  d.stride_h = cfg.strides[0];
  d.stride_w = cfg.strides[1];
  d.dil_h = cfg.dilations[0];
  d.dil_w = cfg.dilations[1];
  d.pad_top = cfg.pads[0];
  d.pad_left = cfg.pads[1];
  d.pad_bottom = cfg.pads[2];
  d.pad_right = cfg.pads[3];
  d.group = cfg.group;
  d.auto_pad = cfg.auto_pad == AutoPad::Valid       ? IE_PAD_VALID
               : cfg.auto_pad == AutoPad::SameUpper ? IE_PAD_SAME_UPPER
               : cfg.auto_pad == AutoPad::SameLower ? IE_PAD_SAME_LOWER
                                                    : IE_PAD_NOTSET;
  d.depthwise = depthwise ? 1 : 0;
  // The C ABI's weight-channel check reads C/group from the desc; a weight
  // tensor whose dim 1 differs is rejected here with the reference's message.
  return d;
}

// Host or device source -> device pointer (uploads host data into `slot`).
ie::Result<const void*> to_device(DeviceBuffers& dev, int slot, const ie::Tensor& t,
                                  cudaStream_t st) {
  if (t.device == ie::Device::CUDA) return static_cast<const void*>(t.buffer);
  auto buf = dev.scratch(slot, t.bytes());
  if (!buf.has_value()) return buf.error();
  if (auto s = cuda_status(cudaMemcpyAsync(*buf, t.buffer, t.bytes(), cudaMemcpyHostToDevice, st),
                           "cudaMemcpyAsync H2D");
      !s.has_value()) {
    return s.error();
  }
  return static_cast<const void*>(*buf);
}

ie::Status finish(cudaStream_t st) {
  if (auto s = cuda_status(cudaStreamSynchronize(st), "cudaStreamSynchronize"); !s.has_value()) {
    return s;
  }
  uint32_t code = 0;
  if (ie_cuda_take_device_error(&code) != IE_OK || code != 0) {
    return ie::Error::runtime("device-side wait timed out (site 0x" + std::to_string(code) + ")");
  }
  return {};
}

// True when the caller keeps values in device memory (CudaExecutor): the
// context's allocator hands out device memory, outputs stay there and the
// op returns without synchronizing (the executor does, once per run).
bool device_mode(const ie::ExecutionContext& context) {
  return context.device == ie::Device::CUDA;
}

// outputs[0] from a device result: copied to a host tensor (and the stream
// synchronized) normally, or to a device tensor from the context's allocator
// in device mode.
ie::Status deliver(const void* ydev, ie::Shape shape, ie::DType dtype,
                   ie::ExecutionContext& context, std::vector<ie::Tensor*>& outputs,
                   cudaStream_t st) {
  auto out = ie::Tensor::allocate(shape, dtype, context.allocator);
  if (!out.has_value()) return out.error();
  const bool dev = device_mode(context);
  if (auto e = cuda_status(cudaMemcpyAsync(out->buffer, ydev, out->bytes(),
                                           dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st),
                           "cudaMemcpyAsync");
      !e.has_value()) {
    return e;
  }
  if (dev) {
    out->device = ie::Device::CUDA;
  } else if (auto e = finish(st); !e.has_value()) {
    return e;
  }
  *outputs[0] = std::move(*out);
  return {};
}

enum Slot { kSlotX = 0, kSlotXPacked, kSlotY, kSlotYPacked, kSlotWork, kSlotResidual, kSlotWPacked };
enum CacheKind { kCacheW = 0, kCacheWPacked, kCacheBias, kCacheMult, kCacheBiasI32 };

}  // namespace

// ------------------------------------------------ public helpers

ie::Status parse_conv_config(const ie::Attrs& attrs, ConvConfig& config) {
  config = ConvConfig{};
  if (auto st = read_pair(attrs, "strides", config.strides); !st.has_value()) return st;
  if (auto st = read_pair(attrs, "dilations", config.dilations); !st.has_value()) return st;
  if (auto st = read_pads(attrs, config.pads); !st.has_value()) return st;
  bool found = false;
  int64_t group = 0;
  if (auto st = read_int(attrs, "group", &found, &group); !st.has_value()) return st;
  if (found) {
    if (group <= 0) return ie::Error::invalid_argument("group must be positive");
    config.group = group;
  }
  if (auto st = read_auto_pad(attrs, config.auto_pad); !st.has_value()) return st;
  IntListAttr kernel;
  if (auto st = read_int_list(attrs, "kernel_shape", kernel); !st.has_value()) return st;
  if (kernel.found) {
    if (kernel.values.size() != 2) return ie::Error::invalid_argument("kernel_shape must contain 2 values");
    if (kernel.values[0] <= 0 || kernel.values[1] <= 0) {
      return ie::Error::invalid_argument("kernel_shape values must be positive");
    }
    config.has_kernel_shape = true;
    config.kernel_shape = {kernel.values[0], kernel.values[1]};
  }
  return {};
}

ie::Status to_status(int rc) {
  if (rc == IE_OK) return {};
  const char* msg = ie_cuda_last_error();
  std::string m = msg != nullptr ? msg : "";
  switch (rc) {
    case IE_INVALID_ARGUMENT: return ie::Error::invalid_argument(m);
    case IE_UNSUPPORTED: return ie::Error::unsupported(m);
    case IE_NOT_FOUND: return ie::Error::not_found(m);
    case IE_ALREADY_EXISTS: return ie::Error::already_exists(m);
    case IE_OUT_OF_MEMORY: return ie::Error::out_of_memory(m);
    default: return ie::Error::runtime(m);
  }
}

namespace {
int cuda_malloc_default(void** p, size_t bytes) { return static_cast<int>(cudaMalloc(p, bytes)); }
DeviceAllocFn g_device_alloc = cuda_malloc_default;
}  // namespace

void set_device_alloc(DeviceAllocFn fn) { g_device_alloc = fn != nullptr ? fn : cuda_malloc_default; }

DeviceBuffers::~DeviceBuffers() {
  for (auto& kv : scratch_) cudaFree(kv.second.ptr);
  for (auto& kv : cache_) cudaFree(kv.second.ptr);
}

ie::Result<void*> DeviceBuffers::scratch(int slot, size_t bytes) {
  Block& b = scratch_[slot];
  if (b.bytes < bytes || b.ptr == nullptr) {
    if (b.ptr != nullptr) cudaFree(b.ptr);
    b = Block{};
    void* p = nullptr;
    if (auto s = cuda_status(static_cast<cudaError_t>(g_device_alloc(&p, bytes == 0 ? 256 : bytes)), "cudaMalloc");
        !s.has_value()) {
      return s.error();
    }
    b.ptr = p;
    b.bytes = bytes;
  }
  return b.ptr;
}

ie::Result<void*> DeviceBuffers::cached(const void* host_key, size_t bytes, int kind, bool* fresh) {
  const Key k{host_key, bytes, kind};
  auto it = cache_.find(k);
  if (it != cache_.end()) {
    *fresh = false;
    return it->second.ptr;
  }
  void* p = nullptr;
  if (auto s = cuda_status(static_cast<cudaError_t>(g_device_alloc(&p, bytes == 0 ? 256 : bytes)), "cudaMalloc"); !s.has_value()) {
    return s.error();
  }
  cache_[k] = Block{p, bytes};
  *fresh = true;
  return p;
}

// ------------------------------------------------ fp32 Conv2D / DepthwiseConv2D

ie::Status CudaConv2DOp::configure(const ie::Attrs& attrs) {
  if (auto st = parse_conv_config(attrs, config_); !st.has_value()) return st;
  // "fused_add": an Add node fused by ConvBnReluFusionPass; the residual is
  // the fourth input
  bool found = false;
  int64_t fa = 0;
  if (auto st = read_int(attrs, "fused_add", &found, &fa); !st.has_value()) return st;
  fused_add_ = found && fa != 0;
  // "activation": a Relu / Clip(0, 6) node fused by ConvBnReluFusionPass
  act_ = IE_ACT_NONE;
  auto it = attrs.find("activation");
  if (it != attrs.end()) {
    const auto* v = std::get_if<std::string>(&it->second);
    if (v == nullptr) return ie::Error::invalid_argument("attribute 'activation' must be a string");
    if (*v == "Relu") {
      act_ = IE_ACT_RELU;
    } else if (*v == "Relu6") {
      act_ = IE_ACT_RELU6;
    } else if (!v->empty()) {
      return ie::Error::invalid_argument("attribute 'activation' must be Relu or Relu6");
    }
  }
  return {};
}

ie::Status CudaConv2DOp::forward(const std::vector<ie::Tensor*>& inputs,
                                 std::vector<ie::Tensor*>& outputs,
                                 ie::ExecutionContext& context) {
  const char* name = depthwise_ ? "DepthwiseConv2D" : "Conv2D";
  if (fused_add_) {
    if (inputs.size() != 4) {
      return ie::Error::invalid_argument("Conv2D with a fused add expects x, w, b and the residual");
    }
  } else if (auto st = validate(inputs, outputs, context, 2, 3, "Conv2D"); !st.has_value()) {
    return st;
  }
  if (fused_add_) {
    std::vector<ie::Tensor*> three(inputs.begin(), inputs.begin() + 3);
    if (auto st = validate(three, outputs, context, 2, 3, "Conv2D"); !st.has_value()) return st;
    if (inputs[3] == nullptr || inputs[3]->buffer == nullptr) {
      return ie::Error::invalid_argument("null tensor or buffer");
    }
  }
  for (const ie::Tensor* t : inputs) {
    if (t->dtype != ie::DType::F32) return ie::Error::unsupported("P0 kernels support F32 only");
  }
  const ie::Tensor& x = *inputs[0];
  const ie::Tensor& w = *inputs[1];
  const ie::Tensor* b = inputs.size() >= 3 ? inputs[2] : nullptr;
  const ie::Tensor* res = fused_add_ ? inputs[3] : nullptr;
  if (auto st = check_ranks(x, w, config_, "Conv2D"); !st.has_value()) return st;
  ie_conv2d_desc d = make_desc(config_, x, w, depthwise_);
  if (d.group > 0 && d.c % d.group == 0 && w.shape.dims[1] != d.c / d.group) {
    return ie::Error::invalid_argument("Conv2D weight channels do not match C/group");
  }
  int64_t bias_len = -1;
  if (b != nullptr) {
    if (b->shape.dims.size() != 1) return ie::Error::invalid_argument("Conv2D bias must have shape [M]");
    bias_len = b->shape.dims[0];
  }
  ie_conv2d_shape s;
  if (auto st = to_status(ie_conv2d_resolve(&d, bias_len, &s)); !st.has_value()) return st;
  (void)name;
  if (res != nullptr) {
    if (d.group != 1) return ie::Error::unsupported("a fused add needs a dense convolution");
    const std::vector<int64_t> want{d.n, d.m, s.out_h, s.out_w};
    if (res->shape.dims != want) {
      return ie::Error::invalid_argument("the fused add's residual must have the output's shape");
    }
  }
  if (auto st = require_device(); !st.has_value()) return st;

  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  auto xd = to_device(dev_, kSlotX, x, st);
  if (!xd.has_value()) return xd.error();
  // host weights (and bias) stay on the device for the op's lifetime, keyed
  // by the host buffer; the dense path also keeps them in packed bf16 hi/lo
  // form.  Device-resident weights may be runtime values at an address that
  // is reused with new contents, so they are read (and packed) every call.
  const bool dense = d.group == 1;
  const void* wdev = nullptr;
  if (w.device == ie::Device::CUDA && !dense) {
    wdev = w.buffer;
  } else if (w.device == ie::Device::CUDA) {
    auto slot = dev_.scratch(kSlotWPacked, ie_cuda_f32_packed_weight_bytes(&d));
    if (!slot.has_value()) return slot.error();
    if (auto e = to_status(ie_cuda_f32_pack_weights(&d, static_cast<const float*>(w.buffer), *slot, st));
        !e.has_value()) {
      return e;
    }
    wdev = *slot;
  } else {
    bool fresh = false;
    const size_t bytes = dense ? ie_cuda_f32_packed_weight_bytes(&d) : w.bytes();
    auto slot = dev_.cached(w.buffer, bytes, dense ? kCacheWPacked : kCacheW, &fresh);
    if (!slot.has_value()) return slot.error();
    if (fresh) {
      const void* wsrc = w.buffer;
      if (w.device != ie::Device::CUDA) {
        auto tmp = dev_.scratch(kSlotWork, w.bytes());
        if (!tmp.has_value()) return tmp.error();
        if (auto e = cuda_status(cudaMemcpyAsync(dense ? *tmp : *slot, w.buffer, w.bytes(),
                                                 cudaMemcpyHostToDevice, st),
                                 "cudaMemcpyAsync H2D");
            !e.has_value()) {
          return e;
        }
        wsrc = dense ? *tmp : *slot;
      }
      if (dense) {
        if (auto e = to_status(ie_cuda_f32_pack_weights(&d, static_cast<const float*>(wsrc), *slot, st));
            !e.has_value()) {
          return e;
        }
      }
    }
    wdev = *slot;
  }
  const float* bdev = nullptr;
  if (b != nullptr) {
    if (b->device == ie::Device::CUDA) {
      bdev = b->data<float>();
    } else {
      bool fresh = false;
      auto slot = dev_.cached(b->buffer, b->bytes(), kCacheBias, &fresh);
      if (!slot.has_value()) return slot.error();
      if (fresh) {
        if (auto e = cuda_status(cudaMemcpyAsync(*slot, b->buffer, b->bytes(), cudaMemcpyHostToDevice, st),
                                 "cudaMemcpyAsync H2D");
            !e.has_value()) {
          return e;
        }
      }
      bdev = static_cast<const float*>(*slot);
    }
  }
  const size_t y_bytes = static_cast<size_t>(d.n * d.m * s.out_h * s.out_w) * sizeof(float);
  const ie::Shape y_shape{{d.n, d.m, s.out_h, s.out_w}};
  std::optional<ie::Tensor> dev_out;  // device mode: the result is written in place
  if (device_mode(context)) {
    auto t = ie::Tensor::allocate(y_shape, ie::DType::F32, context.allocator);
    if (!t.has_value()) return t.error();
    t->device = ie::Device::CUDA;
    dev_out = std::move(*t);
  }
  auto ydev = dev_out ? ie::Result<void*>(dev_out->buffer) : dev_.scratch(kSlotY, y_bytes);
  if (!ydev.has_value()) return ydev.error();
  int rc;
  if (dense) {
    // activations split into bf16 hi/lo NHWC planes, then the bf16x3
    // tensor-core GEMM writes NCHW fp32 directly
    const int64_t c_store = (d.c + 15) / 16 * 16;
    auto xs = dev_.scratch(kSlotXPacked, static_cast<size_t>(d.n * d.h * d.w * c_store) * 4);
    if (!xs.has_value()) return xs.error();
    rc = ie_cuda_f32_pack_input(static_cast<const float*>(*xd), *xs, d.n, d.c, d.h, d.w, c_store, st);
    if (rc == IE_OK) {
      const float* rdev = nullptr;
      if (res != nullptr) {
        auto r = to_device(dev_, kSlotResidual, *res, st);
        if (!r.has_value()) return r.error();
        rdev = static_cast<const float*>(*r);
      }
      rc = ie_cuda_conv2d_bf16x3_residual(&d, act_, *xs, wdev, bdev, rdev, *ydev, IE_Y_F32_NCHW, st);
    }
  } else {
    rc = ie_cuda_conv2d_f32(&d, act_, static_cast<const float*>(*xd),
                            static_cast<const float*>(wdev), bdev, static_cast<float*>(*ydev),
                            nullptr, 0, st);
  }
  if (auto e = to_status(rc); !e.has_value()) return e;

  if (dev_out) {
    *outputs[0] = std::move(*dev_out);
    return {};
  }
  return deliver(*ydev, y_shape, ie::DType::F32, context, outputs, st);
}

// ------------------------------------------------ int8 QLinearConv2D

ie::Status CudaQLinearConv2DOp::configure(const ie::Attrs& attrs) {
  if (auto st = parse_conv_config(attrs, config_); !st.has_value()) return st;
  bool found = false;
  std::vector<double> mult;
  if (auto st = read_double_list(attrs, "multiplier", &found, &mult); !st.has_value()) return st;
  if (!found || mult.empty()) {
    return ie::Error::invalid_argument("attribute 'multiplier' must be a float list");
  }
  mult_.assign(mult.size(), 0.0f);
  for (size_t i = 0; i < mult.size(); ++i) {
    if (!std::isfinite(mult[i])) return ie::Error::invalid_argument("multiplier must be finite");
    mult_[i] = static_cast<float>(mult[i]);
  }
  IntListAttr bias;
  if (auto st = read_int_list(attrs, "bias", bias); !st.has_value()) return st;
  bias_.clear();
  for (int64_t v : bias.values) {
    if (v < INT32_MIN || v > INT32_MAX) return ie::Error::invalid_argument("bias values must fit int32");
    bias_.push_back(static_cast<int32_t>(v));
  }
  int64_t v = 0;
  if (auto st = read_int(attrs, "x_zero_point", &found, &v); !st.has_value()) return st;
  zp_x_ = found ? v : 0;
  if (auto st = read_int(attrs, "y_zero_point", &found, &v); !st.has_value()) return st;
  zp_y_ = found ? v : 0;
  if (auto st = read_int(attrs, "y_signed", &found, &v); !st.has_value()) return st;
  y_signed_ = found && v != 0;
  if (auto st = read_int(attrs, "qmin", &has_qmin_, &qmin_); !st.has_value()) return st;
  if (auto st = read_int(attrs, "qmax", &has_qmax_, &qmax_); !st.has_value()) return st;
  return {};
}

ie::Status CudaQLinearConv2DOp::forward(const std::vector<ie::Tensor*>& inputs,
                                        std::vector<ie::Tensor*>& outputs,
                                        ie::ExecutionContext& context) {
  if (auto st = validate(inputs, outputs, context, 2, 2, "QLinearConv2D"); !st.has_value()) return st;
  const ie::Tensor& x = *inputs[0];
  const ie::Tensor& w = *inputs[1];
  if ((x.dtype != ie::DType::U8 && x.dtype != ie::DType::I8) || w.dtype != ie::DType::I8) {
    return ie::Error::unsupported("QLinearConv2D takes U8/I8 activations and I8 weights");
  }
  if (auto st = check_ranks(x, w, config_, "QLinearConv2D"); !st.has_value()) return st;
  const bool depthwise = config_.group > 1;
  ie_conv2d_desc d = make_desc(config_, x, w, depthwise);
  if (d.group > 0 && d.c % d.group == 0 && w.shape.dims[1] != d.c / d.group) {
    return ie::Error::invalid_argument("Conv2D weight channels do not match C/group");
  }
  ie_conv2d_shape s;
  const int64_t bias_len = bias_.empty() ? -1 : static_cast<int64_t>(bias_.size());
  if (auto st = to_status(ie_conv2d_resolve(&d, bias_len, &s)); !st.has_value()) return st;
  if (static_cast<int64_t>(mult_.size()) != d.m) {
    return ie::Error::invalid_argument("multiplier must have M values");
  }
  ie_q8_params q;
  q.x_signed = x.dtype == ie::DType::I8 ? 1 : 0;
  q.zp_x = static_cast<int32_t>(zp_x_);
  q.y_signed = y_signed_ ? 1 : 0;
  q.zp_y = static_cast<int32_t>(zp_y_);
  q.qmin = has_qmin_ ? static_cast<int32_t>(qmin_) : (y_signed_ ? -128 : 0);
  q.qmax = has_qmax_ ? static_cast<int32_t>(qmax_) : (y_signed_ ? 127 : 255);
  const bool dev_mode = device_mode(context);
  // x in the int8 activation layout (a previous int8 node's device output)
  const bool x_nhwc = x.layout == ie::Layout::NHWC;
  if (x_nhwc && x.device != ie::Device::CUDA) {
    return ie::Error::invalid_argument("an NHWC int8 activation must be a device tensor");
  }
  const bool padded = (s.pad_top | s.pad_left | s.pad_bottom | s.pad_right) != 0;
  uint32_t xor_mask = 0;
  bool halo = false;
  if (!depthwise) {
    if (d.group != 1) return ie::Error::unsupported("grouped int8 convolution (1 < group < C)");
    if (q.zp_x != 0) {
      // uint8 with zero point 128 is int8 with zero point 0 after flipping
      // the top bit (while packing NCHW input); any other zero point, and
      // every zero point of an NHWC input, reads a haloed input whose padding
      // holds the zero point (the kernel folds -zp_x * sum(w) into the bias)
      if (!x_nhwc && q.x_signed == 0 && q.zp_x == 128) {
        xor_mask = 0x80;
        q.zp_x = 0;
        q.x_signed = 1;
      } else {
        halo = padded;
      }
    }
  } else if (!(d.group == d.c && d.c == d.m && w.shape.dims[1] == 1)) {
    return ie::Error::unsupported("grouped int8 convolution (1 < group < C)");
  }
  if (auto st = require_device(); !st.has_value()) return st;
  // A ResNet stem (7x7 / 2, pad 3, at most 4 channels, even extent) over an
  // NCHW input with zero point 0 after the re-basing above runs as its
  // space-to-depth equivalent: a 4x1 stride-1 layer over 64 stored channels
  // (ie_cuda_q8_stem_*), bit-identical to the direct 7x7 / 2 convolution.
  ie_conv2d_desc stem_d;
  const bool stem = !depthwise && !x_nhwc && !halo && q.zp_x == 0 && d.kh == 7 && d.kw == 7 &&
                    d.stride_h == 2 && d.stride_w == 2 && d.dil_h == 1 && d.dil_w == 1 &&
                    s.pad_top == 3 && s.pad_left == 3 && s.pad_bottom == 3 && s.pad_right == 3 &&
                    d.c <= 4 && d.h % 2 == 0 && d.w % 2 == 0 &&
                    ie_cuda_q8_stem_desc(d.n, d.c, d.h, d.w, d.m, &stem_d) == IE_OK;
  const ie_conv2d_desc& kd = stem ? stem_d : d;  // the layer the kernel runs

  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  const int64_t c_store = (d.c + 15) / 16 * 16, m_store = (d.m + 15) / 16 * 16;
  const void* xin = nullptr;  // the kernel's input: NHWC, haloed when `halo`
  if (x_nhwc) {
    if (halo) {
      auto xh = dev_.scratch(kSlotXPacked, ie_cuda_q8_halo_input_bytes(&d));
      if (!xh.has_value()) return xh.error();
      if (auto e = to_status(ie_cuda_q8_halo_nhwc(&d, x.buffer, *xh, q.zp_x, st)); !e.has_value()) {
        return e;
      }
      xin = *xh;
    } else {
      xin = x.buffer;
    }
  } else {
    auto xd = to_device(dev_, kSlotX, x, st);
    if (!xd.has_value()) return xd.error();
    const size_t xn_bytes = halo ? ie_cuda_q8_halo_input_bytes(&d)
                            : stem ? static_cast<size_t>(kd.n * kd.h * kd.w * kd.c)
                                   : static_cast<size_t>(d.n * d.h * d.w * c_store);
    auto xn = dev_.scratch(kSlotXPacked, xn_bytes);
    if (!xn.has_value()) return xn.error();
    const int prc = halo   ? ie_cuda_q8_pack_input_halo(&d, *xd, *xn, q.zp_x, st)
                    : stem ? ie_cuda_q8_stem_pack_input(*xd, *xn, d.n, d.c, d.h, d.w, xor_mask, st)
                           : ie_cuda_q8_pack_input(*xd, *xn, d.n, d.c, d.h, d.w, c_store, xor_mask, st);
    if (auto e = to_status(prc); !e.has_value()) return e;
    xin = *xn;
  }
  // packed weights, bias and multipliers: uploaded once per host buffer;
  // device-resident weights (possibly runtime values) are packed every call
  bool fresh = true;
  const size_t wbytes = depthwise ? ie_cuda_dw_q8_packed_weight_bytes(&d)
                                  : ie_cuda_q8_packed_weight_bytes(&kd);
  auto wp = w.device == ie::Device::CUDA ? dev_.scratch(kSlotWPacked, wbytes)
                                         : dev_.cached(w.buffer, wbytes, kCacheWPacked, &fresh);
  if (!wp.has_value()) return wp.error();
  if (fresh) {
    const void* wsrc = w.buffer;
    if (w.device != ie::Device::CUDA) {
      auto tmp = dev_.scratch(kSlotWork, w.bytes());
      if (!tmp.has_value()) return tmp.error();
      if (auto e = cuda_status(cudaMemcpyAsync(*tmp, w.buffer, w.bytes(), cudaMemcpyHostToDevice, st),
                               "cudaMemcpyAsync H2D");
          !e.has_value()) {
        return e;
      }
      wsrc = *tmp;
    }
    const int8_t* w8 = static_cast<const int8_t*>(wsrc);
    const int rc = depthwise ? ie_cuda_dw_q8_pack_weights(&d, w8, *wp, st)
                   : stem    ? ie_cuda_q8_stem_pack_weights(w8, *wp, d.m, d.c, st)
                             : ie_cuda_q8_pack_weights(&d, w8, *wp, st);
    if (auto e = to_status(rc); !e.has_value()) return e;
  }
  auto md = dev_.cached(mult_.data(), mult_.size() * sizeof(float), kCacheMult, &fresh);
  if (!md.has_value()) return md.error();
  if (fresh) {
    if (auto e = cuda_status(cudaMemcpyAsync(*md, mult_.data(), mult_.size() * sizeof(float),
                                             cudaMemcpyHostToDevice, st),
                             "cudaMemcpyAsync H2D");
        !e.has_value()) {
      return e;
    }
  }
  const int32_t* bd = nullptr;
  if (!bias_.empty()) {
    auto bp = dev_.cached(bias_.data(), bias_.size() * sizeof(int32_t), kCacheBiasI32, &fresh);
    if (!bp.has_value()) return bp.error();
    if (fresh) {
      if (auto e = cuda_status(cudaMemcpyAsync(*bp, bias_.data(), bias_.size() * sizeof(int32_t),
                                               cudaMemcpyHostToDevice, st),
                               "cudaMemcpyAsync H2D");
          !e.has_value()) {
        return e;
      }
    }
    bd = static_cast<const int32_t*>(*bp);
  }
  const ie::DType y_dtype = y_signed_ ? ie::DType::I8 : ie::DType::U8;
  const ie::Shape y_shape{{d.n, d.m, s.out_h, s.out_w}};
  std::optional<ie::Tensor> dev_out;  // device mode: written in the activation layout
  void* yn = nullptr;
  if (dev_mode) {
    auto t = ie::Tensor::allocate(ie::Shape{{d.n, s.out_h, s.out_w, m_store}}, y_dtype,
                                  context.allocator);
    if (!t.has_value()) return t.error();
    t->shape = y_shape;
    t->layout = ie::Layout::NHWC;
    t->device = ie::Device::CUDA;
    yn = t->buffer;
    dev_out = std::move(*t);
  } else {
    auto ys = dev_.scratch(kSlotYPacked, static_cast<size_t>(d.n * s.out_h * s.out_w * m_store));
    if (!ys.has_value()) return ys.error();
    yn = *ys;
  }
  const int rc = depthwise
                     ? ie_cuda_dwconv2d_q8(&d, &q, xin, *wp, bd, static_cast<const float*>(*md), yn, st)
                     : ie_cuda_conv2d_q8(&kd, &q, xin, *wp, bd, static_cast<const float*>(*md), yn, st);
  if (auto e = to_status(rc); !e.has_value()) return e;
  if (dev_out) {
    *outputs[0] = std::move(*dev_out);
    return {};
  }
  const size_t y_bytes = static_cast<size_t>(d.n * d.m * s.out_h * s.out_w);
  auto yd = dev_.scratch(kSlotY, y_bytes);
  if (!yd.has_value()) return yd.error();
  if (auto e = to_status(ie_cuda_q8_unpack_output(yn, *yd, d.n, d.m, s.out_h, s.out_w, m_store, st));
      !e.has_value()) {
    return e;
  }
  auto out = ie::Tensor::allocate(y_shape, y_dtype, context.allocator);
  if (!out.has_value()) return out.error();
  if (auto e = cuda_status(cudaMemcpyAsync(out->buffer, *yd, y_bytes, cudaMemcpyDeviceToHost, st),
                           "cudaMemcpyAsync D2H");
      !e.has_value()) {
    return e;
  }
  if (auto e = finish(st); !e.has_value()) return e;
  *outputs[0] = std::move(*out);
  return {};
}

// ------------------------------------------------ int8 Add

ie::Status CudaQLinearAddOp::configure(const ie::Attrs& attrs) {
  bool found_a = false, found_b = false;
  std::vector<double> ma, mb;
  if (auto st = read_double_list(attrs, "a_multiplier", &found_a, &ma); !st.has_value()) return st;
  if (auto st = read_double_list(attrs, "b_multiplier", &found_b, &mb); !st.has_value()) return st;
  if (!found_a && !found_b) {
    return ie::Error::unsupported(
        "Add of fp32 tensors runs fused into a convolution (ConvBnReluFusionPass) on this backend");
  }
  if (!found_a || !found_b || ma.size() != 1 || mb.size() != 1 || !std::isfinite(ma[0]) ||
      !std::isfinite(mb[0])) {
    return ie::Error::invalid_argument("int8 Add needs one finite a_multiplier and b_multiplier");
  }
  q_ = ie_qadd_params{};
  q_.mult_a = static_cast<float>(ma[0]);
  q_.mult_b = static_cast<float>(mb[0]);
  bool found = false;
  int64_t v = 0;
  if (auto st = read_int(attrs, "a_zero_point", &found, &v); !st.has_value()) return st;
  q_.zp_a = found ? static_cast<int32_t>(v) : 0;
  if (auto st = read_int(attrs, "b_zero_point", &found, &v); !st.has_value()) return st;
  q_.zp_b = found ? static_cast<int32_t>(v) : 0;
  if (auto st = read_int(attrs, "y_zero_point", &found, &v); !st.has_value()) return st;
  q_.zp_y = found ? static_cast<int32_t>(v) : 0;
  if (auto st = read_int(attrs, "y_signed", &found, &v); !st.has_value()) return st;
  q_.y_signed = found && v != 0 ? 1 : 0;
  if (auto st = read_int(attrs, "qmin", &has_qmin_, &qmin_); !st.has_value()) return st;
  if (auto st = read_int(attrs, "qmax", &has_qmax_, &qmax_); !st.has_value()) return st;
  return {};
}

ie::Status CudaQLinearAddOp::forward(const std::vector<ie::Tensor*>& inputs,
                                     std::vector<ie::Tensor*>& outputs,
                                     ie::ExecutionContext& context) {
  if (inputs.size() != 2 || outputs.size() != 1 || outputs[0] == nullptr) {
    return ie::Error::invalid_argument("Add expects two inputs and one output");
  }
  if (context.allocator == nullptr) return ie::Error::invalid_argument("Add requires an allocator");
  for (const ie::Tensor* t : inputs) {
    if (t == nullptr || t->buffer == nullptr) return ie::Error::invalid_argument("null tensor or buffer");
    if (t->dtype != ie::DType::U8 && t->dtype != ie::DType::I8) {
      return ie::Error::unsupported("int8 Add takes U8/I8 tensors");
    }
  }
  const ie::Tensor& a = *inputs[0];
  const ie::Tensor& b = *inputs[1];
  if (a.shape.dims != b.shape.dims) return ie::Error::invalid_argument("Add operands differ in shape");
  ie_qadd_params q = q_;
  q.a_signed = a.dtype == ie::DType::I8 ? 1 : 0;
  q.b_signed = b.dtype == ie::DType::I8 ? 1 : 0;
  q.qmin = has_qmin_ ? static_cast<int32_t>(qmin_) : (q.y_signed ? -128 : 0);
  q.qmax = has_qmax_ ? static_cast<int32_t>(qmax_) : (q.y_signed ? 127 : 255);
  const bool a_nhwc = a.layout == ie::Layout::NHWC, b_nhwc = b.layout == ie::Layout::NHWC;
  const bool nhwc = a_nhwc || b_nhwc;
  if ((a_nhwc && a.device != ie::Device::CUDA) || (b_nhwc && b.device != ie::Device::CUDA)) {
    return ie::Error::invalid_argument("an NHWC int8 activation must be a device tensor");
  }
  if (nhwc && a.shape.dims.size() != 4) {
    return ie::Error::invalid_argument("the int8 activation layout is 4-D");
  }
  if (auto st = require_device(); !st.has_value()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  // operands in one layout: an NCHW operand meets an NHWC one after packing
  int64_t count = a.numel();
  int64_t n = 0, c = 0, h = 0, w = 0, c_store = 0;
  if (nhwc) {
    n = a.shape.dims[0];
    c = a.shape.dims[1];
    h = a.shape.dims[2];
    w = a.shape.dims[3];
    c_store = (c + 15) / 16 * 16;
    count = n * h * w * c_store;
  }
  auto operand = [&](const ie::Tensor& t, bool t_nhwc, int slot) -> ie::Result<const void*> {
    if (t_nhwc || !nhwc) return to_device(dev_, slot, t, st);
    auto td = to_device(dev_, slot, t, st);
    if (!td.has_value()) return td.error();
    auto packed = dev_.scratch(slot == kSlotX ? kSlotXPacked : kSlotWork, static_cast<size_t>(count));
    if (!packed.has_value()) return packed.error();
    if (auto e = to_status(ie_cuda_q8_pack_input(*td, *packed, n, c, h, w, c_store, 0, st));
        !e.has_value()) {
      return e.error();
    }
    return static_cast<const void*>(*packed);
  };
  auto ad = operand(a, a_nhwc, kSlotX);
  if (!ad.has_value()) return ad.error();
  auto bd = operand(b, b_nhwc, kSlotResidual);
  if (!bd.has_value()) return bd.error();
  const ie::DType y_dtype = q.y_signed ? ie::DType::I8 : ie::DType::U8;
  if (device_mode(context)) {
    auto t = nhwc ? ie::Tensor::allocate(ie::Shape{{n, h, w, c_store}}, y_dtype, context.allocator)
                  : ie::Tensor::allocate(a.shape, y_dtype, context.allocator);
    if (!t.has_value()) return t.error();
    t->shape = a.shape;
    t->layout = nhwc ? ie::Layout::NHWC : ie::Layout::ROW_MAJOR;
    t->device = ie::Device::CUDA;
    if (auto e = to_status(ie_cuda_qadd(&q, *ad, *bd, t->buffer, count, st)); !e.has_value()) return e;
    *outputs[0] = std::move(*t);
    return {};
  }
  auto yd = dev_.scratch(kSlotY, static_cast<size_t>(count));
  if (!yd.has_value()) return yd.error();
  if (auto e = to_status(ie_cuda_qadd(&q, *ad, *bd, *yd, count, st)); !e.has_value()) return e;
  const void* ysrc = *yd;
  if (nhwc) {  // host mode returns NCHW
    auto yc = dev_.scratch(kSlotYPacked, static_cast<size_t>(a.numel()));
    if (!yc.has_value()) return yc.error();
    if (auto e = to_status(ie_cuda_q8_unpack_output(*yd, *yc, n, c, h, w, c_store, st)); !e.has_value()) {
      return e;
    }
    ysrc = *yc;
  }
  return deliver(ysrc, a.shape, y_dtype, context, outputs, st);
}

// ------------------------------------------------ Conv2D node dispatch

ie::Status CudaConvNodeOp::configure(const ie::Attrs& attrs) {
  if (attrs.count("multiplier") != 0) {
    impl_ = std::make_unique<CudaQLinearConv2DOp>();
  } else {
    impl_ = std::make_unique<CudaConv2DOp>(depthwise_);
  }
  return impl_->configure(attrs);
}

ie::Status CudaConvNodeOp::forward(const std::vector<ie::Tensor*>& inputs,
                                   std::vector<ie::Tensor*>& outputs, ie::ExecutionContext& context) {
  if (!impl_) return ie::Error::invalid_argument("Conv2D used before configure()");
  return impl_->forward(inputs, outputs, context);
}

// ------------------------------------------------ pooling and Gemm

namespace {

// Host NCHW F32 out of a device buffer: allocate outputs[0] and copy back.
ie::Status download_f32(const void* ydev, ie::Shape shape, ie::ExecutionContext& context,
                        std::vector<ie::Tensor*>& outputs, cudaStream_t st) {
  return deliver(ydev, std::move(shape), ie::DType::F32, context, outputs, st);
}

// Device copy of a constant input (weights, bias), uploaded once per host buffer.
ie::Result<const void*> cached_const(DeviceBuffers& dev, const ie::Tensor& t, int kind,
                                     cudaStream_t st) {
  if (t.device == ie::Device::CUDA) return static_cast<const void*>(t.buffer);
  bool fresh = false;
  auto slot = dev.cached(t.buffer, t.bytes(), kind, &fresh);
  if (!slot.has_value()) return slot.error();
  if (fresh) {
    if (auto e = cuda_status(cudaMemcpyAsync(*slot, t.buffer, t.bytes(), cudaMemcpyHostToDevice, st),
                             "cudaMemcpyAsync H2D");
        !e.has_value()) {
      return e.error();
    }
  }
  return static_cast<const void*>(*slot);
}

ie::Status validate_unary(const std::vector<ie::Tensor*>& inputs,
                          std::vector<ie::Tensor*>& outputs, const ie::ExecutionContext& context,
                          const char* name) {
  if (inputs.size() != 1 || outputs.size() != 1 || outputs[0] == nullptr) {
    return ie::Error::invalid_argument(std::string(name) + " expects one input and one output");
  }
  if (context.allocator == nullptr) {
    return ie::Error::invalid_argument(std::string(name) + " requires an allocator");
  }
  if (inputs[0] == nullptr || inputs[0]->buffer == nullptr) {
    return ie::Error::invalid_argument("null tensor or buffer");
  }
  if (inputs[0]->dtype != ie::DType::F32) return ie::Error::unsupported("P0 kernels support F32 only");
  const auto& dims = inputs[0]->shape.dims;
  if (dims.size() != 4) return ie::Error::invalid_argument(std::string(name) + " expects 4D NCHW tensors");
  for (int64_t v : dims) {
    if (v <= 0) return ie::Error::invalid_argument(std::string(name) + " expects positive dimensions");
  }
  return {};
}

}  // namespace

ie::Status parse_pool_config(const ie::Attrs& attrs, PoolConfig& config) {
  config = PoolConfig{};
  IntListAttr kernel;
  if (auto st = read_int_list(attrs, "kernel_shape", kernel); !st.has_value()) return st;
  if (!kernel.found || kernel.values.empty()) return ie::Error::invalid_argument("kernel_shape is required");
  if (kernel.values.size() != 2) return ie::Error::invalid_argument("kernel_shape must contain 2 values");
  if (kernel.values[0] <= 0 || kernel.values[1] <= 0) {
    return ie::Error::invalid_argument("kernel_shape values must be positive");
  }
  config.has_kernel_shape = true;
  config.kernel_shape = {kernel.values[0], kernel.values[1]};
  if (auto st = read_pair(attrs, "strides", config.strides); !st.has_value()) return st;
  if (auto st = read_pads(attrs, config.pads); !st.has_value()) return st;
  if (auto st = read_auto_pad(attrs, config.auto_pad); !st.has_value()) return st;
  bool found = false;
  int64_t v = 0;
  if (auto st = read_int(attrs, "ceil_mode", &found, &v); !st.has_value()) return st;
  config.ceil_mode = found && v != 0;
  if (auto st = read_int(attrs, "count_include_pad", &found, &v); !st.has_value()) return st;
  config.count_include_pad = found && v != 0;
  return {};
}

ie::Status CudaPool2DOp::configure(const ie::Attrs& attrs) { return parse_pool_config(attrs, config_); }

ie::Status CudaPool2DOp::forward(const std::vector<ie::Tensor*>& inputs,
                                 std::vector<ie::Tensor*>& outputs,
                                 ie::ExecutionContext& context) {
  const bool q8 = inputs.size() == 1 && inputs[0] != nullptr &&
                  (inputs[0]->dtype == ie::DType::U8 || inputs[0]->dtype == ie::DType::I8);
  if (q8) return forward_q8(*inputs[0], outputs, context);
  if (auto st = validate_unary(inputs, outputs, context, "Pooling"); !st.has_value()) return st;
  if (!config_.has_kernel_shape) return ie::Error::invalid_argument("kernel_shape is required");
  const ie::Tensor& x = *inputs[0];
  const ie_pool2d_desc d = pool_desc(x);
  ie_conv2d_shape s;
  if (auto st = to_status(ie_pool2d_resolve(&d, &s)); !st.has_value()) return st;
  if (auto st = require_device(); !st.has_value()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  auto xd = to_device(dev_, kSlotX, x, st);
  if (!xd.has_value()) return xd.error();
  auto ydev = dev_.scratch(kSlotY, static_cast<size_t>(d.n * d.c * s.out_h * s.out_w) * sizeof(float));
  if (!ydev.has_value()) return ydev.error();
  if (auto e = to_status(ie_cuda_pool2d_f32(&d, max_pool_ ? 1 : 0, static_cast<const float*>(*xd),
                                            static_cast<float*>(*ydev), st));
      !e.has_value()) {
    return e;
  }
  return download_f32(*ydev, ie::Shape{{d.n, d.c, s.out_h, s.out_w}}, context, outputs, st);
}

ie_pool2d_desc CudaPool2DOp::pool_desc(const ie::Tensor& x) const {
  ie_pool2d_desc d;
  std::memset(&d, 0, sizeof(d));
  d.n = x.shape.dims[0];
  d.c = x.shape.dims[1];
  d.h = x.shape.dims[2];
  d.w = x.shape.dims[3];
  d.kh = config_.kernel_shape[0];
  d.kw = config_.kernel_shape[1];
  d.stride_h = config_.strides[0];
  d.stride_w = config_.strides[1];
  d.pad_top = config_.pads[0];
  d.pad_left = config_.pads[1];
  d.pad_bottom = config_.pads[2];
  d.pad_right = config_.pads[3];
  d.auto_pad = config_.auto_pad == AutoPad::Valid       ? IE_PAD_VALID
               : config_.auto_pad == AutoPad::SameUpper ? IE_PAD_SAME_UPPER
               : config_.auto_pad == AutoPad::SameLower ? IE_PAD_SAME_LOWER
                                                        : IE_PAD_NOTSET;
  d.ceil_mode = config_.ceil_mode ? 1 : 0;
  d.count_include_pad = config_.count_include_pad ? 1 : 0;
  return d;
}

// MaxPool2D of an int8 activation: NCHW (host or device) or the int8
// activation layout (device).  Device mode returns the activation layout
// without synchronizing, like CudaQLinearConv2DOp; host mode returns NCHW.
ie::Status CudaPool2DOp::forward_q8(const ie::Tensor& x, std::vector<ie::Tensor*>& outputs,
                                    ie::ExecutionContext& context) {
  if (outputs.size() != 1 || outputs[0] == nullptr) {
    return ie::Error::invalid_argument("Pooling expects one input and one output");
  }
  if (context.allocator == nullptr) return ie::Error::invalid_argument("Pooling requires an allocator");
  if (x.buffer == nullptr) return ie::Error::invalid_argument("null tensor or buffer");
  if (!max_pool_) {
    return ie::Error::unsupported("average pooling of int8 activations has no requantize rule");
  }
  if (x.shape.dims.size() != 4) return ie::Error::invalid_argument("Pooling expects 4D NCHW tensors");
  for (int64_t v : x.shape.dims) {
    if (v <= 0) return ie::Error::invalid_argument("Pooling expects positive dimensions");
  }
  if (!config_.has_kernel_shape) return ie::Error::invalid_argument("kernel_shape is required");
  const bool x_nhwc = x.layout == ie::Layout::NHWC;
  if (x_nhwc && x.device != ie::Device::CUDA) {
    return ie::Error::invalid_argument("an NHWC int8 activation must be a device tensor");
  }
  const ie_pool2d_desc d = pool_desc(x);
  ie_conv2d_shape s;
  if (auto st = to_status(ie_pool2d_resolve(&d, &s)); !st.has_value()) return st;
  if (auto st = require_device(); !st.has_value()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  const int32_t is_signed = x.dtype == ie::DType::I8 ? 1 : 0;
  const int64_t c_store = (d.c + 15) / 16 * 16;
  auto xd = to_device(dev_, kSlotX, x, st);
  if (!xd.has_value()) return xd.error();
  const void* xn = *xd;
  if (!x_nhwc) {
    auto packed = dev_.scratch(kSlotXPacked, static_cast<size_t>(d.n * d.h * d.w * c_store));
    if (!packed.has_value()) return packed.error();
    if (auto e = to_status(ie_cuda_q8_pack_input(*xd, *packed, d.n, d.c, d.h, d.w, c_store, 0, st));
        !e.has_value()) {
      return e;
    }
    xn = *packed;
  }
  const ie::Shape logical{{d.n, d.c, s.out_h, s.out_w}};
  const size_t y_bytes = static_cast<size_t>(d.n * s.out_h * s.out_w * c_store);
  if (device_mode(context)) {
    auto t = ie::Tensor::allocate(ie::Shape{{d.n, s.out_h, s.out_w, c_store}}, x.dtype,
                                  context.allocator);
    if (!t.has_value()) return t.error();
    t->shape = logical;
    t->layout = ie::Layout::NHWC;
    t->device = ie::Device::CUDA;
    if (auto e = to_status(ie_cuda_q8_maxpool2d_nhwc(&d, is_signed, xn, t->buffer, st)); !e.has_value()) {
      return e;
    }
    *outputs[0] = std::move(*t);
    return {};
  }
  auto yd = dev_.scratch(kSlotY, y_bytes);
  if (!yd.has_value()) return yd.error();
  if (auto e = to_status(ie_cuda_q8_maxpool2d_nhwc(&d, is_signed, xn, *yd, st)); !e.has_value()) return e;
  auto yc = dev_.scratch(kSlotYPacked, static_cast<size_t>(d.n * d.c * s.out_h * s.out_w));
  if (!yc.has_value()) return yc.error();
  if (auto e = to_status(ie_cuda_q8_unpack_output(*yd, *yc, d.n, d.c, s.out_h, s.out_w, c_store, st));
      !e.has_value()) {
    return e;
  }
  return deliver(*yc, logical, x.dtype, context, outputs, st);
}

ie::Status CudaGlobalAvgPoolOp::configure(const ie::Attrs& attrs) {
  has_scale_ = false;
  x_scale_ = 0.0;
  x_zero_point_ = 0;
  if (auto st = read_double(attrs, "x_scale", &has_scale_, &x_scale_); !st.has_value()) return st;
  if (has_scale_ && !(x_scale_ > 0.0 && std::isfinite(x_scale_))) {
    return ie::Error::invalid_argument("GlobalAvgPool x_scale must be positive and finite");
  }
  bool found = false;
  if (auto st = read_int(attrs, "x_zero_point", &found, &x_zero_point_); !st.has_value()) return st;
  if (found && (x_zero_point_ < -128 || x_zero_point_ > 255)) {
    return ie::Error::invalid_argument("GlobalAvgPool x_zero_point out of the 8-bit range");
  }
  return {};
}

ie::Status CudaGlobalAvgPoolOp::forward_q8(const ie::Tensor& x, std::vector<ie::Tensor*>& outputs,
                                          ie::ExecutionContext& context) {
  if (outputs.size() != 1 || outputs[0] == nullptr) {
    return ie::Error::invalid_argument("GlobalAvgPool expects one input and one output");
  }
  if (context.allocator == nullptr) return ie::Error::invalid_argument("GlobalAvgPool requires an allocator");
  if (x.buffer == nullptr) return ie::Error::invalid_argument("null tensor or buffer");
  if (!has_scale_) {
    return ie::Error::invalid_argument("GlobalAvgPool of an int8 activation needs \"x_scale\"");
  }
  const bool is_signed = x.dtype == ie::DType::I8;
  if ((is_signed && x_zero_point_ > 127) || (!is_signed && x_zero_point_ < 0)) {
    return ie::Error::invalid_argument("GlobalAvgPool x_zero_point outside the input's storage type");
  }
  const auto& dm = x.shape.dims;
  if (dm.size() != 4) return ie::Error::invalid_argument("GlobalAvgPool expects 4D NCHW tensors");
  for (int64_t v : dm) {
    if (v <= 0) return ie::Error::invalid_argument("GlobalAvgPool expects positive dimensions");
  }
  const bool x_nhwc = x.layout == ie::Layout::NHWC;
  if (x_nhwc && x.device != ie::Device::CUDA) {
    return ie::Error::invalid_argument("an NHWC int8 activation must be a device tensor");
  }
  if (auto st = require_device(); !st.has_value()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  const int64_t n = dm[0], c = dm[1], h = dm[2], w = dm[3];
  const int64_t c_store = (c + 15) / 16 * 16;
  auto xd = to_device(dev_, kSlotX, x, st);
  if (!xd.has_value()) return xd.error();
  const void* xn = *xd;
  if (!x_nhwc) {
    auto packed = dev_.scratch(kSlotXPacked, static_cast<size_t>(n * h * w * c_store));
    if (!packed.has_value()) return packed.error();
    if (auto e = to_status(ie_cuda_q8_pack_input(*xd, *packed, n, c, h, w, c_store, 0, st));
        !e.has_value()) {
      return e;
    }
    xn = *packed;
  }
  auto ydev = dev_.scratch(kSlotY, static_cast<size_t>(n * c) * sizeof(float));
  if (!ydev.has_value()) return ydev.error();
  if (auto e = to_status(ie_cuda_q8_global_avg_pool_nhwc(xn, static_cast<float*>(*ydev), n, c, h, w,
                                                         is_signed ? 1 : 0,
                                                         static_cast<int32_t>(x_zero_point_),
                                                         x_scale_, st));
      !e.has_value()) {
    return e;
  }
  return download_f32(*ydev, ie::Shape{{n, c, 1, 1}}, context, outputs, st);
}

ie::Status CudaGlobalAvgPoolOp::forward(const std::vector<ie::Tensor*>& inputs,
                                        std::vector<ie::Tensor*>& outputs,
                                        ie::ExecutionContext& context) {
  if (inputs.size() == 1 && inputs[0] != nullptr &&
      (inputs[0]->dtype == ie::DType::U8 || inputs[0]->dtype == ie::DType::I8)) {
    return forward_q8(*inputs[0], outputs, context);
  }
  if (auto st = validate_unary(inputs, outputs, context, "GlobalAvgPool"); !st.has_value()) return st;
  if (auto st = require_device(); !st.has_value()) return st;
  const ie::Tensor& x = *inputs[0];
  const auto& dm = x.shape.dims;
  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  auto xd = to_device(dev_, kSlotX, x, st);
  if (!xd.has_value()) return xd.error();
  auto ydev = dev_.scratch(kSlotY, static_cast<size_t>(dm[0] * dm[1]) * sizeof(float));
  if (!ydev.has_value()) return ydev.error();
  if (auto e = to_status(ie_cuda_global_avg_pool_f32(static_cast<const float*>(*xd),
                                                     static_cast<float*>(*ydev), dm[0], dm[1],
                                                     dm[2], dm[3], st));
      !e.has_value()) {
    return e;
  }
  return download_f32(*ydev, ie::Shape{{dm[0], dm[1], 1, 1}}, context, outputs, st);
}

ie::Status CudaGemmOp::configure(const ie::Attrs& attrs) {
  alpha_ = beta_ = 1.0;
  trans_a_ = trans_b_ = 0;
  bool found = false;
  double d = 0.0;
  if (auto st = read_double(attrs, "alpha", &found, &d); !st.has_value()) return st;
  if (found) alpha_ = d;
  if (auto st = read_double(attrs, "beta", &found, &d); !st.has_value()) return st;
  if (found) beta_ = d;
  int64_t v = 0;
  if (auto st = read_int(attrs, "transA", &found, &v); !st.has_value()) return st;
  if (found) {
    if (v != 0 && v != 1) return ie::Error::invalid_argument("Gemm transA must be 0 or 1");
    trans_a_ = v;
  }
  if (auto st = read_int(attrs, "transB", &found, &v); !st.has_value()) return st;
  if (found) {
    if (v != 0 && v != 1) return ie::Error::invalid_argument("Gemm transB must be 0 or 1");
    trans_b_ = v;
  }
  return {};
}

ie::Status CudaGemmOp::forward(const std::vector<ie::Tensor*>& inputs,
                               std::vector<ie::Tensor*>& outputs, ie::ExecutionContext& context) {
  if ((inputs.size() != 2 && inputs.size() != 3) || outputs.size() != 1 || outputs[0] == nullptr) {
    return ie::Error::invalid_argument("Gemm expects two or three inputs and one output");
  }
  if (context.allocator == nullptr) return ie::Error::invalid_argument("Gemm requires an allocator");
  for (const ie::Tensor* t : inputs) {
    if (t == nullptr || t->buffer == nullptr) return ie::Error::invalid_argument("null tensor or buffer");
    if (t->dtype != ie::DType::F32) return ie::Error::unsupported("P0 kernels support F32 only");
  }
  const ie::Tensor& a = *inputs[0];
  const ie::Tensor& b = *inputs[1];
  if (a.shape.dims.size() != 2 || b.shape.dims.size() != 2) {
    return ie::Error::invalid_argument("Gemm expects 2D A and B tensors");
  }
  const int64_t m = trans_a_ ? a.shape.dims[1] : a.shape.dims[0];
  const int64_t k_a = trans_a_ ? a.shape.dims[0] : a.shape.dims[1];
  const int64_t k_b = trans_b_ ? b.shape.dims[1] : b.shape.dims[0];
  const int64_t n = trans_b_ ? b.shape.dims[0] : b.shape.dims[1];
  if (m <= 0 || k_a <= 0 || n <= 0 || k_b <= 0) {
    return ie::Error::invalid_argument("Gemm expects positive dimensions");
  }
  if (k_a != k_b) return ie::Error::invalid_argument("Gemm inner dimensions mismatch");
  // C broadcast, the reference's rules (gemm_op.cpp:103-139)
  int32_t c_mode = IE_GEMM_C_NONE;
  const ie::Tensor* c = inputs.size() == 3 ? inputs[2] : nullptr;
  if (c != nullptr) {
    const auto& dims = c->shape.dims;
    if (dims.empty() || c->numel() == 1) {
      c_mode = IE_GEMM_C_SCALAR;
    } else if (dims.size() == 1) {
      if (dims[0] == n) {
        c_mode = IE_GEMM_C_COLUMN;
      } else if (dims[0] == m) {
        c_mode = IE_GEMM_C_ROW;
      } else {
        return ie::Error::invalid_argument("Gemm bias must broadcast to [M,N]");
      }
    } else if (dims.size() == 2) {
      if (dims[0] == m && dims[1] == n) {
        c_mode = IE_GEMM_C_FULL;
      } else if (dims[0] == m && dims[1] == 1) {
        c_mode = IE_GEMM_C_ROW;
      } else if (dims[0] == 1 && dims[1] == n) {
        c_mode = IE_GEMM_C_COLUMN;
      } else {
        return ie::Error::invalid_argument("Gemm bias must broadcast to [M,N]");
      }
    } else {
      return ie::Error::invalid_argument("Gemm bias must broadcast to [M,N]");
    }
  }
  if (auto st = require_device(); !st.has_value()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(context.stream);
  auto ad = to_device(dev_, kSlotX, a, st);
  if (!ad.has_value()) return ad.error();
  auto bd = cached_const(dev_, b, kCacheW, st);
  if (!bd.has_value()) return bd.error();
  const void* cd = nullptr;
  if (c != nullptr) {
    auto r = cached_const(dev_, *c, kCacheBias, st);
    if (!r.has_value()) return r.error();
    cd = *r;
  }
  const size_t ws_bytes = ie_cuda_gemm_f32_workspace_bytes(m, n, m > 0 ? k_a : 0,
                                                           static_cast<int32_t>(trans_a_),
                                                           static_cast<int32_t>(trans_b_));
  auto ws = dev_.scratch(kSlotWork, ws_bytes);
  if (!ws.has_value()) return ws.error();
  auto ydev = dev_.scratch(kSlotY, static_cast<size_t>(m * n) * sizeof(float));
  if (!ydev.has_value()) return ydev.error();
  if (auto e = to_status(ie_cuda_gemm_f32(
          m, n, k_a, static_cast<int32_t>(trans_a_), static_cast<int32_t>(trans_b_),
          static_cast<float>(alpha_), static_cast<float>(beta_), static_cast<const float*>(*ad),
          static_cast<const float*>(*bd), static_cast<const float*>(cd), c_mode,
          static_cast<float*>(*ydev), *ws, ws_bytes, st));
      !e.has_value()) {
    return e;
  }
  return download_f32(*ydev, ie::Shape{{m, n}}, context, outputs, st);
}

namespace {

template <class Registry>
ie::Status register_into(Registry& registry) {
  const std::pair<ie::OpType, std::function<std::unique_ptr<ie::Op>()>> ops[] = {
      {ie::OpType::Conv2D, [] { return std::make_unique<CudaConvNodeOp>(false); }},
      {ie::OpType::DepthwiseConv2D, [] { return std::make_unique<CudaConvNodeOp>(true); }},
      {ie::OpType::Add, [] { return std::make_unique<CudaQLinearAddOp>(); }},
      {ie::OpType::MaxPool2D, [] { return std::make_unique<CudaPool2DOp>(true); }},
      {ie::OpType::AvgPool2D, [] { return std::make_unique<CudaPool2DOp>(false); }},
      {ie::OpType::GlobalAvgPool, [] { return std::make_unique<CudaGlobalAvgPoolOp>(); }},
      {ie::OpType::Gemm, [] { return std::make_unique<CudaGemmOp>(); }},
  };
  for (const auto& [type, creator] : ops) {
    if (auto st = registry.register_op(type, creator); !st.has_value()) return st;
  }
  return {};
}

}  // namespace

ie::Status register_cuda_ops(ie::OpRegistry& registry) { return register_into(registry); }
ie::Status register_cuda_ops(CudaOpTable& table) { return register_into(table); }

ie::Status CudaOpTable::register_op(ie::OpType op, Creator creator) {
  if (!creator) return ie::Error::invalid_argument("empty op creator");
  std::lock_guard<std::mutex> lock(mutex_);
  if (creators_.count(op) != 0) return ie::Error::already_exists("op already registered");
  creators_.emplace(op, std::move(creator));
  return {};
}

ie::Result<std::unique_ptr<ie::Op>> CudaOpTable::create(ie::OpType op) {
  Creator creator;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = creators_.find(op);
    if (it == creators_.end()) return ie::Error::not_found("no CUDA kernel for op");
    creator = it->second;
  }
  auto instance = creator();
  if (!instance) return ie::Error::runtime("op factory returned null");
  return instance;
}

std::vector<ie::OpType> CudaOpTable::list() const {
  std::lock_guard<std::mutex> lock(mutex_);
  std::vector<ie::OpType> out;
  for (const auto& kv : creators_) out.push_back(kv.first);
  return out;
}

}  // namespace ie_b200
