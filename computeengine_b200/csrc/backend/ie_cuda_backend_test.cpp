// Test driver for the C++ CUDA ops (built by computeengine_b200/build.py).
//
//   ie_cuda_backend_test cpu         configure/validation/registry checks that
//                                    need no GPU, plus the loud failure of
//                                    forward() when no CUDA device exists
//   ie_cuda_backend_test gpu <dir>   runs the ops on seeded inputs and writes
//                                    every tensor to <dir> (raw little-endian,
//                                    with manifest.txt) for the Python side
//                                    to check against the oracle
//
// The cases follow the reference's Conv2DOp tests
// (tests/unit/traditional_ops_test.cpp:82-340): attribute errors are
// InvalidArgument, a non-F32 input is Unsupported.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "cuda_conv_ops.h"

using ie::Error;

namespace {

int g_failures = 0;

void expect(bool ok, const char* what) {
  std::printf("%s %s\n", ok ? "ok  " : "FAIL", what);
  if (!ok) ++g_failures;
}

bool has_code(const ie::Status& st, Error::Code code) {
  return !st.has_value() && st.error().code == code;
}

struct Lcg {
  uint64_t s;
  explicit Lcg(uint64_t seed) : s(seed * 6364136223846793005ull + 1442695040888963407ull) {}
  uint32_t next() {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return static_cast<uint32_t>(s >> 33);
  }
  float uniform(float lo, float hi) { return lo + (hi - lo) * (next() / 2147483648.0f); }
};

struct HostTensor {
  ie::Tensor t;
  std::vector<uint8_t> storage;
  HostTensor(std::vector<int64_t> dims, ie::DType dt) {
    t.shape = ie::Shape{std::move(dims)};
    t.dtype = dt;
    storage.resize(t.bytes());
    t.buffer = storage.data();
  }
  template <class T>
  T* data() { return reinterpret_cast<T*>(storage.data()); }
};

ie::ExecutionContext host_context() {
  ie::ExecutionContext ctx;
  ctx.allocator = std::make_shared<ie::MallocAllocator>();
  return ctx;
}

// ------------------------------------------------------------ cpu checks

int run_cpu() {
  using ie_b200::ConvConfig;
  using ie_b200::parse_conv_config;
  ConvConfig cfg;
  expect(parse_conv_config({}, cfg).has_value() && cfg.strides[0] == 1 && cfg.group == 1,
         "defaults");
  expect(parse_conv_config({{"pads", std::vector<int64_t>{1, 2}}}, cfg).has_value() &&
             cfg.pads[0] == 1 && cfg.pads[1] == 2 && cfg.pads[2] == 1 && cfg.pads[3] == 2,
         "two pads are symmetric");
  expect(has_code(parse_conv_config({{"pads", std::vector<int64_t>{1, 2, 3}}}, cfg),
                  Error::Code::InvalidArgument),
         "three pads rejected");
  expect(has_code(parse_conv_config({{"pads", std::vector<int64_t>{-1, 0}}}, cfg),
                  Error::Code::InvalidArgument),
         "negative pad rejected");
  expect(has_code(parse_conv_config({{"strides", std::vector<int64_t>{0, 1}}}, cfg),
                  Error::Code::InvalidArgument),
         "zero stride rejected");
  expect(has_code(parse_conv_config({{"group", int64_t{0}}}, cfg), Error::Code::InvalidArgument),
         "zero group rejected");
  expect(has_code(parse_conv_config({{"group", std::string("2")}}, cfg),
                  Error::Code::InvalidArgument),
         "string group rejected");
  expect(has_code(parse_conv_config({{"auto_pad", std::string("SAME")}}, cfg),
                  Error::Code::InvalidArgument),
         "unknown auto_pad rejected");
  expect(parse_conv_config({{"auto_pad", std::string("SAME_LOWER")}}, cfg).has_value() &&
             cfg.auto_pad == ie_b200::AutoPad::SameLower,
         "SAME_LOWER parsed");
  expect(has_code(parse_conv_config({{"kernel_shape", std::vector<int64_t>{3}}}, cfg),
                  Error::Code::InvalidArgument),
         "one-value kernel_shape rejected");

  // registry: AlreadyExists on a second registration, NotFound for a gap
  ie::OpRegistry reg;
  expect(ie_b200::register_cuda_ops(reg).has_value(), "register_cuda_ops");
  expect(has_code(ie_b200::register_cuda_ops(reg), Error::Code::AlreadyExists),
         "second registration is AlreadyExists");
  auto op = reg.create(ie::OpType::Conv2D);
  expect(op.has_value() && *op != nullptr, "create Conv2D");

  // forward validation (no device needed before the shape checks pass)
  auto ctx = host_context();
  HostTensor x({1, 4, 5, 5}, ie::DType::F32), w({6, 4, 3, 3}, ie::DType::F32);
  HostTensor bias({6}, ie::DType::F32);
  ie::Tensor y;
  std::vector<ie::Tensor*> outs{&y};
  ie_b200::CudaConv2DOp conv;
  expect(conv.configure({{"pads", std::vector<int64_t>{1, 1}}}).has_value(), "configure");
  expect(has_code(conv.forward({&x.t}, outs, ctx), Error::Code::InvalidArgument),
         "one input rejected");
  HostTensor xi({1, 4, 5, 5}, ie::DType::I8);
  expect(has_code(conv.forward({&xi.t, &w.t}, outs, ctx), Error::Code::Unsupported),
         "int8 input to the fp32 op is Unsupported");
  HostTensor wbad({6, 3, 3, 3}, ie::DType::F32);
  expect(has_code(conv.forward({&x.t, &wbad.t}, outs, ctx), Error::Code::InvalidArgument),
         "weight channels != C/group rejected");
  HostTensor bbad({5}, ie::DType::F32);
  expect(has_code(conv.forward({&x.t, &w.t, &bbad.t}, outs, ctx), Error::Code::InvalidArgument),
         "bias of the wrong length rejected");
  ie_b200::CudaConv2DOp grouped;
  grouped.configure({{"group", int64_t{3}}});
  expect(has_code(grouped.forward({&x.t, &w.t}, outs, ctx), Error::Code::InvalidArgument),
         "group not dividing C rejected");
  ie_b200::CudaConv2DOp dw(true);
  dw.configure({});
  expect(has_code(dw.forward({&x.t, &w.t}, outs, ctx), Error::Code::InvalidArgument),
         "depthwise needs group == C");
  ie::ExecutionContext no_alloc;
  expect(has_code(conv.forward({&x.t, &w.t}, outs, no_alloc), Error::Code::InvalidArgument),
         "missing allocator rejected");

  int count = 0;
  const bool has_gpu = cudaGetDeviceCount(&count) == cudaSuccess && count > 0;
  cudaGetLastError();
  if (!has_gpu) {
    // a valid convolution fails loudly: no CPU fallback
    const ie::Status st = conv.forward({&x.t, &w.t, &bias.t}, outs, ctx);
    expect(has_code(st, Error::Code::Runtime), "no device: forward is a Runtime error");
  }
  std::printf("%s (%d failures)\n", g_failures == 0 ? "PASSED" : "FAILED", g_failures);
  return g_failures == 0 ? 0 : 1;
}

// ------------------------------------------------------------ gpu run

void dump(const std::string& dir, std::ofstream& manifest, const char* name,
          const ie::Tensor& t) {
  const std::string path = dir + "/" + name + ".bin";
  std::ofstream f(path, std::ios::binary);
  f.write(static_cast<const char*>(t.buffer), static_cast<std::streamsize>(t.bytes()));
  manifest << name << " " << static_cast<int>(t.dtype);
  for (int64_t d : t.shape.dims) manifest << " " << d;
  manifest << "\n";
}

int run_gpu(const std::string& dir) {
  std::ofstream manifest(dir + "/manifest.txt");
  auto ctx = host_context();
  cudaStream_t stream;
  cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  ctx.stream = stream;
  ie::OpRegistry reg;
  if (!ie_b200::register_cuda_ops(reg).has_value()) return 2;

  // fp32 Conv2D, the 3x3 / 64-channel single-image case, bias, pads 1
  {
    Lcg rng(1);
    HostTensor x({1, 64, 56, 56}, ie::DType::F32), w({64, 64, 3, 3}, ie::DType::F32),
        b({64}, ie::DType::F32);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-1.f, 1.f);
    for (int64_t i = 0; i < w.t.numel(); ++i) w.data<float>()[i] = rng.uniform(-0.1f, 0.1f);
    for (int64_t i = 0; i < b.t.numel(); ++i) b.data<float>()[i] = rng.uniform(-0.01f, 0.01f);
    auto op = reg.create(ie::OpType::Conv2D);
    if (!op.has_value()) return 3;
    (*op)->configure({{"pads", std::vector<int64_t>{1, 1, 1, 1}}});
    ie::Tensor y;
    std::vector<ie::Tensor*> outs{&y};
    ie::Status st = (*op)->forward({&x.t, &w.t, &b.t}, outs, ctx);
    expect(st.has_value(), "Conv2D forward");
    if (!st.has_value()) std::printf("  %s\n", st.error().message.c_str());
    // second call reuses the cached device weights
    ie::Tensor y2;
    std::vector<ie::Tensor*> outs2{&y2};
    st = (*op)->forward({&x.t, &w.t, &b.t}, outs2, ctx);
    expect(st.has_value() && std::memcmp(y.buffer, y2.buffer, y.bytes()) == 0,
           "Conv2D second call identical");
    dump(dir, manifest, "f32_x", x.t);
    dump(dir, manifest, "f32_w", w.t);
    dump(dir, manifest, "f32_b", b.t);
    dump(dir, manifest, "f32_y", y);
  }
  // fp32 DepthwiseConv2D, stride 2, SAME_UPPER
  {
    Lcg rng(2);
    HostTensor x({2, 32, 17, 15}, ie::DType::F32), w({32, 1, 3, 3}, ie::DType::F32);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-1.f, 1.f);
    for (int64_t i = 0; i < w.t.numel(); ++i) w.data<float>()[i] = rng.uniform(-0.5f, 0.5f);
    auto op = reg.create(ie::OpType::DepthwiseConv2D);
    if (!op.has_value()) return 3;
    (*op)->configure({{"group", int64_t{32}},
                      {"strides", std::vector<int64_t>{2, 2}},
                      {"auto_pad", std::string("SAME_UPPER")}});
    ie::Tensor y;
    std::vector<ie::Tensor*> outs{&y};
    const ie::Status st = (*op)->forward({&x.t, &w.t}, outs, ctx);
    expect(st.has_value(), "DepthwiseConv2D forward");
    dump(dir, manifest, "dw_x", x.t);
    dump(dir, manifest, "dw_w", w.t);
    dump(dir, manifest, "dw_y", y);
  }
  // int8 QLinearConv2D, uint8 input with zero point 128, ReLU folded
  {
    Lcg rng(3);
    const int64_t m = 128, c = 128;
    HostTensor x({2, c, 14, 14}, ie::DType::U8), w({m, c, 3, 3}, ie::DType::I8);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<uint8_t>()[i] = static_cast<uint8_t>(rng.next() & 255);
    for (int64_t i = 0; i < w.t.numel(); ++i) {
      w.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int>(rng.next() % 255) - 127);
    }
    std::vector<double> mult(m);
    std::vector<int64_t> bias(m);
    for (int64_t i = 0; i < m; ++i) {
      mult[i] = 0.02 * rng.uniform(0.001f, 0.01f) / 0.05;
      bias[i] = static_cast<int64_t>(rng.next() % 4001) - 2000;
    }
    ie_b200::CudaQLinearConv2DOp op;
    const ie::Status cst = op.configure({{"pads", std::vector<int64_t>{1, 1}},
                                         {"multiplier", mult},
                                         {"bias", bias},
                                         {"x_zero_point", int64_t{128}}});
    expect(cst.has_value(), "QLinearConv2D configure");
    ie::Tensor y;
    std::vector<ie::Tensor*> outs{&y};
    const ie::Status st = op.forward({&x.t, &w.t}, outs, ctx);
    expect(st.has_value(), "QLinearConv2D forward");
    if (!st.has_value()) std::printf("  %s\n", st.error().message.c_str());
    HostTensor mt({m}, ie::DType::F32), bt({m}, ie::DType::F32);
    for (int64_t i = 0; i < m; ++i) {
      mt.data<float>()[i] = static_cast<float>(mult[i]);
      bt.data<float>()[i] = static_cast<float>(bias[i]);  // exact: |bias| <= 2000
    }
    dump(dir, manifest, "q8_x", x.t);
    dump(dir, manifest, "q8_w", w.t);
    dump(dir, manifest, "q8_mult", mt.t);
    dump(dir, manifest, "q8_bias", bt.t);
    dump(dir, manifest, "q8_y", y);
  }
  cudaStreamDestroy(stream);
  std::printf("%s (%d failures)\n", g_failures == 0 ? "PASSED" : "FAILED", g_failures);
  return g_failures == 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 2 && std::strcmp(argv[1], "cpu") == 0) return run_cpu();
  if (argc >= 3 && std::strcmp(argv[1], "gpu") == 0) return run_gpu(argv[2]);
  std::fprintf(stderr, "usage: %s cpu | gpu <outdir>\n", argv[0]);
  return 2;
}
