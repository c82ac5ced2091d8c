// Test driver for the C++ CUDA ops (built by computeengine_b200/build.py).
//
//   ie_cuda_backend_test cpu         configure/validation/registry checks that
//                                    need no GPU, plus the loud failure of
//                                    forward() when no CUDA device exists
//   ie_cuda_backend_test gpu <dir>   runs the ops on seeded inputs and writes
//                                    every tensor to <dir> (raw little-endian,
//                                    with manifest.txt) for the Python side
//                                    to check against the oracle
//   ie_cuda_backend_test quant <dir> runs the int8 quantizer on seeded host
//                                    tensors (no GPU) and writes its outputs
//                                    for the Python side to check
//   ie_cuda_backend_test engine-bench <batch> <iters> <warmup>
//                                    times the int8 ResNet-50 graph through
//                                    CudaExecutor with host tensors (one JSON
//                                    line)
//
// The cases follow the reference's Conv2DOp tests
// (tests/unit/traditional_ops_test.cpp:82-340): attribute errors are
// InvalidArgument, a non-F32 input is Unsupported.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "cuda_conv_ops.h"
#include "cuda_executor.h"
#include "graph_passes.h"
#include "int8_quant.h"

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

// x -> Conv2D(w, b) -> BatchNorm(scale, bias, mean, var) -> act -> y, with
// seeded constants (act: Relu node, or Clip(0, 6) when clip is set).
struct BnGraph {
  ie::Graph g;
  std::vector<std::unique_ptr<HostTensor>> keep;
};

// With with_add: ... -> BatchNorm -> Add(., r) -> act, r a graph input [2, m, 11, 9].
std::unique_ptr<BnGraph> make_bn_graph(bool clip, bool with_add = false, int64_t c = 8,
                                       int64_t m = 12) {
  auto bg = std::make_unique<BnGraph>();
  ie::Graph& g = bg->g;
  Lcg rng(21);
  auto value = [&](ie::ValueId id, const char* name, bool in, bool out) {
    ie::Value v;
    v.id = id;
    v.name = name;
    v.is_input = in;
    v.is_output = out;
    g.values.push_back(v);
  };
  auto constant = [&](const char* name, std::vector<int64_t> dims, float lo, float hi) {
    bg->keep.push_back(std::make_unique<HostTensor>(dims, ie::DType::F32));
    HostTensor& t = *bg->keep.back();
    for (int64_t i = 0; i < t.t.numel(); ++i) t.data<float>()[i] = rng.uniform(lo, hi);
    g.weights.emplace(name, t.t);
  };
  value(0, "x", true, false);
  value(1, "w", false, false);
  value(2, "b", false, false);
  value(3, "conv_out", false, false);
  value(4, "bn_scale", false, false);
  value(5, "bn_bias", false, false);
  value(6, "bn_mean", false, false);
  value(7, "bn_var", false, false);
  value(8, "bn_out", false, false);
  value(9, "y", false, true);
  if (with_add) {
    value(10, "r", true, false);
    value(11, "add_out", false, false);
  }
  constant("w", {m, c, 3, 3}, -0.3f, 0.3f);
  constant("b", {m}, -0.1f, 0.1f);
  constant("bn_scale", {m}, 0.5f, 1.5f);
  constant("bn_bias", {m}, -0.2f, 0.2f);
  constant("bn_mean", {m}, -0.3f, 0.3f);
  constant("bn_var", {m}, 0.2f, 1.2f);
  ie::Node conv;
  conv.id = 0;
  conv.op = ie::OpType::Conv2D;
  conv.inputs = {0, 1, 2};
  conv.outputs = {3};
  conv.attrs = {{"pads", std::vector<int64_t>{1, 1, 1, 1}}};
  ie::Node bn;
  bn.id = 1;
  bn.op = ie::OpType::BatchNorm;
  bn.inputs = {3, 4, 5, 6, 7};
  bn.outputs = {8};
  bn.attrs = {{"epsilon", 1e-3}};
  ie::Node act;
  act.id = 2;
  act.op = clip ? ie::OpType::Clip : ie::OpType::Relu;
  act.inputs = {8};
  act.outputs = {9};
  if (clip) act.attrs = {{"min", 0.0}, {"max", 6.0}};
  if (with_add) {
    ie::Node add;
    add.id = 3;
    add.op = ie::OpType::Add;
    add.inputs = {10, 8};  // residual first: either order is an Add of the conv output
    add.outputs = {11};
    act.inputs = {11};
    g.nodes = {conv, bn, add, act};
    g.edges = {{3, 0u, 1u}, {8, 1u, 3u}, {10, std::nullopt, 3u}, {11, 3u, 2u},
               {9, 2u, std::nullopt}};
  } else {
    g.nodes = {conv, bn, act};
    g.edges = {{3, 0u, 1u}, {8, 1u, 2u}, {9, 2u, std::nullopt}};
  }
  return bg;
}

// A ResNet-shaped graph: conv3x3+BN+Relu -> MaxPool -> conv1x1+BN -> Add
// (pool shortcut) -> Relu -> GlobalAvgPool -> Flatten -> Gemm (FC + bias).
struct NetGraph {
  ie::Graph g;
  std::vector<std::unique_ptr<HostTensor>> keep;
  std::vector<std::string> names;  // constants in creation order
};

std::unique_ptr<NetGraph> make_net_graph() {
  auto ng = std::make_unique<NetGraph>();
  ie::Graph& g = ng->g;
  Lcg rng(31);
  ie::ValueId next = 0;
  auto value = [&](const std::string& name, bool in = false, bool out = false) {
    ie::Value v;
    v.id = next++;
    v.name = name;
    v.is_input = in;
    v.is_output = out;
    g.values.push_back(v);
    return v.id;
  };
  auto constant = [&](const std::string& name, std::vector<int64_t> dims, float lo, float hi) {
    ng->keep.push_back(std::make_unique<HostTensor>(dims, ie::DType::F32));
    HostTensor& t = *ng->keep.back();
    for (int64_t i = 0; i < t.t.numel(); ++i) t.data<float>()[i] = rng.uniform(lo, hi);
    g.weights.emplace(name, t.t);
    ng->names.push_back(name);
    return value(name);
  };
  auto node = [&](ie::OpType op, std::vector<ie::ValueId> in, ie::ValueId out, ie::Attrs attrs = {}) {
    ie::Node n;
    n.id = static_cast<ie::NodeId>(g.nodes.size());
    n.op = op;
    n.inputs = std::move(in);
    n.outputs = {out};
    n.attrs = std::move(attrs);
    g.nodes.push_back(n);
  };
  const ie::ValueId x = value("x", true);
  const ie::ValueId w1 = constant("w1", {16, 3, 3, 3}, -0.4f, 0.4f);
  const ie::ValueId b1 = constant("b1", {16}, -0.1f, 0.1f);
  const ie::ValueId bn1[4] = {constant("bn1_scale", {16}, 0.5f, 1.5f),
                              constant("bn1_bias", {16}, -0.2f, 0.2f),
                              constant("bn1_mean", {16}, -0.2f, 0.2f),
                              constant("bn1_var", {16}, 0.3f, 1.3f)};
  const ie::ValueId w2 = constant("w2", {16, 16, 1, 1}, -0.4f, 0.4f);
  const ie::ValueId bn2[4] = {constant("bn2_scale", {16}, 0.5f, 1.5f),
                              constant("bn2_bias", {16}, -0.2f, 0.2f),
                              constant("bn2_mean", {16}, -0.2f, 0.2f),
                              constant("bn2_var", {16}, 0.3f, 1.3f)};
  const ie::ValueId wfc = constant("wfc", {10, 16}, -0.5f, 0.5f);
  const ie::ValueId bfc = constant("bfc", {10}, -0.1f, 0.1f);
  const ie::ValueId c1 = value("c1"), n1 = value("n1"), r1 = value("r1"), pl = value("pool");
  const ie::ValueId c2 = value("c2"), n2 = value("n2"), ad = value("add"), r2 = value("r2");
  const ie::ValueId gp = value("gap"), fl = value("flat"), y = value("y", false, true);
  node(ie::OpType::Conv2D, {x, w1, b1}, c1, {{"pads", std::vector<int64_t>{1, 1, 1, 1}}});
  node(ie::OpType::BatchNorm, {c1, bn1[0], bn1[1], bn1[2], bn1[3]}, n1);
  node(ie::OpType::Relu, {n1}, r1);
  node(ie::OpType::MaxPool2D, {r1}, pl,
       {{"kernel_shape", std::vector<int64_t>{3, 3}}, {"strides", std::vector<int64_t>{2, 2}},
        {"pads", std::vector<int64_t>{1, 1, 1, 1}}});
  node(ie::OpType::Conv2D, {pl, w2}, c2);
  node(ie::OpType::BatchNorm, {c2, bn2[0], bn2[1], bn2[2], bn2[3]}, n2);
  node(ie::OpType::Add, {n2, pl}, ad);
  node(ie::OpType::Relu, {ad}, r2);
  node(ie::OpType::GlobalAvgPool, {r2}, gp);
  node(ie::OpType::Flatten, {gp}, fl);
  node(ie::OpType::Gemm, {fl, wfc, bfc}, y, {{"transB", int64_t{1}}});
  return ng;
}

// A quantized ResNet bottleneck as the int8 converter would emit it: Conv2D
// nodes carrying the int8 attributes (1x1 -> 3x3 -> 1x1) and an Add node with
// the int8 Add attributes for the shortcut (ReLU folded into its qmin).  The
// input's zero point (37) and conv1's output zero point (10) are neither 0 nor
// 128, so the 3x3 reads a haloed NHWC input and the Add packs the NCHW graph
// input to meet conv3's NHWC output.
struct QGraph {
  ie::Graph g;
  std::vector<std::unique_ptr<HostTensor>> keep;
  std::vector<std::vector<double>> mult;
  std::vector<std::vector<int64_t>> bias;
};

std::unique_ptr<QGraph> make_q8_block_graph(int64_t c = 32, int64_t mid = 16) {
  auto qg = std::make_unique<QGraph>();
  ie::Graph& g = qg->g;
  Lcg rng(41);
  ie::ValueId next = 0;
  auto value = [&](const std::string& name, bool in = false, bool out = false) {
    ie::Value v;
    v.id = next++;
    v.name = name;
    v.is_input = in;
    v.is_output = out;
    g.values.push_back(v);
    return v.id;
  };
  auto weight = [&](const std::string& name, std::vector<int64_t> dims) {
    qg->keep.push_back(std::make_unique<HostTensor>(dims, ie::DType::I8));
    HostTensor& t = *qg->keep.back();
    for (int64_t i = 0; i < t.t.numel(); ++i) {
      t.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 255) - 127);
    }
    g.weights.emplace(name, t.t);
    return value(name);
  };
  auto qattrs = [&](int64_t m, double mlo, double mhi, int64_t zp_x, int64_t zp_y, int64_t qmin,
                    int64_t pad) {
    std::vector<double> mult(static_cast<size_t>(m));
    std::vector<int64_t> bias(static_cast<size_t>(m));
    for (int64_t i = 0; i < m; ++i) {
      mult[static_cast<size_t>(i)] = static_cast<double>(static_cast<float>(mlo + (mhi - mlo) * rng.uniform(0.f, 1.f)));
      bias[static_cast<size_t>(i)] = static_cast<int64_t>(rng.next() % 4001) - 2000;
    }
    qg->mult.push_back(mult);
    qg->bias.push_back(bias);
    return ie::Attrs{{"multiplier", mult}, {"bias", bias}, {"x_zero_point", zp_x},
                     {"y_zero_point", zp_y}, {"qmin", qmin}, {"qmax", int64_t{255}},
                     {"pads", std::vector<int64_t>{pad, pad, pad, pad}}};
  };
  auto node = [&](ie::OpType op, std::vector<ie::ValueId> in, ie::ValueId out, ie::Attrs attrs) {
    ie::Node n;
    n.id = static_cast<ie::NodeId>(g.nodes.size());
    n.op = op;
    n.inputs = std::move(in);
    n.outputs = {out};
    n.attrs = std::move(attrs);
    g.nodes.push_back(n);
  };
  const ie::ValueId x = value("x", true);
  const ie::ValueId w1 = weight("qw1", {mid, c, 1, 1});
  const ie::ValueId w2 = weight("qw2", {mid, mid, 3, 3});
  const ie::ValueId w3 = weight("qw3", {c, mid, 1, 1});
  const ie::ValueId c1 = value("qc1"), c2 = value("qc2"), c3 = value("qc3"), sum = value("qsum");
  const ie::ValueId y = value("qy", false, true);
  node(ie::OpType::Conv2D, {x, w1}, c1, qattrs(mid, 0.004, 0.008, 37, 10, 10, 0));
  node(ie::OpType::Conv2D, {c1, w2}, c2, qattrs(mid, 0.0015, 0.003, 10, 0, 0, 1));
  node(ie::OpType::Conv2D, {c2, w3}, c3, qattrs(c, 0.004, 0.008, 0, 128, 0, 0));
  node(ie::OpType::Add, {c3, x}, sum,
       {{"a_multiplier", std::vector<double>{0.5}}, {"b_multiplier", std::vector<double>{0.75}},
        {"a_zero_point", int64_t{128}}, {"b_zero_point", int64_t{37}},
        {"y_zero_point", int64_t{0}}, {"qmin", int64_t{0}}});
  // the stem's pool shape on the int8 activation layout
  node(ie::OpType::MaxPool2D, {sum}, y,
       {{"kernel_shape", std::vector<int64_t>{3, 3}}, {"strides", std::vector<int64_t>{2, 2}},
        {"pads", std::vector<int64_t>{1, 1, 1, 1}}});
  return qg;
}

// A whole quantized network, stem to logits: int8 stem Conv2D 7x7 / 2 (input
// zero point 128) -> MaxPool 3x3 / 2 -> bottleneck (1x1 -> 3x3 -> 1x1, the
// last with zero point 128 and no ReLU) + int8 shortcut Add with ReLU ->
// GlobalAvgPool of the int8 activation into fp32 -> Flatten -> fp32 Gemm.
std::unique_ptr<QGraph> make_q8_net_graph() {
  auto qg = std::make_unique<QGraph>();
  ie::Graph& g = qg->g;
  Lcg rng(53);
  ie::ValueId next = 0;
  auto value = [&](const std::string& name, bool in = false, bool out = false) {
    ie::Value v;
    v.id = next++;
    v.name = name;
    v.is_input = in;
    v.is_output = out;
    g.values.push_back(v);
    return v.id;
  };
  auto tensor = [&](const std::string& name, std::vector<int64_t> dims, ie::DType dt) {
    qg->keep.push_back(std::make_unique<HostTensor>(dims, dt));
    HostTensor& t = *qg->keep.back();
    for (int64_t i = 0; i < t.t.numel(); ++i) {
      if (dt == ie::DType::I8) {
        t.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 255) - 127);
      } else {
        t.data<float>()[i] = rng.uniform(-0.5f, 0.5f);
      }
    }
    g.weights.emplace(name, t.t);
    return value(name);
  };
  auto qattrs = [&](int64_t m, double mlo, double mhi, int64_t zp_x, int64_t zp_y, int64_t qmin,
                    int64_t pad, int64_t stride) {
    std::vector<double> mult(static_cast<size_t>(m));
    std::vector<int64_t> bias(static_cast<size_t>(m));
    for (int64_t i = 0; i < m; ++i) {
      mult[static_cast<size_t>(i)] = static_cast<double>(static_cast<float>(mlo + (mhi - mlo) * rng.uniform(0.f, 1.f)));
      bias[static_cast<size_t>(i)] = static_cast<int64_t>(rng.next() % 2001) - 1000;
    }
    qg->mult.push_back(mult);
    qg->bias.push_back(bias);
    return ie::Attrs{{"multiplier", mult}, {"bias", bias}, {"x_zero_point", zp_x},
                     {"y_zero_point", zp_y}, {"qmin", qmin}, {"qmax", int64_t{255}},
                     {"pads", std::vector<int64_t>{pad, pad, pad, pad}},
                     {"strides", std::vector<int64_t>{stride, stride}}};
  };
  auto node = [&](ie::OpType op, std::vector<ie::ValueId> in, ie::ValueId out, ie::Attrs attrs = {}) {
    ie::Node n;
    n.id = static_cast<ie::NodeId>(g.nodes.size());
    n.op = op;
    n.inputs = std::move(in);
    n.outputs = {out};
    n.attrs = std::move(attrs);
    g.nodes.push_back(n);
  };
  const ie::ValueId x = value("x", true);
  const ie::ValueId w0 = tensor("nw0", {16, 3, 7, 7}, ie::DType::I8);
  const ie::ValueId w1 = tensor("nw1", {8, 16, 1, 1}, ie::DType::I8);
  const ie::ValueId w2 = tensor("nw2", {8, 8, 3, 3}, ie::DType::I8);
  const ie::ValueId w3 = tensor("nw3", {16, 8, 1, 1}, ie::DType::I8);
  const ie::ValueId wfc = tensor("nfcw", {10, 16}, ie::DType::F32);
  const ie::ValueId bfc = tensor("nfcb", {10}, ie::DType::F32);
  const ie::ValueId s0 = value("ns0"), pl = value("npool"), c1 = value("nc1"), c2 = value("nc2"),
                    c3 = value("nc3"), sum = value("nsum"), gp = value("ngap"), fl = value("nflat");
  const ie::ValueId y = value("ny", false, true);
  node(ie::OpType::Conv2D, {x, w0}, s0, qattrs(16, 0.002, 0.004, 128, 0, 0, 3, 2));
  node(ie::OpType::MaxPool2D, {s0}, pl,
       {{"kernel_shape", std::vector<int64_t>{3, 3}}, {"strides", std::vector<int64_t>{2, 2}},
        {"pads", std::vector<int64_t>{1, 1, 1, 1}}});
  node(ie::OpType::Conv2D, {pl, w1}, c1, qattrs(8, 0.004, 0.008, 0, 0, 0, 0, 1));
  node(ie::OpType::Conv2D, {c1, w2}, c2, qattrs(8, 0.002, 0.004, 0, 0, 0, 1, 1));
  node(ie::OpType::Conv2D, {c2, w3}, c3, qattrs(16, 0.004, 0.008, 0, 128, 0, 0, 1));
  node(ie::OpType::Add, {c3, pl}, sum,
       {{"a_multiplier", std::vector<double>{0.5}}, {"b_multiplier", std::vector<double>{0.75}},
        {"a_zero_point", int64_t{128}}, {"b_zero_point", int64_t{0}},
        {"y_zero_point", int64_t{0}}, {"qmin", int64_t{0}}});
  node(ie::OpType::GlobalAvgPool, {sum}, gp, {{"x_scale", 0.05}, {"x_zero_point", int64_t{0}}});
  node(ie::OpType::Flatten, {gp}, fl);
  node(ie::OpType::Gemm, {fl, wfc, bfc}, y, {{"transB", int64_t{1}}});
  return qg;
}


// The whole int8 ResNet-50 v1.5 as one engine graph: the 7x7 / 2 stem (uint8
// input, zero point 128), MaxPool 3x3 / 2, 16 bottlenecks (1x1 -> 3x3 -> 1x1,
// stride on the 3x3, 1x1 projection on each stage's first block) with the
// int8 shortcut Add + ReLU, the int8 GlobalAvgPool into fp32, Flatten and the
// fp32 FC 2048 -> 1000.  The int8 scheme of the benchmark's convolution
// stack: per-channel weights U{-127..127} with scales U(0.001, 0.01), int32
// bias U{-1000..1000}, activation scale 0.05 (input 0.02), multiplier
// fp32(s_x * s_w / s_y); ReLU outputs have zero point 0, the block's last
// 1x1 and the projection (no ReLU before the Add) zero point 128.
std::unique_ptr<QGraph> make_resnet50_q8_graph() {
  auto qg = std::make_unique<QGraph>();
  ie::Graph& g = qg->g;
  Lcg rng(50);
  ie::ValueId next = 0;
  auto value = [&](const std::string& name, bool in = false, bool out = false) {
    ie::Value v;
    v.id = next++;
    v.name = name;
    v.is_input = in;
    v.is_output = out;
    g.values.push_back(v);
    return v.id;
  };
  auto node = [&](ie::OpType op, std::vector<ie::ValueId> in, ie::ValueId out, ie::Attrs attrs = {}) {
    ie::Node n;
    n.id = static_cast<ie::NodeId>(g.nodes.size());
    n.op = op;
    n.inputs = std::move(in);
    n.outputs = {out};
    n.attrs = std::move(attrs);
    g.nodes.push_back(n);
  };
  constexpr double kAct = 0.05, kIn = 0.02;
  int conv_id = 0;
  // a quantized Conv2D node; returns its output value
  auto conv = [&](ie::ValueId x, int64_t cin, int64_t cout, int64_t k, int64_t stride, double s_x,
                  int64_t zp_x, bool relu) {
    const std::string name = "c" + std::to_string(conv_id++);
    qg->keep.push_back(std::make_unique<HostTensor>(std::vector<int64_t>{cout, cin, k, k}, ie::DType::I8));
    HostTensor& w = *qg->keep.back();
    for (int64_t i = 0; i < w.t.numel(); ++i) {
      w.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 255) - 127);
    }
    g.weights.emplace(name + "_w", w.t);
    const ie::ValueId wv = value(name + "_w");
    std::vector<double> mult(static_cast<size_t>(cout));
    std::vector<int64_t> bias(static_cast<size_t>(cout));
    for (int64_t i = 0; i < cout; ++i) {
      const double s_w = 0.001 + 0.009 * rng.uniform(0.f, 1.f);
      mult[static_cast<size_t>(i)] = static_cast<double>(static_cast<float>(s_x * s_w / kAct));
      bias[static_cast<size_t>(i)] = static_cast<int64_t>(rng.next() % 2001) - 1000;
    }
    const int64_t pad = k / 2;
    const ie::ValueId y = value(name);
    node(ie::OpType::Conv2D, {x, wv}, y,
         ie::Attrs{{"multiplier", mult}, {"bias", bias}, {"x_zero_point", zp_x},
                   {"y_zero_point", int64_t{relu ? 0 : 128}}, {"qmin", int64_t{0}},
                   {"qmax", int64_t{255}}, {"pads", std::vector<int64_t>{pad, pad, pad, pad}},
                   {"strides", std::vector<int64_t>{stride, stride}}});
    return y;
  };
  const ie::ValueId x = value("x", true);
  ie::ValueId h = conv(x, 3, 64, 7, 2, kIn, 128, true);
  const ie::ValueId pooled = value("pool");
  node(ie::OpType::MaxPool2D, {h}, pooled,
       {{"kernel_shape", std::vector<int64_t>{3, 3}}, {"strides", std::vector<int64_t>{2, 2}},
        {"pads", std::vector<int64_t>{1, 1, 1, 1}}});
  h = pooled;
  int64_t cin = 64;
  const int64_t widths[4] = {64, 128, 256, 512}, blocks[4] = {3, 4, 6, 3};
  int add_id = 0;
  for (int st = 0; st < 4; ++st) {
    for (int64_t b = 0; b < blocks[st]; ++b) {
      const int64_t wd = widths[st], stride = (st > 0 && b == 0) ? 2 : 1;
      const ie::ValueId c1 = conv(h, cin, wd, 1, 1, kAct, 0, true);
      const ie::ValueId c2 = conv(c1, wd, wd, 3, stride, kAct, 0, true);
      const ie::ValueId c3 = conv(c2, wd, 4 * wd, 1, 1, kAct, 0, false);
      ie::ValueId sc = h;
      int64_t zp_sc = 0;
      if (b == 0) {
        sc = conv(h, cin, 4 * wd, 1, stride, kAct, 0, false);
        zp_sc = 128;
      }
      const ie::ValueId sum = value("add" + std::to_string(add_id++));
      node(ie::OpType::Add, {c3, sc}, sum,
           {{"a_multiplier", std::vector<double>{1.0}}, {"b_multiplier", std::vector<double>{1.0}},
            {"a_zero_point", int64_t{128}}, {"b_zero_point", zp_sc},
            {"y_zero_point", int64_t{0}}, {"qmin", int64_t{0}}});
      h = sum;
      cin = 4 * wd;
    }
  }
  const ie::ValueId gp = value("gap"), fl = value("flat"), y = value("logits", false, true);
  node(ie::OpType::GlobalAvgPool, {h}, gp, {{"x_scale", kAct}, {"x_zero_point", int64_t{0}}});
  node(ie::OpType::Flatten, {gp}, fl);
  qg->keep.push_back(std::make_unique<HostTensor>(std::vector<int64_t>{1000, 2048}, ie::DType::F32));
  HostTensor& fw = *qg->keep.back();
  for (int64_t i = 0; i < fw.t.numel(); ++i) fw.data<float>()[i] = rng.uniform(-0.05f, 0.05f);
  qg->keep.push_back(std::make_unique<HostTensor>(std::vector<int64_t>{1000}, ie::DType::F32));
  HostTensor& fb = *qg->keep.back();
  for (int64_t i = 0; i < fb.t.numel(); ++i) fb.data<float>()[i] = rng.uniform(-0.1f, 0.1f);
  g.weights.emplace("fc_w", fw.t);
  g.weights.emplace("fc_b", fb.t);
  const ie::ValueId fwv = value("fc_w"), fbv = value("fc_b");
  node(ie::OpType::Gemm, {fl, fwv, fbv}, y, {{"transB", int64_t{1}}});
  return qg;
}

// Page-locked host memory behind the engine's Allocator interface, so the
// executor's input upload and logits download run at full link speed.
class PinnedAllocator final : public ie::Allocator {
 public:
  ie::Result<ie::BufferHandle> alloc(std::size_t bytes, ie::MemoryKind) override {
    void* p = nullptr;
    if (cudaHostAlloc(&p, bytes == 0 ? 1 : bytes, cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      return ie::Error::out_of_memory("cudaHostAlloc");
    }
    return p;
  }
  void free(ie::BufferHandle handle) override {
    if (handle != nullptr) cudaFreeHost(handle);
  }
  std::size_t available(ie::MemoryKind) const override { return 0; }
};


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

  // Conv + BatchNorm + Relu fusion pass on the graph
  {
    auto bg = make_bn_graph(false);
    ie_b200::ConvBnReluFusionPass pass;
    ie::PassContext pctx;
    const ie::Status st = pass.run(bg->g, pctx);
    const ie::Graph& g = bg->g;
    expect(st.has_value() && pass.folded_batch_norms() == 1 && pass.fused_activations() == 1 &&
               g.nodes.size() == 1,
           "conv + BN + Relu fused into one node");
    if (g.nodes.size() == 1) {
      const ie::Node& n = g.nodes[0];
      const auto* act = std::get_if<std::string>(&n.attrs.at("activation"));
      expect(act != nullptr && *act == "Relu" && n.outputs == std::vector<ie::ValueId>{9} &&
                 n.inputs.size() == 3 && n.inputs[0] == 0,
             "fused node writes y with activation Relu");
      const ie::Value* wv = g.find_value(n.inputs[1]);
      expect(wv != nullptr && wv->name == "w.bn_folded" && g.weights.count("w.bn_folded") == 1 &&
                 g.weights.count("w") == 1,
             "folded weights added beside the originals");
      expect(g.edges.size() == 1 && g.edges[0].value == 9 && g.edges[0].from.has_value() &&
                 *g.edges[0].from == 0u,
             "edges rewired to the fused node");
    }
    auto bc = make_bn_graph(true);
    ie_b200::ConvBnReluFusionPass pass2;
    expect(pass2.run(bc->g, pctx).has_value() && bc->g.nodes.size() == 1 &&
               *std::get_if<std::string>(&bc->g.nodes[0].attrs.at("activation")) == "Relu6",
           "Clip(0, 6) fused as Relu6");
    auto bo = make_bn_graph(false);
    for (ie::Value& v : bo->g.values) {
      if (v.name == "conv_out") v.is_output = true;
    }
    ie_b200::ConvBnReluFusionPass pass3;
    expect(pass3.run(bo->g, pctx).has_value() && bo->g.nodes.size() == 3 &&
               pass3.folded_batch_norms() == 0,
           "no fold when the conv output is a graph output");
    auto bt = make_bn_graph(false);
    bt->g.nodes[2].inputs = {3};  // a second consumer of the conv output
    ie_b200::ConvBnReluFusionPass pass4;
    expect(pass4.run(bt->g, pctx).has_value() && pass4.folded_batch_norms() == 0,
           "no fold when the conv output has two consumers");
    auto bv = make_bn_graph(false);
    bv->keep[5]->data<float>()[3] = -1.0f;  // var + eps < 0
    ie_b200::ConvBnReluFusionPass pass5;
    expect(has_code(pass5.run(bv->g, pctx), Error::Code::InvalidArgument),
           "negative variance rejected");
    ie_b200::CudaConv2DOp act_op;
    expect(has_code(act_op.configure({{"activation", std::string("Tanh")}}),
                    Error::Code::InvalidArgument),
           "unknown activation rejected");
    auto ba = make_bn_graph(false, true);
    ie_b200::ConvBnReluFusionPass pass6;
    expect(pass6.run(ba->g, pctx).has_value() && ba->g.nodes.size() == 1 &&
               pass6.folded_batch_norms() == 1 && pass6.fused_adds() == 1 &&
               pass6.fused_activations() == 1,
           "conv + BN + Add + Relu fused into one node");
    if (ba->g.nodes.size() == 1) {
      const ie::Node& n = ba->g.nodes[0];
      const auto* fa = std::get_if<int64_t>(&n.attrs.at("fused_add"));
      expect(fa != nullptr && *fa == 1 && n.inputs.size() == 4 && n.inputs[3] == 10 &&
                 n.outputs == std::vector<ie::ValueId>{9},
             "residual is the fused node's fourth input");
      bool edge_ok = false;
      for (const ie::Edge& e : ba->g.edges) {
        if (e.value == 10 && e.to.has_value() && *e.to == 0u) edge_ok = true;
      }
      expect(edge_ok && ba->g.edges.size() == 2, "residual edge now feeds the fused node");
    }
    auto bl = make_bn_graph(false, true);
    for (ie::Value& v : bl->g.values) {
      if (v.id == 10) v.is_input = false;  // the residual is produced by nothing before the conv
    }
    ie_b200::ConvBnReluFusionPass pass7;
    expect(pass7.run(bl->g, pctx).has_value() && pass7.fused_adds() == 0,
           "no add fusion when the residual is not available at the conv");
    ie_b200::CudaConv2DOp fa_op;
    fa_op.configure({{"fused_add", int64_t{1}}});
    expect(has_code(fa_op.forward({&x.t, &w.t, &bias.t}, outs, ctx), Error::Code::InvalidArgument),
           "fused add without the residual input rejected");
  }

  // pooling and Gemm ops: attribute and shape errors as the reference reports them
  {
    ie_b200::PoolConfig pc;
    expect(has_code(ie_b200::parse_pool_config({}, pc), Error::Code::InvalidArgument),
           "pool without kernel_shape rejected");
    expect(has_code(ie_b200::parse_pool_config({{"kernel_shape", std::vector<int64_t>{3, 3, 3}}}, pc),
                    Error::Code::InvalidArgument),
           "three-value kernel_shape rejected");
    expect(ie_b200::parse_pool_config({{"kernel_shape", std::vector<int64_t>{3, 3}},
                                       {"ceil_mode", int64_t{1}}},
                                      pc)
                   .has_value() &&
               pc.ceil_mode && pc.kernel_shape[0] == 3,
           "pool config parsed");
    auto mp = reg.create(ie::OpType::MaxPool2D);
    auto gp = reg.create(ie::OpType::GlobalAvgPool);
    auto gm = reg.create(ie::OpType::Gemm);
    expect(mp.has_value() && gp.has_value() && gm.has_value(), "create pool / GAP / Gemm ops");
    ie_b200::CudaPool2DOp pool(true);
    pool.configure({{"kernel_shape", std::vector<int64_t>{7, 7}}});
    expect(has_code(pool.forward({&x.t}, outs, ctx), Error::Code::InvalidArgument),
           "pool window larger than the input rejected");
    ie_b200::CudaGlobalAvgPoolOp gap;
    HostTensor x3({4, 5, 5}, ie::DType::F32);
    expect(has_code(gap.forward({&x3.t}, outs, ctx), Error::Code::InvalidArgument),
           "GAP on a 3D tensor rejected");
    ie_b200::CudaGemmOp gemm;
    expect(has_code(gemm.configure({{"transA", int64_t{2}}}), Error::Code::InvalidArgument),
           "Gemm transA = 2 rejected");
    gemm.configure({});
    HostTensor ga({4, 5}, ie::DType::F32), gb({6, 3}, ie::DType::F32), gc({7}, ie::DType::F32),
        gb2({5, 3}, ie::DType::F32);
    expect(has_code(gemm.forward({&ga.t, &gb.t}, outs, ctx), Error::Code::InvalidArgument),
           "Gemm inner dimension mismatch rejected");
    expect(has_code(gemm.forward({&ga.t, &gb2.t, &gc.t}, outs, ctx), Error::Code::InvalidArgument),
           "Gemm bias that does not broadcast rejected");
    HostTensor gi({4, 5}, ie::DType::I8);
    expect(has_code(gemm.forward({&gi.t, &gb2.t}, outs, ctx), Error::Code::Unsupported),
           "Gemm on int8 is Unsupported");
  }

  // int8 quantizer: the reference plugin contract and its error codes
  {
    ie_b200::Int8QuantPlugin plug;
    const ie::PluginMeta meta = plug.meta();
    expect(meta.name == "int8_quant" && meta.api_version == "0.1", "quant plugin meta");
    HostTensor wt({2, 3}, ie::DType::F32);
    const float wv[6] = {1.0f, -0.5f, 0.25f, 0.0f, 0.0f, 0.0f};
    std::memcpy(wt.data<float>(), wv, sizeof(wv));
    ie::QuantConfig sym;  // int8, symmetric
    auto q = plug.quantize(wt.t, sym);
    expect(q.has_value() && q->dtype == ie::DType::I8 && q->shape.dims == wt.t.shape.dims,
           "symmetric quantize gives I8 of the same shape");
    if (q.has_value()) {
      const int8_t* qv = q->data<int8_t>();
      // channel 0: scale 1/127, -63.5 rounds to even (-64), 31.75 -> 32; channel 1 all zero
      expect(qv[0] == 127 && qv[1] == -64 && qv[2] == 32 && qv[3] == 0 && qv[5] == 0,
             "per-channel symmetric known answer");
      const ie_b200::QuantParams* p = plug.params(*q);
      expect(p != nullptr && p->per_channel && p->scales.size() == 2 && p->scales[1] == 1.0f,
             "params kept with the result (all-zero channel has scale 1)");
      auto back = plug.dequantize(*q, sym);
      expect(back.has_value() && back->dtype == ie::DType::F32 &&
                 back->data<float>()[0] == 127.0f * p->scales[0],
             "dequantize with the kept parameters");
    }
    ie::QuantConfig four = sym;
    four.bits = 4;
    expect(!plug.quantize(wt.t, four).has_value() &&
               plug.quantize(wt.t, four).error().code == Error::Code::Unsupported,
           "4-bit quantization is Unsupported");
    ie::QuantConfig gguf = sym;
    gguf.format = "gguf";
    expect(plug.quantize(wt.t, gguf).error().code == Error::Code::Unsupported,
           "unknown format is Unsupported");
    HostTensor wi({2, 3}, ie::DType::I8);
    expect(plug.quantize(wi.t, sym).error().code == Error::Code::Unsupported,
           "non-F32 input is Unsupported");
    HostTensor nan_t({3}, ie::DType::F32);
    nan_t.data<float>()[0] = 0.0f;
    nan_t.data<float>()[1] = std::nanf("");
    nan_t.data<float>()[2] = 1.0f;
    expect(plug.quantize(nan_t.t, sym).error().code == Error::Code::InvalidArgument,
           "non-finite value is InvalidArgument");
    ie::Tensor empty;
    empty.shape = ie::Shape{{0}};
    expect(plug.quantize(empty, sym).error().code == Error::Code::InvalidArgument,
           "empty tensor is InvalidArgument");
    HostTensor foreign({3}, ie::DType::I8);
    expect(plug.dequantize(foreign.t, sym).error().code == Error::Code::NotFound,
           "dequantize of a foreign tensor is NotFound");
    ie_b200::ActivationCalibrator cal;
    expect(!cal.params().has_value(), "empty calibrator has no range");
    ie_b200::QuantParams xp = ie_b200::u8_params_for_range(0.0f, 2.55f);
    ie_b200::QuantParams bad_w = xp;  // U8 where int8 weights are expected
    expect(ie_b200::make_qlinear_conv_attrs({}, xp, bad_w, xp, 1, nullptr,
                                            ie_b200::FusedActivation::None)
                   .error()
                   .code == Error::Code::InvalidArgument,
           "qlinear attrs reject uint8 weights");
  }

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

  // Device-resident weights are read on every call: the same device buffer
  // rewritten with new weights gives the result of the new weights (int8 and
  // fp32 convolutions), never a packed copy of the old ones.
  {
    Lcg rng(71);
    HostTensor xq({2, 16, 9, 9}, ie::DType::U8), xf({2, 16, 9, 9}, ie::DType::F32);
    HostTensor wq1({8, 16, 3, 3}, ie::DType::I8), wq2({8, 16, 3, 3}, ie::DType::I8);
    HostTensor wf1({8, 16, 3, 3}, ie::DType::F32), wf2({8, 16, 3, 3}, ie::DType::F32);
    for (int64_t i = 0; i < xq.t.numel(); ++i) {
      xq.data<uint8_t>()[i] = static_cast<uint8_t>(rng.next() % 256);
      xf.data<float>()[i] = rng.uniform(-1.f, 1.f);
    }
    for (int64_t i = 0; i < wq1.t.numel(); ++i) {
      wq1.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 255) - 127);
      wq2.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 255) - 127);
      wf1.data<float>()[i] = rng.uniform(-0.2f, 0.2f);
      wf2.data<float>()[i] = rng.uniform(-0.2f, 0.2f);
    }
    const ie::Attrs qattrs{{"multiplier", std::vector<double>(8, 0.004)},
                           {"bias", std::vector<int64_t>(8, 100)},
                           {"x_zero_point", int64_t{128}},
                           {"y_zero_point", int64_t{0}},
                           {"pads", std::vector<int64_t>{1, 1, 1, 1}}};
    const ie::Attrs fattrs{{"pads", std::vector<int64_t>{1, 1, 1, 1}}};
    struct Case {
      const char* name;
      HostTensor* x;
      HostTensor* w1;
      HostTensor* w2;
      const ie::Attrs* attrs;
    } cases[] = {{"DEVW int8", &xq, &wq1, &wq2, &qattrs}, {"DEVW fp32", &xf, &wf1, &wf2, &fattrs}};
    for (const Case& c : cases) {
      void* wd = nullptr;
      if (cudaMalloc(&wd, c.w1->t.bytes()) != cudaSuccess) return 3;
      ie::Tensor wdev = c.w1->t;
      wdev.buffer = wd;
      wdev.device = ie::Device::CUDA;
      auto op = reg.create(ie::OpType::Conv2D);
      auto fresh_op = reg.create(ie::OpType::Conv2D);
      if (!op.has_value() || !fresh_op.has_value()) return 3;
      expect((*op)->configure(*c.attrs).has_value() && (*fresh_op)->configure(*c.attrs).has_value(),
             c.name);
      ie::Tensor y1, y2, y2_ref;
      std::vector<ie::Tensor*> o1{&y1}, o2{&y2}, o3{&y2_ref};
      cudaMemcpy(wd, c.w1->t.buffer, c.w1->t.bytes(), cudaMemcpyHostToDevice);
      const bool ok1 = (*op)->forward({&c.x->t, &wdev}, o1, ctx).has_value();
      cudaMemcpy(wd, c.w2->t.buffer, c.w2->t.bytes(), cudaMemcpyHostToDevice);
      const bool ok2 = (*op)->forward({&c.x->t, &wdev}, o2, ctx).has_value();
      const bool ok3 = (*fresh_op)->forward({&c.x->t, &c.w2->t}, o3, ctx).has_value();
      expect(ok1 && ok2 && ok3, c.name);
      if (ok1 && ok2 && ok3) {
        expect(y2.bytes() == y2_ref.bytes() && std::memcmp(y2.buffer, y2_ref.buffer, y2.bytes()) == 0,
               c.name);
        expect(std::memcmp(y1.buffer, y2.buffer, y1.bytes()) != 0, c.name);
      }
      cudaFree(wd);
    }
  }
  // Executor liveness: a value that is a graph output and also read by a
  // later node stays alive to the end of the run (int8 x -> conv1 -> c1
  // (output) -> conv2 -> y (output)); c1 equals conv1 run on its own, and a
  // second run of the same executor gives the same bytes.
  {
    Lcg rng(83);
    ie::Graph g;
    std::vector<std::unique_ptr<HostTensor>> keep;
    ie::ValueId next = 0;
    auto value = [&](const std::string& name, bool in = false, bool out = false) {
      ie::Value v;
      v.id = next++;
      v.name = name;
      v.is_input = in;
      v.is_output = out;
      g.values.push_back(v);
      return v.id;
    };
    auto weight = [&](const std::string& name, std::vector<int64_t> dims) {
      keep.push_back(std::make_unique<HostTensor>(dims, ie::DType::I8));
      for (int64_t i = 0; i < keep.back()->t.numel(); ++i) {
        keep.back()->data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 255) - 127);
      }
      g.weights.emplace(name, keep.back()->t);
      return value(name);
    };
    const ie::Attrs qa{{"multiplier", std::vector<double>(16, 0.003)},
                       {"bias", std::vector<int64_t>(16, -50)},
                       {"x_zero_point", int64_t{0}},
                       {"y_zero_point", int64_t{0}},
                       {"pads", std::vector<int64_t>{1, 1, 1, 1}}};
    const ie::ValueId x = value("x", true);
    const ie::ValueId w1 = weight("lw1", {16, 16, 3, 3}), w2 = weight("lw2", {16, 16, 3, 3});
    const ie::ValueId c1 = value("c1", false, true), y = value("y", false, true);
    auto add_node = [&](ie::ValueId in, ie::ValueId w, ie::ValueId out) {
      ie::Node n;
      n.id = static_cast<ie::NodeId>(g.nodes.size());
      n.op = ie::OpType::Conv2D;
      n.inputs = {in, w};
      n.outputs = {out};
      n.attrs = qa;
      g.nodes.push_back(n);
    };
    add_node(x, w1, c1);
    add_node(c1, w2, y);
    HostTensor xin({2, 16, 12, 10}, ie::DType::U8);
    for (int64_t i = 0; i < xin.t.numel(); ++i) xin.data<uint8_t>()[i] = static_cast<uint8_t>(rng.next() % 256);
    ie_b200::CudaExecutor exec(reg);
    std::unordered_map<std::string, ie::Tensor> in{{"x", xin.t}};
    auto r1 = exec.run(g, in, std::make_shared<ie::MallocAllocator>(), stream);
    auto r2 = exec.run(g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(r1.has_value() && r2.has_value() && r1->size() == 2 && r2->size() == 2, "LIVE: runs");
    auto op = reg.create(ie::OpType::Conv2D);
    if (!op.has_value()) return 3;
    expect((*op)->configure(qa).has_value(), "LIVE: configure");
    ie::Tensor c1_ref;
    std::vector<ie::Tensor*> o{&c1_ref};
    const bool ok = (*op)->forward({&xin.t, &keep[0]->t}, o, ctx).has_value();
    if (r1.has_value() && r2.has_value() && r1->size() == 2 && r2->size() == 2 && ok) {
      const ie::Tensor& c1_out = (*r1)[0];
      expect(c1_out.shape.dims == c1_ref.shape.dims && c1_out.bytes() == c1_ref.bytes() &&
                 std::memcmp(c1_out.buffer, c1_ref.buffer, c1_ref.bytes()) == 0,
             "LIVE: output read by a later node equals conv1 alone");
      bool same = true;
      for (size_t k = 0; k < 2; ++k) {
        same = same && (*r1)[k].bytes() == (*r2)[k].bytes() &&
               std::memcmp((*r1)[k].buffer, (*r2)[k].buffer, (*r1)[k].bytes()) == 0;
      }
      expect(same, "LIVE: second run identical");
    } else {
      expect(false, "LIVE: results");
    }
  }
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
  // a failed device allocation is reported as OutOfMemory, and the op works
  // again once allocation succeeds
  {
    Lcg rng(9);
    HostTensor x({1, 16, 10, 10}, ie::DType::F32), w({16, 16, 3, 3}, ie::DType::F32);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-1.f, 1.f);
    for (int64_t i = 0; i < w.t.numel(); ++i) w.data<float>()[i] = rng.uniform(-0.1f, 0.1f);
    auto op = reg.create(ie::OpType::Conv2D);
    if (!op.has_value()) return 3;
    (*op)->configure({{"pads", std::vector<int64_t>{1, 1, 1, 1}}});
    ie_b200::set_device_alloc([](void** p, size_t) -> int {
      *p = nullptr;
      return static_cast<int>(cudaErrorMemoryAllocation);
    });
    ie::Tensor y;
    std::vector<ie::Tensor*> outs{&y};
    ie::Status st = (*op)->forward({&x.t, &w.t}, outs, ctx);
    expect(!st.has_value() && st.error().code == ie::Error::Code::OutOfMemory,
           "failed device allocation -> OutOfMemory");
    ie_b200::set_device_alloc(nullptr);
    st = (*op)->forward({&x.t, &w.t}, outs, ctx);
    expect(st.has_value() && y.buffer != nullptr, "forward after the allocator recovers");
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
  // a fused Conv + BatchNorm + Relu node from the fusion pass, run by the
  // CUDA op with the folded constants and the activation attribute
  {
    auto bg = make_bn_graph(false);
    HostTensor x({2, 8, 11, 9}, ie::DType::F32);
    Lcg rng(22);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-1.f, 1.f);
    std::vector<ie::Tensor> orig;
    for (const char* k : {"w", "b", "bn_scale", "bn_bias", "bn_mean", "bn_var"}) {
      orig.push_back(bg->g.weights.at(k));
    }
    ie_b200::ConvBnReluFusionPass pass;
    ie::PassContext pctx;
    expect(pass.run(bg->g, pctx).has_value() && bg->g.nodes.size() == 1, "PASS: fuse");
    const ie::Node& n = bg->g.nodes[0];
    auto op = reg.create(n.op);
    if (!op.has_value()) return 3;
    expect((*op)->configure(n.attrs).has_value(), "PASS: configure fused conv");
    ie::Tensor* wf = &bg->g.weights.at(bg->g.find_value(n.inputs[1])->name);
    ie::Tensor* bf = &bg->g.weights.at(bg->g.find_value(n.inputs[2])->name);
    ie::Tensor y;
    std::vector<ie::Tensor*> outs{&y};
    const ie::Status st = (*op)->forward({&x.t, wf, bf}, outs, ctx);
    expect(st.has_value(), "PASS: fused conv forward");
    if (!st.has_value()) return 4;
    dump(dir, manifest, "bn_x", x.t);
    const char* names[] = {"bn_w", "bn_b", "bn_scale", "bn_bias", "bn_mean", "bn_var"};
    for (size_t i = 0; i < orig.size(); ++i) dump(dir, manifest, names[i], orig[i]);
    dump(dir, manifest, "bn_wf", *wf);
    dump(dir, manifest, "bn_bf", *bf);
    dump(dir, manifest, "bn_y", y);
  }
  // the ResNet-shaped graph: fusion pass, then the device-resident executor
  {
    auto ng = make_net_graph();
    ie::Graph& g = ng->g;
    ie_b200::ConvBnReluFusionPass pass;
    ie::PassContext pctx;
    expect(pass.run(g, pctx).has_value() && pass.folded_batch_norms() == 2 &&
               pass.fused_adds() == 1 && pass.fused_activations() == 2 && g.nodes.size() == 6,
           "EXEC: graph fused to 6 nodes");
    HostTensor x({2, 3, 32, 32}, ie::DType::F32);
    Lcg rng(32);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-1.f, 1.f);
    ie_b200::CudaExecutor exec(reg);
    std::unordered_map<std::string, ie::Tensor> in{{"x", x.t}};
    auto r1 = exec.run(g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(r1.has_value() && r1->size() == 1, "EXEC: run");
    if (!r1.has_value()) {
      std::printf("  %s\n", r1.error().message.c_str());
      return 4;
    }
    auto r2 = exec.run(g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(r2.has_value() && std::memcmp((*r1)[0].buffer, (*r2)[0].buffer, (*r1)[0].bytes()) == 0,
           "EXEC: second run (cached weights) identical");
    expect((*r1)[0].shape.dims == std::vector<int64_t>{2, 10} && (*r1)[0].device == ie::Device::CPU,
           "EXEC: host output [2, 10]");
    dump(dir, manifest, "net_x", x.t);
    for (size_t i = 0; i < ng->names.size(); ++i) {
      dump(dir, manifest, ("net_" + ng->names[i]).c_str(), ng->keep[i]->t);
    }
    dump(dir, manifest, "net_y", (*r1)[0]);
    auto raw = make_net_graph();  // unfused: BatchNorm has no CUDA op
    ie_b200::CudaExecutor exec2(reg);
    auto bad = exec2.run(raw->g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(!bad.has_value() && bad.error().code == Error::Code::Unsupported,
           "EXEC: unfused graph is Unsupported");
  }
  // the int8 bottleneck, device-resident through the executor (int8 values
  // stay in the NHWC activation layout between nodes)
  {
    auto qg = make_q8_block_graph();
    HostTensor x({2, 32, 14, 14}, ie::DType::U8);
    Lcg rng(43);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<uint8_t>()[i] = static_cast<uint8_t>(rng.next() % 256);
    ie_b200::CudaExecutor exec(reg);
    std::unordered_map<std::string, ie::Tensor> in{{"x", x.t}};
    auto r1 = exec.run(qg->g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(r1.has_value() && r1->size() == 1, "Q8EXEC: run");
    if (!r1.has_value()) {
      std::printf("  %s\n", r1.error().message.c_str());
      return 4;
    }
    auto r2 = exec.run(qg->g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(r2.has_value() && std::memcmp((*r1)[0].buffer, (*r2)[0].buffer, (*r1)[0].bytes()) == 0,
           "Q8EXEC: second run identical");
    expect((*r1)[0].shape.dims == std::vector<int64_t>{2, 32, 7, 7} &&
               (*r1)[0].dtype == ie::DType::U8 && (*r1)[0].device == ie::Device::CPU,
           "Q8EXEC: host NCHW uint8 output");
    dump(dir, manifest, "q8g_x", x.t);
    for (const char* k : {"qw1", "qw2", "qw3"}) dump(dir, manifest, (std::string("q8g_") + k).c_str(), qg->g.weights.at(k));
    for (size_t l = 0; l < 3; ++l) {
      const int64_t m = static_cast<int64_t>(qg->mult[l].size());
      HostTensor mt({m}, ie::DType::F32), bt({m}, ie::DType::F32);
      for (int64_t i = 0; i < m; ++i) {
        mt.data<float>()[i] = static_cast<float>(qg->mult[l][static_cast<size_t>(i)]);
        bt.data<float>()[i] = static_cast<float>(qg->bias[l][static_cast<size_t>(i)]);
      }
      dump(dir, manifest, ("q8g_mult" + std::to_string(l + 1)).c_str(), mt.t);
      dump(dir, manifest, ("q8g_bias" + std::to_string(l + 1)).c_str(), bt.t);
    }
    dump(dir, manifest, "q8g_y", (*r1)[0]);
  }
  // a whole quantized network through CudaExecutor: int8 from the stem to the
  // GlobalAvgPool, fp32 logits from the Gemm
  {
    auto qn = make_q8_net_graph();
    HostTensor x({2, 3, 32, 32}, ie::DType::U8);
    Lcg rng(59);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<uint8_t>()[i] = static_cast<uint8_t>(rng.next() % 256);
    ie_b200::CudaExecutor exec(reg);
    std::unordered_map<std::string, ie::Tensor> in{{"x", x.t}};
    auto r = exec.run(qn->g, in, std::make_shared<ie::MallocAllocator>(), stream);
    expect(r.has_value() && r->size() == 1, "Q8NET: run");
    if (!r.has_value()) {
      std::printf("  %s\n", r.error().message.c_str());
      return 4;
    }
    expect((*r)[0].shape.dims == std::vector<int64_t>{2, 10} && (*r)[0].dtype == ie::DType::F32,
           "Q8NET: fp32 logits [2, 10]");
    dump(dir, manifest, "q8n_x", x.t);
    for (const char* k : {"nw0", "nw1", "nw2", "nw3", "nfcw", "nfcb"}) {
      dump(dir, manifest, (std::string("q8n_") + k).c_str(), qn->g.weights.at(k));
    }
    for (size_t l = 0; l < 4; ++l) {
      const int64_t m = static_cast<int64_t>(qn->mult[l].size());
      HostTensor mt({m}, ie::DType::F32), bt({m}, ie::DType::F32);
      for (int64_t i = 0; i < m; ++i) {
        mt.data<float>()[i] = static_cast<float>(qn->mult[l][static_cast<size_t>(i)]);
        bt.data<float>()[i] = static_cast<float>(qn->bias[l][static_cast<size_t>(i)]);
      }
      dump(dir, manifest, ("q8n_mult" + std::to_string(l)).c_str(), mt.t);
      dump(dir, manifest, ("q8n_bias" + std::to_string(l)).c_str(), bt.t);
    }
    dump(dir, manifest, "q8n_y", (*r)[0]);
  }
  // conv + BN + shortcut add + Relu fused, run with a residual input
  {
    auto bg = make_bn_graph(false, true);
    HostTensor x({2, 8, 11, 9}, ie::DType::F32), r({2, 12, 11, 9}, ie::DType::F32);
    Lcg rng(23);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-1.f, 1.f);
    for (int64_t i = 0; i < r.t.numel(); ++i) r.data<float>()[i] = rng.uniform(-1.f, 1.f);
    std::vector<ie::Tensor> orig;
    for (const char* k : {"w", "b", "bn_scale", "bn_bias", "bn_mean", "bn_var"}) {
      orig.push_back(bg->g.weights.at(k));
    }
    ie_b200::ConvBnReluFusionPass pass;
    ie::PassContext pctx;
    expect(pass.run(bg->g, pctx).has_value() && bg->g.nodes.size() == 1, "ADD: fuse");
    const ie::Node& n = bg->g.nodes[0];
    auto op = reg.create(n.op);
    if (!op.has_value()) return 3;
    expect((*op)->configure(n.attrs).has_value(), "ADD: configure fused conv");
    ie::Tensor* wf = &bg->g.weights.at(bg->g.find_value(n.inputs[1])->name);
    ie::Tensor* bf = &bg->g.weights.at(bg->g.find_value(n.inputs[2])->name);
    ie::Tensor y;
    std::vector<ie::Tensor*> outs{&y};
    const ie::Status st = (*op)->forward({&x.t, wf, bf, &r.t}, outs, ctx);
    expect(st.has_value(), "ADD: fused conv forward");
    if (!st.has_value()) {
      std::printf("  %s\n", st.error().message.c_str());
      return 4;
    }
    dump(dir, manifest, "add_x", x.t);
    dump(dir, manifest, "add_r", r.t);
    const char* names[] = {"add_w", "add_b", "add_scale", "add_bias", "add_mean", "add_var"};
    for (size_t i = 0; i < orig.size(); ++i) dump(dir, manifest, names[i], orig[i]);
    dump(dir, manifest, "add_y", y);
  }
  // the head of a ResNet through the registry: max pool, average pool,
  // global average pool, Gemm (FC with bias)
  {
    Lcg rng(5);
    HostTensor x({2, 16, 15, 13}, ie::DType::F32);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-2.f, 2.f);
    auto mp = reg.create(ie::OpType::MaxPool2D);
    auto ap = reg.create(ie::OpType::AvgPool2D);
    auto gp = reg.create(ie::OpType::GlobalAvgPool);
    auto gm = reg.create(ie::OpType::Gemm);
    if (!mp.has_value() || !ap.has_value() || !gp.has_value() || !gm.has_value()) return 3;
    (*mp)->configure({{"kernel_shape", std::vector<int64_t>{3, 3}},
                      {"strides", std::vector<int64_t>{2, 2}},
                      {"pads", std::vector<int64_t>{1, 1, 1, 1}}});
    (*ap)->configure({{"kernel_shape", std::vector<int64_t>{3, 3}},
                      {"strides", std::vector<int64_t>{2, 2}},
                      {"pads", std::vector<int64_t>{1, 1, 1, 1}},
                      {"ceil_mode", int64_t{1}},
                      {"count_include_pad", int64_t{1}}});
    (*gm)->configure({{"transB", int64_t{1}}});
    ie::Tensor ym, ya, yg, yf;
    std::vector<ie::Tensor*> om{&ym}, oa{&ya}, og{&yg}, of{&yf};
    expect((*mp)->forward({&x.t}, om, ctx).has_value(), "MaxPool2D forward");
    expect((*ap)->forward({&x.t}, oa, ctx).has_value(), "AvgPool2D forward");
    expect((*gp)->forward({&x.t}, og, ctx).has_value(), "GlobalAvgPool forward");
    HostTensor feat({2, 16}, ie::DType::F32), wfc({10, 16}, ie::DType::F32), bfc({10}, ie::DType::F32);
    if (yg.buffer != nullptr) std::memcpy(feat.storage.data(), yg.buffer, feat.t.bytes());
    for (int64_t i = 0; i < wfc.t.numel(); ++i) wfc.data<float>()[i] = rng.uniform(-0.5f, 0.5f);
    for (int64_t i = 0; i < 10; ++i) bfc.data<float>()[i] = rng.uniform(-0.1f, 0.1f);
    const ie::Status gst = (*gm)->forward({&feat.t, &wfc.t, &bfc.t}, of, ctx);
    expect(gst.has_value(), "Gemm forward");
    if (!gst.has_value()) std::printf("  %s\n", gst.error().message.c_str());
    if (ym.buffer == nullptr || ya.buffer == nullptr || yg.buffer == nullptr || yf.buffer == nullptr) {
      return 4;
    }
    dump(dir, manifest, "head_x", x.t);
    dump(dir, manifest, "head_max", ym);
    dump(dir, manifest, "head_avg", ya);
    dump(dir, manifest, "head_gap", yg);
    dump(dir, manifest, "head_wfc", wfc.t);
    dump(dir, manifest, "head_bfc", bfc.t);
    dump(dir, manifest, "head_fc", yf);
    // int8 MaxPool2D on a host NCHW tensor: rectangular kernel, asymmetric
    // pads, ceil_mode, a channel count that is not a multiple of 16
    HostTensor xq({2, 5, 13, 11}, ie::DType::I8);
    for (int64_t i = 0; i < xq.t.numel(); ++i) {
      xq.data<int8_t>()[i] = static_cast<int8_t>(static_cast<int32_t>(rng.next() % 256) - 128);
    }
    auto mq = reg.create(ie::OpType::MaxPool2D);
    auto aq = reg.create(ie::OpType::AvgPool2D);
    if (!mq.has_value() || !aq.has_value()) return 3;
    (*mq)->configure({{"kernel_shape", std::vector<int64_t>{2, 3}},
                      {"strides", std::vector<int64_t>{2, 1}},
                      {"pads", std::vector<int64_t>{0, 1, 1, 0}},
                      {"ceil_mode", int64_t{1}}});
    (*aq)->configure({{"kernel_shape", std::vector<int64_t>{2, 2}}});
    ie::Tensor yq, yqa;
    std::vector<ie::Tensor*> oq{&yq}, oqa{&yqa};
    const ie::Status qst = (*mq)->forward({&xq.t}, oq, ctx);
    expect(qst.has_value() && yq.dtype == ie::DType::I8 && yq.device == ie::Device::CPU,
           "int8 MaxPool2D forward");
    if (!qst.has_value()) std::printf("  %s\n", qst.error().message.c_str());
    const ie::Status ast = (*aq)->forward({&xq.t}, oqa, ctx);
    expect(!ast.has_value() && ast.error().code == ie::Error::Code::Unsupported,
           "int8 AvgPool2D is Unsupported");
    if (yq.buffer == nullptr) return 4;
    dump(dir, manifest, "head_q8x", xq.t);
    dump(dir, manifest, "head_q8max", yq);
  }
  // int8 post-training quantization of an fp32 Conv2D + ReLU: calibrate the
  // input and output ranges on the fp32 op, quantize, run the int8 op with
  // the emitted attributes, dequantize.  The input range [-0.3, 1.0] is not
  // symmetric about 0, so the calibrated activation zero point (about 59) is
  // neither 0 nor 128 and the dense int8 kernel runs on its haloed input.
  {
    Lcg rng(4);
    const int64_t n = 2, c = 32, h = 20, w = 20, m = 48;
    HostTensor x({n, c, h, w}, ie::DType::F32), wt({m, c, 3, 3}, ie::DType::F32),
        b({m}, ie::DType::F32);
    for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-0.3f, 1.f);
    for (int64_t i = 0; i < wt.t.numel(); ++i) wt.data<float>()[i] = rng.uniform(-0.1f, 0.1f);
    for (int64_t i = 0; i < m; ++i) b.data<float>()[i] = rng.uniform(-0.05f, 0.05f);
    const ie::Attrs conv_attrs{{"pads", std::vector<int64_t>{1, 1, 1, 1}}};
    ie_b200::CudaConv2DOp fp;
    fp.configure(conv_attrs);
    ie::Tensor yf;
    std::vector<ie::Tensor*> outs{&yf};
    ie::Status st = fp.forward({&x.t, &wt.t, &b.t}, outs, ctx);
    expect(st.has_value(), "PTQ: fp32 forward");
    if (!st.has_value()) return 4;
    for (int64_t i = 0; i < yf.numel(); ++i) {
      yf.data<float>()[i] = std::max(yf.data<float>()[i], 0.0f);  // the ReLU node
    }
    ie_b200::ActivationCalibrator cal_x, cal_y;
    expect(cal_x.observe(x.t).has_value() && cal_y.observe(yf).has_value(), "PTQ: calibrate");
    ie_b200::Int8QuantPlugin plug;
    auto xp = cal_x.params(), yp = cal_y.params();
    auto wq = plug.quantize(wt.t, ie::QuantConfig{});
    auto xq = plug.quantize_with(x.t, *xp);
    expect(xp.has_value() && yp.has_value() && wq.has_value() && xq.has_value(),
           "PTQ: quantize weights and input");
    if (!wq.has_value() || !xq.has_value()) return 4;
    auto attrs = ie_b200::make_qlinear_conv_attrs(conv_attrs, *xp, *plug.params(*wq), *yp, m,
                                                  b.data<float>(), ie_b200::FusedActivation::Relu);
    expect(attrs.has_value(), "PTQ: qlinear attrs");
    if (!attrs.has_value()) return 4;
    ie_b200::CudaQLinearConv2DOp qop;
    expect(qop.configure(*attrs).has_value(), "PTQ: QLinearConv2D configure");
    ie::Tensor yq;
    std::vector<ie::Tensor*> qouts{&yq};
    st = qop.forward({&*xq, &*wq}, qouts, ctx);
    expect(st.has_value(), "PTQ: QLinearConv2D forward");
    if (!st.has_value()) return 4;
    auto ydq = plug.dequantize_with(yq, *yp);
    expect(ydq.has_value(), "PTQ: dequantize output");
    if (!ydq.has_value()) return 4;
    const auto& mult = std::get<std::vector<double>>(attrs->at("multiplier"));
    const auto& bias = std::get<std::vector<int64_t>>(attrs->at("bias"));
    HostTensor mt({m}, ie::DType::F32), bt({m}, ie::DType::F32), zp({3}, ie::DType::F32);
    for (int64_t i = 0; i < m; ++i) {
      mt.data<float>()[i] = static_cast<float>(mult[static_cast<size_t>(i)]);
      bt.data<float>()[i] = static_cast<float>(bias[static_cast<size_t>(i)]);  // |bias| < 2^24
    }
    zp.data<float>()[0] = static_cast<float>(xp->zero_point);
    zp.data<float>()[1] = static_cast<float>(yp->zero_point);
    zp.data<float>()[2] = static_cast<float>(std::get<int64_t>(attrs->at("qmin")));
    dump(dir, manifest, "ptq_yf", yf);
    dump(dir, manifest, "ptq_ydq", *ydq);
    dump(dir, manifest, "ptq_xq", *xq);
    dump(dir, manifest, "ptq_wq", *wq);
    dump(dir, manifest, "ptq_yq", yq);
    dump(dir, manifest, "ptq_mult", mt.t);
    dump(dir, manifest, "ptq_bias", bt.t);
    dump(dir, manifest, "ptq_zp", zp.t);
  }
  cudaStreamDestroy(stream);
  std::printf("%s (%d failures)\n", g_failures == 0 ? "PASSED" : "FAILED", g_failures);
  return g_failures == 0 ? 0 : 1;
}

// ------------------------------------------------------------ quantizer

int run_quant(const std::string& dir) {
  std::ofstream manifest(dir + "/manifest.txt");
  ie_b200::Int8QuantPlugin plug;
  Lcg rng(11);
  // weights: per-channel symmetric, one channel all zero, one with a single value
  HostTensor w({16, 8, 3, 3}, ie::DType::F32);
  for (int64_t i = 0; i < w.t.numel(); ++i) w.data<float>()[i] = rng.uniform(-0.3f, 0.3f);
  for (int64_t i = 0; i < 72; ++i) w.data<float>()[3 * 72 + i] = 0.0f;
  for (int64_t i = 0; i < 72; ++i) w.data<float>()[5 * 72 + i] = (i == 7) ? -0.02f : 0.0f;
  auto wq = plug.quantize(w.t, ie::QuantConfig{});
  // activations: asymmetric uint8 over the tensor's own range
  HostTensor x({3, 5, 7, 9}, ie::DType::F32);
  for (int64_t i = 0; i < x.t.numel(); ++i) x.data<float>()[i] = rng.uniform(-0.7f, 2.3f);
  ie::QuantConfig asym;
  asym.symmetric = false;
  auto xq = plug.quantize(x.t, asym);
  // per-tensor symmetric
  ie::QuantConfig pt;
  pt.format = "int8_per_tensor";
  auto wt = plug.quantize(w.t, pt);
  // percentile calibration over two batches
  HostTensor a1({4096}, ie::DType::F32), a2({4096}, ie::DType::F32);
  for (int64_t i = 0; i < 4096; ++i) {
    a1.data<float>()[i] = rng.uniform(0.0f, 1.0f);
    a2.data<float>()[i] = rng.uniform(-0.2f, 3.0f);
  }
  a2.data<float>()[17] = 40.0f;  // an outlier the percentile range drops
  ie_b200::ActivationCalibrator cal(99.9), mm;
  cal.observe(a1.t);
  cal.observe(a2.t);
  mm.observe(a1.t);
  mm.observe(a2.t);
  auto cp = cal.params(), mp = mm.params();
  if (!wq.has_value() || !xq.has_value() || !wt.has_value() || !cp.has_value() || !mp.has_value()) {
    std::printf("FAILED: quantize\n");
    return 1;
  }
  // layer attributes from those parameters (bias small enough to be exact in fp32)
  HostTensor bias({16}, ie::DType::F32);
  for (int64_t i = 0; i < 16; ++i) bias.data<float>()[i] = rng.uniform(-0.02f, 0.02f);
  const ie_b200::QuantParams yq = ie_b200::u8_params_for_range(0.0f, 4.0f);
  auto attrs = ie_b200::make_qlinear_conv_attrs({}, *plug.params(*xq), *plug.params(*wq), yq, 16,
                                                bias.data<float>(),
                                                ie_b200::FusedActivation::Relu6);
  if (!attrs.has_value()) {
    std::printf("FAILED: attrs %s\n", attrs.error().message.c_str());
    return 1;
  }
  HostTensor ws({16}, ie::DType::F32), xs({2}, ie::DType::F32), wts({1}, ie::DType::F32),
      cal_t({6}, ie::DType::F32), mt({16}, ie::DType::F32), bt({16}, ie::DType::F32),
      qclamp({3}, ie::DType::F32);
  for (int i = 0; i < 16; ++i) ws.data<float>()[i] = plug.params(*wq)->scales[i];
  xs.data<float>()[0] = plug.params(*xq)->scales[0];
  xs.data<float>()[1] = static_cast<float>(plug.params(*xq)->zero_point);
  wts.data<float>()[0] = plug.params(*wt)->scales[0];
  cal_t.data<float>()[0] = cp->scales[0];
  cal_t.data<float>()[1] = static_cast<float>(cp->zero_point);
  cal_t.data<float>()[2] = mp->scales[0];
  cal_t.data<float>()[3] = static_cast<float>(mp->zero_point);
  cal_t.data<float>()[4] = mm.lo();
  cal_t.data<float>()[5] = mm.hi();
  const auto& mult = std::get<std::vector<double>>(attrs->at("multiplier"));
  const auto& bq = std::get<std::vector<int64_t>>(attrs->at("bias"));
  for (int i = 0; i < 16; ++i) {
    mt.data<float>()[i] = static_cast<float>(mult[i]);
    bt.data<float>()[i] = static_cast<float>(bq[i]);
  }
  qclamp.data<float>()[0] = static_cast<float>(std::get<int64_t>(attrs->at("qmin")));
  qclamp.data<float>()[1] = static_cast<float>(std::get<int64_t>(attrs->at("qmax")));
  qclamp.data<float>()[2] = static_cast<float>(std::get<int64_t>(attrs->at("y_zero_point")));
  dump(dir, manifest, "w", w.t);
  dump(dir, manifest, "wq", *wq);
  dump(dir, manifest, "w_scales", ws.t);
  dump(dir, manifest, "x", x.t);
  dump(dir, manifest, "xq", *xq);
  dump(dir, manifest, "x_params", xs.t);
  dump(dir, manifest, "wt", *wt);
  dump(dir, manifest, "wt_scale", wts.t);
  dump(dir, manifest, "a1", a1.t);
  dump(dir, manifest, "a2", a2.t);
  dump(dir, manifest, "cal", cal_t.t);
  dump(dir, manifest, "bias", bias.t);
  dump(dir, manifest, "mult", mt.t);
  dump(dir, manifest, "bias_q", bt.t);
  dump(dir, manifest, "clamp", qclamp.t);
  auto wdq = plug.dequantize(*wq, ie::QuantConfig{});
  auto xdq = plug.dequantize(*xq, asym);
  if (!wdq.has_value() || !xdq.has_value()) {
    std::printf("FAILED: dequantize\n");
    return 1;
  }
  dump(dir, manifest, "wdq", *wdq);
  dump(dir, manifest, "xdq", *xdq);
  std::printf("PASSED\n");
  return 0;
}

// The int8 ResNet-50 graph through CudaExecutor::run with host tensors in and
// out (the call an engine makes per batch): per run the upload of the uint8
// NCHW batch, 53 convolutions, the max pool, 16 int8 Adds, the int8 GAP, the
// FC and the download of the logits, then one synchronize.  Times `iters`
// runs after `warmup` with the host clock around the synchronous calls and
// prints one JSON line.  Check: image 0 alone through the same executor gives
// the batch's first row of logits (the int8 stages do not depend on the batch;
// the FC may split K by batch size, so within 1e-5 of max|y|).
int run_engine_bench(int64_t batch, int iters, int warmup) {
  if (batch < 1 || iters < 1 || warmup < 0) return 2;
  cudaStream_t stream;
  if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) return 3;
  ie::OpRegistry reg;
  if (!ie_b200::register_cuda_ops(reg).has_value()) return 2;
  auto qg = make_resnet50_q8_graph();
  auto pinned = std::make_shared<PinnedAllocator>();
  auto x = ie::Tensor::allocate(ie::Shape{{batch, 3, 224, 224}}, ie::DType::U8, pinned);
  auto x1 = ie::Tensor::allocate(ie::Shape{{1, 3, 224, 224}}, ie::DType::U8, pinned);
  if (!x.has_value() || !x1.has_value()) return 3;
  Lcg rng(224);
  for (int64_t i = 0; i < x->numel(); ++i) x->data<uint8_t>()[i] = static_cast<uint8_t>(rng.next() >> 8);
  std::memcpy(x1->buffer, x->buffer, x1->bytes());
  ie_b200::CudaExecutor exec(reg);
  auto run = [&](const ie::Tensor& in) {
    std::unordered_map<std::string, ie::Tensor> inputs{{"x", in}};
    return exec.run(qg->g, inputs, pinned, stream);
  };
  auto fail = [](const ie::Error& e) {
    std::printf("{\"error\": \"%s\"}\n", e.message.c_str());
    return 4;
  };
  for (int i = 0; i < warmup; ++i) {
    auto r = run(*x);
    if (!r.has_value()) return fail(r.error());
  }
  ie_cuda_launch_count(1);
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<ie::Tensor> last;
  for (int i = 0; i < iters; ++i) {
    auto r = run(*x);
    if (!r.has_value()) return fail(r.error());
    last = std::move(*r);
  }
  const auto t1 = std::chrono::steady_clock::now();
  const uint64_t launches = ie_cuda_launch_count(0);
  const std::size_t reserved = exec.reserved_device_bytes();
  auto one = run(*x1);
  if (!one.has_value()) return fail(one.error());
  const float* yb = static_cast<const float*>(last[0].buffer);
  const float* y1 = static_cast<const float*>((*one)[0].buffer);
  double ymax = 0.0, dmax = 0.0;
  for (int64_t j = 0; j < 1000; ++j) {
    ymax = std::max(ymax, std::fabs(static_cast<double>(yb[j])));
    dmax = std::max(dmax, std::fabs(static_cast<double>(yb[j]) - y1[j]));
  }
  const bool ok = dmax <= 1e-5 * ymax;
  const double ms = std::chrono::duration<double, std::milli>(t1 - t0).count() / iters;
  const double conv_ops_img = 8.174e9;  // 2 x MACs of the 53 convolutions per image
  std::printf("{\"batch\": %lld, \"iters\": %d, \"warmup\": %d, \"ms_per_run\": %.4f, "
              "\"images_per_s\": %.1f, \"conv_tops\": %.2f, \"nodes\": %zu, "
              "\"launches_per_run\": %.1f, \"h2d_bytes_per_run\": %zu, \"d2h_bytes_per_run\": %zu, "
              "\"device_pool_reserved_bytes\": %zu, \"max_abs_logit\": %.6g, "
              "\"batch1_max_abs_diff\": %.6g, \"batch1_ok\": %s}\n",
              static_cast<long long>(batch), iters, warmup, ms, batch / (ms / 1e3),
              conv_ops_img * batch / (ms / 1e3) / 1e12, qg->g.nodes.size(),
              static_cast<double>(launches) / iters, x->bytes(), last[0].bytes(), reserved, ymax, dmax,
              ok ? "true" : "false");
  std::fflush(stdout);
  cudaStreamDestroy(stream);
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 5 && std::strcmp(argv[1], "engine-bench") == 0) {
    return run_engine_bench(std::atoll(argv[2]), std::atoi(argv[3]), std::atoi(argv[4]));
  }
  if (argc >= 2 && std::strcmp(argv[1], "cpu") == 0) return run_cpu();
  if (argc >= 3 && std::strcmp(argv[1], "gpu") == 0) return run_gpu(argv[2]);
  if (argc >= 3 && std::strcmp(argv[1], "quant") == 0) return run_quant(argv[2]);
  std::fprintf(stderr, "usage: %s cpu | gpu <outdir> | quant <outdir> | engine-bench <batch> <iters> <warmup>\n",
               argv[0]);
  return 2;
}
