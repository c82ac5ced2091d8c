// Test harness (test infrastructure, not shipped): the CUDA backend running
// under the reference engine's own runtime.  Built by `make -C oracle
// ref-engine` from the reference's sources where they lie (Engine, Executor,
// OpRegistry, BackendRegistry, the CPU backend and ops, the ONNX loader) plus
// this package's backend sources compiled against the reference headers
// (IE_B200_REFERENCE_HEADERS), linked with libie_cuda_conv.so.
//
//   ref_engine_harness cpu  <model.onnx>
//       no GPU needed: registers the CUDA backend in the reference
//       BackendRegistry (a second registration is AlreadyExists), creates it
//       through the registry, and on a machine without a CUDA device checks
//       that init() fails with Runtime (no CPU fallback).
//   ref_engine_harness gpu  <model.onnx> <input.f32>
//       runs the model (tiny_cnn.onnx from the reference's tests) on the
//       reference Engine (CPU backend) and on the CUDA backend through
//       BackendEngine (EngineConfig::gpu_backend = CUDA) and
//       CudaTraditionalEngine (infer and batched infer_batch), and prints one
//       JSON line with every result for the test to compare.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

#include "core/backend/backend_registry.h"
#include "core/memory/malloc_allocator.h"
#include "core/runtime/engine.h"
#include "cuda_backend.h"
#include "models/traditional/onnx/onnx_loader.h"

namespace {

int g_fail = 0;

void check(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAIL: %s\n", what);
    ++g_fail;
  }
}

std::string json_floats(const ie::Tensor& t) {
  std::string s = "[";
  const float* p = t.data<float>();
  for (int64_t i = 0; i < t.numel(); ++i) {
    char buf[32];
    std::snprintf(buf, sizeof(buf), "%s%.9g", i ? "," : "", static_cast<double>(p[i]));
    s += buf;
  }
  return s + "]";
}

ie::Tensor make_input(const std::vector<float>& v, float scale) {
  auto alloc = std::make_shared<ie::MallocAllocator>();
  auto t = ie::Tensor::allocate(ie::Shape{{1, 3, 8, 8}}, ie::DType::F32, alloc);
  for (size_t i = 0; i < v.size(); ++i) t->data<float>()[i] = v[i] * scale;
  return std::move(*t);
}

int run_cpu(const std::string& model) {
  auto& reg = ie::BackendRegistry::instance();
  check(ie_b200::register_cuda_backend(reg).has_value(), "register CUDA backend");
  auto again = ie_b200::register_cuda_backend(reg);
  check(!again.has_value() && again.error().code == ie::Error::Code::AlreadyExists,
        "second registration is AlreadyExists");
  check(reg.contains(ie::BackendKind::CUDA), "registry lists CUDA");
  auto be = reg.create(ie::BackendKind::CUDA);
  check(be.has_value() && (*be)->device() == ie::Device::CUDA, "create CUDA backend");
  check(be.has_value() && (*be)->meta().name == "cuda", "backend meta");
  int count = 0;
  const bool has_gpu = cudaGetDeviceCount(&count) == cudaSuccess && count > 0;
  cudaGetLastError();
  if (be.has_value() && !has_gpu) {
    auto st = (*be)->init();
    check(!st.has_value() && st.error().code == ie::Error::Code::Runtime,
          "init without a device is Runtime");
    ie::EngineConfig cfg;
    cfg.gpu_backend = ie::GpuBackend::CUDA;
    ie_b200::BackendEngine eng(cfg);
    auto g = ie::load_onnx_model(model);
    check(g.has_value(), "reference ONNX loader reads the model");
    if (g.has_value()) {
      auto st2 = eng.load(*g);
      check(!st2.has_value() && st2.error().code == ie::Error::Code::Runtime,
            "engine on the CUDA backend reports the missing device");
    }
  }
  ie_b200::CudaTraditionalEngine te;
  auto st = te.load_model(model, ie::ModelFormat::TFLITE);
  check(!st.has_value() && st.error().code == ie::Error::Code::Unsupported,
        "non-ONNX format is Unsupported");
  std::printf("%s (%d failures)\n", g_fail == 0 ? "PASSED" : "FAILED", g_fail);
  return g_fail == 0 ? 0 : 1;
}

int run_gpu(const std::string& model, const std::string& input_path) {
  std::ifstream f(input_path, std::ios::binary);
  std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (raw.size() != 192 * sizeof(float)) {
    std::fprintf(stderr, "input must hold 192 floats\n");
    return 2;
  }
  std::vector<float> in(192);
  std::memcpy(in.data(), raw.data(), raw.size());
  auto graph = ie::load_onnx_model(model);
  if (!graph.has_value()) {
    std::fprintf(stderr, "load: %s\n", graph.error().message.c_str());
    return 2;
  }
  std::string name;
  for (const ie::Value& v : graph->values) {
    if (v.is_input) name = v.name;
  }
  // the reference engine, CPU backend
  ie::Engine ref(ie::EngineConfig{});
  check(ref.load(*graph).has_value(), "reference Engine load");
  auto ycpu = ref.infer({{name, make_input(in, 1.0f)}});
  check(ycpu.has_value() && !ycpu->empty(), "reference Engine infer");
  // the CUDA backend through the registry, selected by EngineConfig
  check(ie_b200::register_cuda_backend().has_value(), "register CUDA backend");
  ie::EngineConfig cfg;
  cfg.gpu_backend = ie::GpuBackend::CUDA;
  ie_b200::BackendEngine eng(cfg);
  auto lst = eng.load(*graph);
  check(lst.has_value(), "BackendEngine load");
  if (!lst.has_value()) std::fprintf(stderr, "  %s\n", lst.error().message.c_str());
  auto* cb = dynamic_cast<ie_b200::CudaBackend*>(eng.backend());
  check(cb != nullptr, "the engine runs the CUDA backend");
  auto ycuda = eng.infer({{name, make_input(in, 1.0f)}});
  check(ycuda.has_value() && !ycuda->empty(), "BackendEngine infer");
  if (!ycuda.has_value()) std::fprintf(stderr, "  %s\n", ycuda.error().message.c_str());
  auto ycuda2 = eng.infer({{name, make_input(in, 1.0f)}});
  check(ycuda2.has_value() && !ycuda2->empty(), "BackendEngine second infer");
  // TraditionalEngine on CUDA: single and batched
  ie_b200::CudaTraditionalEngine te;
  check(te.load_model(model, ie::ModelFormat::ONNX).has_value(), "CudaTraditionalEngine load");
  auto y1 = te.infer({make_input(in, 1.0f)});
  auto y2 = te.infer({make_input(in, 0.5f)});
  auto yb = te.infer_batch({{make_input(in, 1.0f)}, {make_input(in, 0.5f)}});
  check(y1.has_value() && y2.has_value() && yb.has_value() && yb->size() == 2,
        "CudaTraditionalEngine infer / infer_batch");
  auto none = te.infer({});
  check(!none.has_value() && none.error().code == ie::Error::Code::InvalidArgument,
        "wrong input count is InvalidArgument");
  auto empty = te.infer_batch({});
  check(empty.has_value() && empty->empty(), "empty batch");
  if (g_fail != 0) {
    std::printf("FAILED (%d failures)\n", g_fail);
    return 1;
  }
  std::printf("{\"cpu\": %s, \"cuda\": %s, \"cuda_again\": %s, \"single0\": %s, \"single1\": %s, "
              "\"batch0\": %s, \"batch1\": %s, \"folded_bn\": %d, \"fused_act\": %d}\n",
              json_floats(ycpu->front()).c_str(), json_floats(ycuda->front()).c_str(),
              json_floats(ycuda2->front()).c_str(), json_floats(*y1).c_str(),
              json_floats(*y2).c_str(), json_floats((*yb)[0]).c_str(),
              json_floats((*yb)[1]).c_str(), cb->folded_batch_norms(), cb->fused_activations());
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 3 && std::strcmp(argv[1], "cpu") == 0) return run_cpu(argv[2]);
  if (argc >= 4 && std::strcmp(argv[1], "gpu") == 0) return run_gpu(argv[2], argv[3]);
  std::fprintf(stderr, "usage: %s cpu <model.onnx> | gpu <model.onnx> <input.f32>\n", argv[0]);
  return 2;
}
