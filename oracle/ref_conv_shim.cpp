// C entry points around the reference engine's own Conv2DOp, compiled from
// the reference sources by oracle/Makefile into oracle/_ref/libref_conv.so.
// TEST INFRASTRUCTURE ONLY: the tests and the CPU-baseline leg of the
// benchmark call it as the checker and as the timed reference CPU conv.
//
// The op runs exactly as the reference's Executor would drive it
// (src/core/runtime/executor.cpp:54-83): configure(attrs) then
// forward({x, w[, b]}, {out}, ctx), with ctx.kernels->matmul_row set to the
// widest row kernel this CPU supports, the same preference order as
// CpuKernelCatalog::select (src/backends/cpu/kernels/cpu_kernel_catalog.cpp:
// 50-86): AVX-512, then AVX2, then SSE2, then scalar.

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "backends/cpu/simd/simd_kernels.h"
#include "core/memory/malloc_allocator.h"
#include "core/ops/kernel_fns.h"
#include "ops/traditional/conv2d_op.h"
#include "ops/traditional/gemm_op.h"
#include "ops/traditional/pool_ops.h"

namespace {

ie::KernelFns select_kernels(int* which) {
    ie::KernelFns fns;
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
        __builtin_cpu_supports("avx512vl")) {
        fns.matmul_row = ie::cpu::matmul_row_avx512;
        *which = 3;
    } else if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) {
        fns.matmul_row = ie::cpu::matmul_row_avx2;
        *which = 2;
    } else if (__builtin_cpu_supports("sse2")) {
        fns.matmul_row = ie::cpu::matmul_row_sse2;
        *which = 1;
    } else {
        fns.matmul_row = ie::cpu::matmul_row_scalar;
        *which = 0;
    }
    return fns;
}

int code_of(const ie::Error& e) {
    return 1 + static_cast<int>(e.code);  // InvalidArgument -> 1, ...
}

// The op's output dims differ from the dims the caller sized y by (not a
// reference error code: those are 1 + Error::Code, all below 100).
constexpr int kShapeMismatch = 100;

ie::Tensor host_tensor(std::vector<int64_t> dims, const float* data,
                       const std::shared_ptr<ie::Allocator>& alloc) {
    auto t = ie::Tensor::allocate(ie::Shape{dims}, ie::DType::F32, alloc);
    if (!t.has_value()) return {};
    std::memcpy(t->data<float>(), data, t->bytes());
    return std::move(*t);
}

struct RunArgs {
    const float* x;
    int64_t n, c, h, w;
    const float* wt;
    int64_t m, cg, kh, kw;
    const float* bias;
    const int64_t* strides;
    const int64_t* dilations;
    const int64_t* pads;
    int64_t group;
    int auto_pad;
    int depthwise;
    int kernel_choice;
    float* y;
    int64_t* out_dims;
};

int run_one(const RunArgs& a, int64_t first, int64_t count) {
    ie::Attrs attrs;
    attrs["strides"] = std::vector<int64_t>{a.strides[0], a.strides[1]};
    attrs["dilations"] = std::vector<int64_t>{a.dilations[0], a.dilations[1]};
    attrs["pads"] = std::vector<int64_t>{a.pads[0], a.pads[1], a.pads[2], a.pads[3]};
    attrs["group"] = a.group;
    static const char* kAuto[] = {"NOTSET", "VALID", "SAME_UPPER", "SAME_LOWER"};
    if (a.auto_pad > 0 && a.auto_pad < 4) attrs["auto_pad"] = std::string(kAuto[a.auto_pad]);

    std::unique_ptr<ie::Op> op;
    if (a.depthwise) {
        op = std::make_unique<ie::DepthwiseConv2DOp>();
    } else {
        op = std::make_unique<ie::Conv2DOp>();
    }
    if (auto st = op->configure(attrs); !st.has_value()) return code_of(st.error());

    auto alloc = std::make_shared<ie::MallocAllocator>();
    const int64_t img = a.c * a.h * a.w;
    ie::Tensor x = host_tensor({count, a.c, a.h, a.w}, a.x + first * img, alloc);
    ie::Tensor w = host_tensor({a.m, a.cg, a.kh, a.kw}, a.wt, alloc);
    ie::Tensor b;
    std::vector<ie::Tensor*> inputs{&x, &w};
    if (a.bias != nullptr) {
        b = host_tensor({a.m}, a.bias, alloc);
        inputs.push_back(&b);
    }
    std::vector<ie::Tensor> out(1);
    std::vector<ie::Tensor*> outputs{&out[0]};
    ie::ExecutionContext ctx;
    ctx.allocator = alloc;
    int which = 0;
    ie::KernelFns fns;
    if (a.kernel_choice < 0) {
        fns = select_kernels(&which);
    } else {
        const ie::KernelFns::MatMulRowFn table[] = {
            ie::cpu::matmul_row_scalar, ie::cpu::matmul_row_sse2,
            ie::cpu::matmul_row_avx2, ie::cpu::matmul_row_avx512};
        fns.matmul_row = table[a.kernel_choice & 3];
    }
    ctx.kernels = &fns;
    if (auto st = op->forward(inputs, outputs, ctx); !st.has_value()) {
        return code_of(st.error());
    }
    const auto& d = out[0].shape.dims;
    if (a.y != nullptr && a.out_dims != nullptr) {
        // y was sized from out_dims by the caller: copy only into a match.
        for (int i = 1; i < 4; ++i) {
            if (a.out_dims[i] != d[i]) return kShapeMismatch;
        }
    } else if (a.out_dims != nullptr && first == 0) {
        for (int i = 0; i < 4; ++i) a.out_dims[i] = d[i];
    }
    if (a.y != nullptr) {
        const int64_t per = d[1] * d[2] * d[3];
        std::memcpy(a.y + first * per, out[0].data<float>(),
                    static_cast<size_t>(count * per) * sizeof(float));
    }
    return 0;
}

}  // namespace

extern "C" {

// Which row kernel the catalog-equivalent selection picks on this CPU:
// 0 scalar, 1 sse2, 2 avx2, 3 avx512.
int ref_row_kernel() {
    int which = 0;
    (void)select_kernels(&which);
    return which;
}

// Runs the reference Conv2DOp (depthwise=0) or DepthwiseConv2DOp (1) on host
// fp32 NCHW buffers.  pads = {top, left, bottom, right}; auto_pad 0..3 =
// NOTSET/VALID/SAME_UPPER/SAME_LOWER; bias may be NULL; y may be NULL (shape
// query); out_dims receives [N, M, Ho, Wo].  kernel_choice -1 selects like the
// CPU catalog, 0..3 forces scalar/sse2/avx2/avx512.  nthreads > 1 runs
// independent images on separate threads, one op call per thread (the
// reference conv itself is single-threaded).  Returns 0 or 1 + the reference
// Error::Code.
int ref_conv2d_f32(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
                   const float* wt, int64_t m, int64_t cg, int64_t kh, int64_t kw,
                   const float* bias, const int64_t* strides,
                   const int64_t* dilations, const int64_t* pads, int64_t group,
                   int auto_pad, int depthwise, int kernel_choice, int nthreads,
                   float* y, int64_t* out_dims) {
    RunArgs a{x, n, c, h, w, wt, m, cg, kh, kw, bias, strides, dilations, pads,
              group, auto_pad, depthwise, kernel_choice, y, out_dims};
    if (y == nullptr && n > 1) {
        // Shape query: the output dims do not depend on the batch, so one
        // image answers it (and reports the same argument errors).
        const int rc = run_one(a, 0, 1);
        if (rc == 0 && out_dims != nullptr) out_dims[0] = n;
        return rc;
    }
    if (nthreads <= 1 || n <= 1 || y == nullptr) return run_one(a, 0, n);
    if (nthreads > n) nthreads = static_cast<int>(n);
    std::vector<int> rc(static_cast<size_t>(nthreads), 0);
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) {
        const int64_t b0 = n * t / nthreads, b1 = n * (t + 1) / nthreads;
        pool.emplace_back([&, t, b0, b1] {
            for (int64_t i = b0; i < b1 && rc[t] == 0; ++i) rc[t] = run_one(a, i, 1);
        });
    }
    for (auto& th : pool) th.join();
    for (int v : rc) {
        if (v != 0) return v;
    }
    if (out_dims != nullptr) out_dims[0] = n;
    return 0;
}

// Runs the reference MaxPool2DOp (max_pool = 1), AvgPool2DOp (0) or
// GlobalAvgPoolOp (2) on a host fp32 NCHW buffer.  pads = {top, left,
// bottom, right}; kernel / strides ignored for the global pool.  out_dims
// receives the output shape; y (may be NULL for a shape query) must hold
// y_capacity floats.  Returns 0 or 1 + the reference Error::Code, or
// kShapeMismatch when y is too small.
int ref_pool2d_f32(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int max_pool,
                   const int64_t* kernel, const int64_t* strides, const int64_t* pads,
                   int auto_pad, int ceil_mode, int count_include_pad, float* y,
                   int64_t y_capacity, int64_t* out_dims) {
    ie::Attrs attrs;
    if (max_pool != 2) {
        attrs["kernel_shape"] = std::vector<int64_t>{kernel[0], kernel[1]};
        attrs["strides"] = std::vector<int64_t>{strides[0], strides[1]};
        attrs["pads"] = std::vector<int64_t>{pads[0], pads[1], pads[2], pads[3]};
        static const char* kAuto[] = {"NOTSET", "VALID", "SAME_UPPER", "SAME_LOWER"};
        if (auto_pad > 0 && auto_pad < 4) attrs["auto_pad"] = std::string(kAuto[auto_pad]);
        attrs["ceil_mode"] = static_cast<int64_t>(ceil_mode);
        attrs["count_include_pad"] = static_cast<int64_t>(count_include_pad);
    }
    std::unique_ptr<ie::Op> op;
    if (max_pool == 1) {
        op = std::make_unique<ie::MaxPool2DOp>();
    } else if (max_pool == 0) {
        op = std::make_unique<ie::AvgPool2DOp>();
    } else {
        op = std::make_unique<ie::GlobalAvgPoolOp>();
    }
    if (auto st = op->configure(attrs); !st.has_value()) return code_of(st.error());
    auto alloc = std::make_shared<ie::MallocAllocator>();
    ie::Tensor xt = host_tensor({n, c, h, w}, x, alloc);
    std::vector<ie::Tensor> out(1);
    std::vector<ie::Tensor*> outputs{&out[0]};
    ie::ExecutionContext ctx;
    ctx.allocator = alloc;
    if (auto st = op->forward({&xt}, outputs, ctx); !st.has_value()) return code_of(st.error());
    const auto& d = out[0].shape.dims;
    for (int i = 0; i < 4; ++i) out_dims[i] = d[i];
    if (y != nullptr) {
        if (out[0].numel() > y_capacity) return kShapeMismatch;
        std::memcpy(y, out[0].data<float>(), static_cast<size_t>(out[0].numel()) * sizeof(float));
    }
    return 0;
}

// Runs the reference GemmOp: a [a0, a1], b [b0, b1], optional c with
// c_ndim (0..2) dims c_dims; y must hold y_capacity floats; out_dims gets
// [M, N].
int ref_gemm_f32(const float* a, int64_t a0, int64_t a1, const float* b, int64_t b0, int64_t b1,
                 const float* c, int c_ndim, const int64_t* c_dims, double alpha, double beta,
                 int trans_a, int trans_b, float* y, int64_t y_capacity, int64_t* out_dims) {
    ie::Attrs attrs;
    attrs["alpha"] = alpha;
    attrs["beta"] = beta;
    attrs["transA"] = static_cast<int64_t>(trans_a);
    attrs["transB"] = static_cast<int64_t>(trans_b);
    ie::GemmOp op;
    if (auto st = op.configure(attrs); !st.has_value()) return code_of(st.error());
    auto alloc = std::make_shared<ie::MallocAllocator>();
    ie::Tensor at = host_tensor({a0, a1}, a, alloc);
    ie::Tensor bt = host_tensor({b0, b1}, b, alloc);
    ie::Tensor ct;
    std::vector<ie::Tensor*> inputs{&at, &bt};
    if (c != nullptr) {
        std::vector<int64_t> dims(c_dims, c_dims + c_ndim);
        ct = host_tensor(dims, c, alloc);
        inputs.push_back(&ct);
    }
    int which = 0;
    ie::KernelFns fns = select_kernels(&which);
    std::vector<ie::Tensor> out(1);
    std::vector<ie::Tensor*> outputs{&out[0]};
    ie::ExecutionContext ctx;
    ctx.allocator = alloc;
    ctx.kernels = &fns;
    if (auto st = op.forward(inputs, outputs, ctx); !st.has_value()) return code_of(st.error());
    out_dims[0] = out[0].shape.dims[0];
    out_dims[1] = out[0].shape.dims[1];
    if (out[0].numel() > y_capacity) return kShapeMismatch;
    std::memcpy(y, out[0].data<float>(), static_cast<size_t>(out[0].numel()) * sizeof(float));
    return 0;
}

}  // extern "C"
