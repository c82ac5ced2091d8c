// Host-side helpers shared by the C ABI implementation: status plumbing, the
// per-thread error text, launch counting and TMA descriptor encoding through
// the driver entry points (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/ie_cuda_conv.h"

namespace ie_cuda {

inline thread_local std::string g_last_error;
inline thread_local uint64_t g_launches = 0;

// Stream (+1; 0 = none) whose last launch by this library packed weights.
// The implicit-GEMM kernel reads resident weights before it waits on the
// kernel launched before it (programmatic dependent launch), which is sound
// only when that kernel did not write them; a convolution launched right
// after a weight-packing launch on the same stream therefore goes without
// the overlap.  Every other launch clears the mark (check_launch).
inline std::atomic<uintptr_t> g_packed_weights_stream{0};

inline uintptr_t stream_key(cudaStream_t s) { return reinterpret_cast<uintptr_t>(s) + 1; }

inline void mark_weights_packed(cudaStream_t s) {
  g_packed_weights_stream.store(stream_key(s), std::memory_order_relaxed);
}

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

inline int check_launch(const char* what) {
  ++g_launches;
  g_packed_weights_stream.store(0, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(IE_RUNTIME, "%s: %s", what, cudaGetErrorString(e));
  }
  return IE_OK;
}

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const int*,
                                    const int*, cuuint32_t, cuuint32_t, const cuuint32_t*,
                                    CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DriverFns {
  EncodeTiledFn tiled = nullptr;
  EncodeIm2colFn im2col = nullptr;
  bool ok = false;
};

inline const DriverFns& driver_fns() {
  static DriverFns fns = [] {
    DriverFns f;
    cudaDriverEntryPointQueryResult q1, q2;
    void* p1 = nullptr;
    void* p2 = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p1, 12000,
                                         cudaEnableDefault, &q1) == cudaSuccess &&
        cudaGetDriverEntryPointByVersion("cuTensorMapEncodeIm2col", &p2, 12000,
                                         cudaEnableDefault, &q2) == cudaSuccess &&
        q1 == cudaDriverEntryPointSuccess && q2 == cudaDriverEntryPointSuccess) {
      f.tiled = reinterpret_cast<EncodeTiledFn>(p1);
      f.im2col = reinterpret_cast<EncodeIm2colFn>(p2);
      f.ok = true;
    }
    return f;
  }();
  return fns;
}

inline CUtensorMapSwizzle swizzle_for(int row_bytes) {
  switch (row_bytes) {
    case 128:
      return CU_TENSOR_MAP_SWIZZLE_128B;
    case 64:
      return CU_TENSOR_MAP_SWIZZLE_64B;
    case 32:
      return CU_TENSOR_MAP_SWIZZLE_32B;
    default:
      return CU_TENSOR_MAP_SWIZZLE_NONE;
  }
}

// im2col descriptor over an NHWC tensor [n, h, w, c_elems] of elem_bytes-wide
// elements.  Each load fetches `pixels` output pixels x box_c channels.
inline int encode_im2col(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                         int elem_bytes, int64_t n, int64_t h, int64_t w, int64_t c_elems,
                         int box_c, int pixels, int lower_w, int lower_h, int upper_w,
                         int upper_h, int stride_w, int stride_h) {
  const DriverFns& f = driver_fns();
  if (!f.ok) return fail(IE_RUNTIME, "cuTensorMapEncodeIm2col entry point unavailable");
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(c_elems), static_cast<cuuint64_t>(w),
                              static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(n)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(c_elems * elem_bytes),
                                 static_cast<cuuint64_t>(w * c_elems * elem_bytes),
                                 static_cast<cuuint64_t>(h * w * c_elems * elem_bytes)};
  const int lower[2] = {lower_w, lower_h};
  const int upper[2] = {upper_w, upper_h};
  const cuuint32_t estrides[4] = {1, static_cast<cuuint32_t>(stride_w),
                                  static_cast<cuuint32_t>(stride_h), 1};
  const CUresult r = f.im2col(map, dtype, 4, const_cast<void*>(base), dims, strides, lower,
                              upper, static_cast<cuuint32_t>(box_c),
                              static_cast<cuuint32_t>(pixels), estrides,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(box_c * elem_bytes),
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(IE_RUNTIME,
                "cuTensorMapEncodeIm2col failed (%d): n=%lld h=%lld w=%lld c=%lld box_c=%d "
                "lower=(%d,%d) upper=(%d,%d) stride=(%d,%d)",
                static_cast<int>(r), static_cast<long long>(n), static_cast<long long>(h),
                static_cast<long long>(w), static_cast<long long>(c_elems), box_c, lower_w,
                lower_h, upper_w, upper_h, stride_w, stride_h);
  }
  return IE_OK;
}

// 4D tiled descriptor over an NHWC tensor [n, h, w, c_elems]; box = box_c x
// box_w x box_h x 1 (channels innermost), swizzled by the box's channel bytes.
inline int encode_nhwc_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                          int elem_bytes, int64_t n, int64_t h, int64_t w, int64_t c_elems,
                          int box_c, int box_w, int box_h) {
  const DriverFns& f = driver_fns();
  if (!f.ok) return fail(IE_RUNTIME, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(c_elems), static_cast<cuuint64_t>(w),
                              static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(n)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(c_elems * elem_bytes),
                                 static_cast<cuuint64_t>(w * c_elems * elem_bytes),
                                 static_cast<cuuint64_t>(h * w * c_elems * elem_bytes)};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(box_c), static_cast<cuuint32_t>(box_w),
                             static_cast<cuuint32_t>(box_h), 1};
  const cuuint32_t estrides[4] = {1, 1, 1, 1};
  const CUresult r = f.tiled(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estrides,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(box_c * elem_bytes),
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(IE_RUNTIME,
                "cuTensorMapEncodeTiled (4D) failed (%d): n=%lld h=%lld w=%lld c=%lld box=%dx%dx%d",
                static_cast<int>(r), static_cast<long long>(n), static_cast<long long>(h),
                static_cast<long long>(w), static_cast<long long>(c_elems), box_c, box_w, box_h);
  }
  return IE_OK;
}

// 2D tiled descriptor over a row-major [rows, cols] matrix; box = box_rows x
// box_cols elements.
inline int encode_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                     int elem_bytes, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  const DriverFns& f = driver_fns();
  if (!f.ok) return fail(IE_RUNTIME, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * elem_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols),
                             static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estrides[2] = {1, 1};
  const CUresult r = f.tiled(map, dtype, 2, const_cast<void*>(base), dims, strides, box,
                             estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             swizzle_for(box_cols * elem_bytes),
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(IE_RUNTIME, "cuTensorMapEncodeTiled failed (%d): rows=%lld cols=%lld box=%dx%d",
                static_cast<int>(r), static_cast<long long>(rows),
                static_cast<long long>(cols), box_rows, box_cols);
  }
  return IE_OK;
}

inline int num_sms() {
  static int sms = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
      return v;
    }
    return 148;
  }();
  return sms;
}

}  // namespace ie_cuda
