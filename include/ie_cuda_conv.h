/*
 * ie_cuda_conv.h -- C ABI of the B200 (sm_100a) Conv2D forward backend.
 *
 * This is the thin extern "C" shim between host code (the engine's
 * CudaConv2DOp / CudaDepthwiseConv2DOp, the benchmark, ctypes tests) and the
 * hand-written CUDA kernels.  Plain pointers and sizes only: every tensor
 * pointer is DEVICE memory unless stated otherwise, every call is
 * asynchronous on the given stream (NULL = legacy default stream), and no call
 * allocates device memory: buffers and workspaces come from the caller.
 *
 * Reference interfaces replaced (grayondream/ComputeEngine):
 *   conv2d_forward          src/ops/traditional/conv2d_op.cpp:73-245
 *   Conv2DOp::forward       src/ops/traditional/conv2d_op.h:42-46
 *   DepthwiseConv2DOp       src/ops/traditional/conv2d_op.h:53-67
 *   parse_conv_config       src/ops/traditional/conv2d_op.cpp:26-71 (attrs)
 *   same_padding            src/ops/traditional/attrs_util.h:185-197
 *   KernelFns::matmul_row   src/core/ops/kernel_fns.h:10-18 (the inner GEMM)
 *   Int8QuantPlugin         src/converter/quantization/quant_plugins.h:7-22
 *                           (stub in the reference; the int8 scheme below is
 *                           this backend's own)
 *
 * Status codes mirror ie::Error::Code (src/core/base/error.h:10-17) shifted
 * by one, so 0 means success.
 */
#ifndef IE_CUDA_CONV_H
#define IE_CUDA_CONV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IE_CUDA_CONV_ABI_VERSION 2

typedef enum ie_status {
  IE_OK = 0,
  IE_INVALID_ARGUMENT = 1, /* Error::Code::InvalidArgument */
  IE_UNSUPPORTED = 2,      /* Error::Code::Unsupported */
  IE_NOT_FOUND = 3,        /* Error::Code::NotFound */
  IE_ALREADY_EXISTS = 4,   /* Error::Code::AlreadyExists */
  IE_OUT_OF_MEMORY = 5,    /* Error::Code::OutOfMemory */
  IE_RUNTIME = 6           /* Error::Code::Runtime (CUDA errors map here) */
} ie_status;

/* auto_pad (attrs_util.h:18: AutoPad::{NotSet, Valid, SameUpper, SameLower}) */
enum { IE_PAD_NOTSET = 0, IE_PAD_VALID = 1, IE_PAD_SAME_UPPER = 2, IE_PAD_SAME_LOWER = 3 };

/* Activation folded into the epilogue.  The reference runs these as separate
 * Relu (core/ops/common/relu_op.h) and Clip (data_ops.cpp:1078) nodes. */
enum { IE_ACT_NONE = 0, IE_ACT_RELU = 1, IE_ACT_RELU6 = 2 };

/* Convolution attributes and shapes, the union of ConvConfig
 * (conv2d_op.h:13-21) and the tensor shapes conv2d_forward reads
 * (conv2d_op.cpp:94-102).  x is [n, c, h, w], weight [m, c/group, kh, kw]. */
typedef struct ie_conv2d_desc {
  int64_t n, c, h, w;
  int64_t m, kh, kw;
  int64_t stride_h, stride_w;
  int64_t dil_h, dil_w;
  int64_t pad_top, pad_left, pad_bottom, pad_right; /* the "pads" attribute */
  int64_t group;
  int32_t auto_pad;  /* IE_PAD_* */
  int32_t depthwise; /* 1: DepthwiseConv2D semantics (group must equal c) */
} ie_conv2d_desc;

/* Output of ie_conv2d_resolve: pads after auto_pad, output extent. */
typedef struct ie_conv2d_shape {
  int64_t pad_top, pad_left, pad_bottom, pad_right;
  int64_t out_h, out_w;
} ie_conv2d_shape;

/* Per-tensor quantization of one int8 convolution.
 *   acc = sum (xq - zp_x) * wq         int32, padding contributes real 0.0
 *   t   = acc + bias[m]                int32 (wrapping)
 *   r   = round_half_away(t * mult[m]) exact: mult (fp32, = s_x * s_w[m] / s_y
 *                                      computed in double and rounded once) is
 *                                      the dyadic rational mant * 2^-shift, so
 *                                      the product is taken in 64-bit integers
 *   yq  = clamp(r + zp_y, qmin, qmax)
 * ReLU folds in as qmin = zp_y, ReLU6 as qmax = zp_y + round(6 / s_y). */
typedef struct ie_q8_params {
  int32_t x_signed; /* activations stored as int8 (1) or uint8 (0) */
  int32_t zp_x;     /* activation zero point, any value of the storage type;
                       for the dense kernel a nonzero zp_x with padding needs
                       the haloed input (ie_cuda_q8_pack_input_halo) */
  int32_t y_signed; /* output stored as int8 (1) or uint8 (0) */
  int32_t zp_y;
  int32_t qmin, qmax;
} ie_q8_params;

/* ------------------------------------------------------------ geometry */

/* Validates a convolution exactly as conv2d_forward does
 * (conv2d_op.cpp:77-165): positive dims, group divides c and m, weight
 * channels == c/group, depthwise needs group == c, bias length (pass -1 for
 * "no bias"), kernel not larger than the padded input, non-empty output.
 * Resolves SAME_UPPER / SAME_LOWER / VALID padding (attrs_util.h:185-197).
 * Host-only, no CUDA call. */
int ie_conv2d_resolve(const ie_conv2d_desc* desc, int64_t bias_len, ie_conv2d_shape* out);

/* ------------------------------------------------------------ int8 path */

/* Bytes of the packed weight buffer for ie_cuda_q8_pack_weights: the packed
 * weights followed by int32 per-output-channel weight sums
 * [round_up(m, 16)] (used to fold a nonzero activation zero point into the
 * bias). */
size_t ie_cuda_q8_packed_weight_bytes(const ie_conv2d_desc* desc);

/* Repacks int8 weights [m, c/group, kh, kw] (device) into the K-major layout
 * the implicit-GEMM kernel reads: [m][kh][kw][c padded to the channel block],
 * zero filled, then writes the weight-sum trailer.  Dense convolutions
 * (group == 1) only. */
int ie_cuda_q8_pack_weights(const ie_conv2d_desc* desc, const int8_t* w, void* packed,
                            void* stream);

/* NCHW -> NHWC for 8-bit activations, c_store >= c channels per pixel
 * (c_store a multiple of 16, extra channels zero).  xor_mask 0x80 turns
 * uint8 with zero point 128 into int8 with zero point 0, so zero padding is
 * exact; pass 0 to copy bytes unchanged. */
int ie_cuda_q8_pack_input(const void* x_nchw, void* x_nhwc, int64_t n, int64_t c, int64_t h,
                          int64_t w, int64_t c_store, int32_t xor_mask, void* stream);

/* Haloed input for a nonzero activation zero point.  The reference's padding
 * is real 0.0, i.e. the stored value zp_x; TMA fills out-of-image reads with
 * byte 0, so for zp_x != 0 the dense kernel instead reads an input grown by
 * the convolution's resolved pads whose border holds zp_x:
 *   [n, h + pad_top + pad_bottom, w + pad_left + pad_right, c_store]
 * (c_store = c rounded up to 16; channels past c also hold zp_x).  The
 * kernel adds -zp_x * sum(w[m]) to the bias (the packed weights' trailer), so
 * every tap contributes (x - zp_x) * w exactly.  Unpadded convolutions need
 * no halo: the plain NHWC tensor is its own haloed form.
 *   ie_cuda_q8_halo_input_bytes   bytes of that buffer (0 on a bad desc)
 *   ie_cuda_q8_pack_input_halo    NCHW 8-bit [n, c, h, w] -> haloed NHWC
 *   ie_cuda_q8_halo_nhwc          NHWC [n, h, w, c_store] (e.g. the previous
 *                                 layer's output) -> haloed NHWC
 * zp_x is the stored byte's value (-128..127 for int8, 0..255 for uint8). */
size_t ie_cuda_q8_halo_input_bytes(const ie_conv2d_desc* desc);
int ie_cuda_q8_pack_input_halo(const ie_conv2d_desc* desc, const void* x_nchw, void* x_halo,
                               int32_t zp_x, void* stream);
int ie_cuda_q8_halo_nhwc(const ie_conv2d_desc* desc, const void* x_nhwc, void* x_halo,
                         int32_t zp_x, void* stream);

/* NHWC (c_store channels per pixel) -> NCHW for 8-bit activations. */
int ie_cuda_q8_unpack_output(const void* y_nhwc, void* y_nchw, int64_t n, int64_t c,
                             int64_t h, int64_t w, int64_t c_store, void* stream);

/* int8 convolution, dense (group == 1), NHWC in and out.
 *   x      [n, h, w, c_store] int8/uint8, c_store = c rounded up to 16;
 *          with q->zp_x != 0 and nonzero pads, the haloed input above
 *   packed ie_cuda_q8_pack_weights output
 *   bias   [m] int32 or NULL;  mult [m] fp32
 *   y      [n, out_h, out_w, m_store], m_store = m rounded up to 16: the
 *          buffer's last dimension is m_store whatever m is (the channels
 *          past m are written too and hold no data)
 * Tensor cores: tcgen05.mma kind::i8, TMA im2col loads, TMEM accumulators,
 * bias + requantize + clamp fused into the epilogue.  Replaces
 * conv2d_forward for quantized graphs. */
int ie_cuda_conv2d_q8(const ie_conv2d_desc* desc, const ie_q8_params* q, const void* x,
                      const void* packed, const int32_t* bias, const float* mult, void* y,
                      void* stream);

/* Same, writing raw int32 (acc + bias) instead of requantized bytes, y
 * [n, out_h, out_w, m_store] int32. */
int ie_cuda_conv2d_q8_acc(const ie_conv2d_desc* desc, const ie_q8_params* q, const void* x,
                          const void* packed, const int32_t* bias, int32_t* y, void* stream);

/* Depthwise int8 weights [c, 1, kh, kw] -> [kh*kw][c rounded up to 16]. */
size_t ie_cuda_dw_q8_packed_weight_bytes(const ie_conv2d_desc* desc);
int ie_cuda_dw_q8_pack_weights(const ie_conv2d_desc* desc, const int8_t* w, void* packed,
                               void* stream);

/* Depthwise int8 convolution (group == c == m), NHWC in and out with c
 * rounded up to 16 channels per pixel.  Any input zero point (padding still
 * contributes real 0.0).  CUDA cores, 128-bit channel vectors, bandwidth
 * bound.  Replaces DepthwiseConv2DOp (conv2d_op.h:53-67) for quantized
 * graphs. */
int ie_cuda_dwconv2d_q8(const ie_conv2d_desc* desc, const ie_q8_params* q, const void* x,
                        const void* packed, const int32_t* bias, const float* mult, void* y,
                        void* stream);

/* Stem of the 53-layer ResNet-50 stack: a 7x7 / stride 2 / pad 3 convolution
 * on c <= 4 input channels (h, w even).  Space-to-depth by 2 plus a 4-column
 * unroll turns it into a 4x1 stride-1 convolution over 64 stored channels that
 * runs on ie_cuda_conv2d_q8 like every other layer:
 *   ie_cuda_q8_stem_desc         fills that equivalent descriptor
 *   ie_cuda_q8_stem_pack_input   NCHW [n, c, h, w] 8-bit -> [n, h/2, w/2, 64],
 *                                xor_mask as in ie_cuda_q8_pack_input
 *   ie_cuda_q8_stem_pack_weights [m, c, 7, 7] int8 -> packed weights of the
 *                                equivalent layer (ie_cuda_q8_packed_weight_bytes
 *                                of the equivalent descriptor)
 * The result equals the direct 7x7 / stride 2 convolution bit for bit.  The
 * re-layout zero-fills its padding, so it takes activations with zero point 0
 * (uint8 with zero point 128: xor_mask 0x80 and x_signed = 1); run other zero
 * points as a plain 7x7 / stride 2 convolution on the haloed input. */
int ie_cuda_q8_stem_desc(int64_t n, int64_t c, int64_t h, int64_t w, int64_t m,
                         ie_conv2d_desc* out);
int ie_cuda_q8_stem_pack_input(const void* x_nchw, void* x_packed, int64_t n, int64_t c,
                               int64_t h, int64_t w, int32_t xor_mask, void* stream);
int ie_cuda_q8_stem_pack_weights(const int8_t* w, void* packed, int64_t m, int64_t c,
                                 void* stream);

/* Max pooling (k x k, stride, symmetric pad, floor output size) over 8-bit
 * NHWC activations with c_store (multiple of 16) channels per pixel.  The
 * graph's MaxPool between the stem and stage 1 (pool_ops.cpp); padding never
 * wins. */
int ie_cuda_q8_maxpool2d(const void* x, void* y, int64_t n, int64_t h, int64_t w,
                         int64_t c_store, int64_t k, int64_t stride, int64_t pad,
                         int32_t is_signed, void* stream);

/* The same pooling over split fp32 activations (the IE_Y_BF16X2_NHWC layout:
 * bf16 [hi plane (c_store) | lo plane (c_store)] per pixel); the pair with the
 * largest hi + lo is kept bit for bit. */
int ie_cuda_f32x2_maxpool2d(const void* x, void* y, int64_t n, int64_t h, int64_t w,
                            int64_t c_store, int64_t k, int64_t stride, int64_t pad,
                            void* stream);

/* int8 Add of two quantized tensors of one layout and size (the shortcut Add
 * of a quantized ResNet block; the reference has no int8 Add, the rule is this
 * backend's, exact like the convolution's requantize):
 *   v  = (a - zp_a) * mult_a + (b - zp_b) * mult_b   (mult = s_in / s_y, fp32;
 *        both are dyadic rationals, summed exactly in 128-bit integers)
 *   yq = clamp(round_half_away(v) + zp_y, qmin, qmax)
 * count = elements (bytes) of each tensor.  IE_UNSUPPORTED when the two
 * nonzero multipliers differ by more than 2^60. */
typedef struct ie_qadd_params {
  int32_t a_signed, zp_a;
  float mult_a;
  int32_t b_signed, zp_b;
  float mult_b;
  int32_t y_signed, zp_y, qmin, qmax;
} ie_qadd_params;
int ie_cuda_qadd(const ie_qadd_params* p, const void* a, const void* b, void* y, int64_t count,
                 void* stream);

/* ------------------------------------------------------------ fp32 path */

/* Output formats of ie_cuda_conv2d_bf16x3. */
enum {
  IE_Y_F32_NHWC = 0,    /* fp32 [n, oh, ow, m rounded up to 16] */
  IE_Y_F32_NCHW = 1,    /* fp32 [n, m, oh, ow], the reference layout */
  IE_Y_BF16X2_NHWC = 2  /* bf16 [n, oh, ow, hi plane | lo plane], next layer's input */
};

/* fp32 weights [m, c, kh, kw] -> bf16 [m][kh*kw][hi (ck) | lo (ck)]. */
size_t ie_cuda_f32_packed_weight_bytes(const ie_conv2d_desc* desc);
int ie_cuda_f32_pack_weights(const ie_conv2d_desc* desc, const float* w, void* packed,
                             void* stream);

/* fp32 NCHW -> NHWC bf16 [hi plane (c_store) | lo plane (c_store)] per pixel,
 * c_store >= c a multiple of 16 (padding channels zero). */
int ie_cuda_f32_pack_input(const float* x_nchw, void* x_split, int64_t n, int64_t c, int64_t h,
                           int64_t w, int64_t c_store, void* stream);

/* Dense fp32 convolution on split inputs (group == 1): tcgen05.mma kind::f16
 * with bf16 operands, three MMAs per K block (hi*hi + hi*lo + lo*hi) into
 * one fp32 TMEM accumulator; bias and activation fused in the epilogue.
 * x_split has c rounded up to 16 channels per plane. */
int ie_cuda_conv2d_bf16x3(const ie_conv2d_desc* desc, int32_t act, const void* x_split,
                          const void* packed, const float* bias, void* y, int32_t y_format,
                          void* stream);

/* fp32 convolution, NCHW in and out, the drop-in for conv2d_forward
 * (conv2d_op.cpp:73-245) on fp32 tensors.  Runs as bf16x3 on the tensor
 * cores (x = xh + xl, w = wh + wl; xh*wh + xh*wl + xl*wh accumulated in
 * fp32) for dense convolutions, on CUDA cores for depthwise / grouped ones.
 * bias may be NULL; act is IE_ACT_*.  workspace must hold
 * ie_cuda_conv2d_f32_workspace_bytes(desc) bytes (256-byte aligned). */
size_t ie_cuda_conv2d_f32_workspace_bytes(const ie_conv2d_desc* desc);
int ie_cuda_conv2d_f32(const ie_conv2d_desc* desc, int32_t act, const float* x,
                       const float* w, const float* bias, float* y, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Residual-add fusion: the dense fp32 convolution with an extra tensor of the
 * output's shape and layout added after the bias and before the activation,
 *   y = act((conv(x, w) + bias) + residual)
 * one rounding per operation, the order of the reference's Conv2D, Add
 * (core/ops) and Relu nodes.  This is the ResNet bottleneck's projection /
 * identity add run in the last 1x1 convolution's epilogue instead of as a
 * separate pass over the activation.  residual may equal y (each element is
 * read before it is written, by the same thread).  Dense (group == 1) only:
 * IE_UNSUPPORTED otherwise.  The bf16x3 form takes split inputs and packed
 * weights like ie_cuda_conv2d_bf16x3 and an fp32 output format; the f32 form
 * is the NCHW drop-in with ie_cuda_conv2d_f32's workspace. */
int ie_cuda_conv2d_bf16x3_residual(const ie_conv2d_desc* desc, int32_t act, const void* x_split,
                                   const void* packed, const float* bias, const float* residual,
                                   void* y, int32_t y_format, void* stream);
int ie_cuda_conv2d_f32_residual(const ie_conv2d_desc* desc, int32_t act, const float* x,
                                const float* w, const float* bias, const float* residual,
                                float* y, void* workspace, size_t workspace_bytes, void* stream);

/* No-allocation variant of ie_cuda_conv2d_f32.  It has no counterpart in the
 * reference.  It is for callers that cannot allocate device memory or hand
 * this library a workspace: an Op::forward that only receives the engine's
 * host allocator, or code that must not call cudaMalloc / cudaFree (they
 * synchronize the device and can break an owner's memory plan).  The caller
 * still passes x, w, bias and y; the packed operands go to a fixed scratch
 * array inside this library's device image (ie_cuda_noalloc_scratch_bytes(),
 * 16 MiB, held on every GPU that loads the library until the process exits).
 *   - Convolutions whose workspace (ie_cuda_conv2d_f32_workspace_bytes) is
 *     larger than the scratch are rejected with IE_INVALID_ARGUMENT before
 *     any device work.
 *   - The first call on a device looks up the scratch's device address with
 *     that device current (cudaGetSymbolAddress); make that first call before
 *     any stream capture on that device.  The address is cached per device
 *     for the life of the process: do not call cudaDeviceReset (or otherwise
 *     tear down the primary context) and keep using this entry point.
 *   - All calls share the one scratch array, which keeps the last call's
 *     contents; every byte a call reads is rewritten by its own packing
 *     kernels first, so nothing needs clearing.  Calls that overlap on the
 *     GPU (different streams, or different host threads without ordering)
 *     race on the scratch: serialize them.
 * No cudaMalloc, cudaFree or allocating library routine is called. */
size_t ie_cuda_noalloc_scratch_bytes(void);
int ie_cuda_conv2d_f32_noalloc(const ie_conv2d_desc* desc, int32_t act, const float* x,
                               const float* w, const float* bias, float* y, void* stream);

/* ------------------------------------------------------------ errors */

/* Human-readable detail of the last failing call on this host thread. */
const char* ie_cuda_last_error(void);

/* Reads and clears the device-side error word of the current device: nonzero
 * when a kernel's bounded wait ran out (the kernel then returned early and
 * its output is invalid).  Synchronizes the device. */
int ie_cuda_take_device_error(uint32_t* code);

/* Self-test of the failure detection of the kernels' bounded waits (no
 * counterpart in the reference; its failure detection is host-side only).
 * Launches one CTA that allocates tensor memory and waits on an mbarrier that
 * nothing ever arrives on; the wait gives up after wait_limit_ns (1 us to
 * 2 s), records code 0x1FF in the device error word (read it with
 * ie_cuda_take_device_error), frees the tensor memory and returns, the same
 * wind-down the convolution kernels take when one of their waits runs out.
 * Synchronizes `stream`; *waited_ns (may be NULL) receives the time the wait
 * took.  IE_OK when the wait gave up as designed. */
int ie_cuda_bounded_wait_probe(uint64_t wait_limit_ns, uint64_t* waited_ns, void* stream);

/* Number of kernel launches this library issued on the calling host thread
 * since the last reset (for the benchmark's launch count). */
uint64_t ie_cuda_launch_count(int reset);

/* Measured int8 tensor-core rate of the current GPU (no counterpart in the
 * reference; the denominator for int8 roofline fractions): one CTA per SM
 * issues `iters` back-to-back tcgen05.mma kind::i8, M=128 N=256 K=32, from
 * shared memory into tensor memory; *tops = 2 * 128 * 256 * 32 * iters * SMs
 * / the launch's event time, in TOPS.  Synchronizes the stream.  iters in
 * [1000, 1e7] (40000 takes a few ms). */
int ie_cuda_mma_i8_peak(int32_t iters, double* tops, void* stream);

/* ---------------------------------------------------------------- head ops
 * The rest of a ResNet graph's head on the GPU, so no node falls back to the
 * host: 2D pooling, global average pooling and Gemm over fp32 tensors. */

/* Pooling attributes and shape, the union of PoolConfig (pool_ops.h:13-21)
 * and the NCHW input shape pool2d_forward reads (pool_ops.cpp:131-136). */
typedef struct ie_pool2d_desc {
  int64_t n, c, h, w;
  int64_t kh, kw;                                    /* kernel_shape */
  int64_t stride_h, stride_w;
  int64_t pad_top, pad_left, pad_bottom, pad_right;  /* the "pads" attribute */
  int32_t auto_pad;                                  /* IE_PAD_* */
  int32_t ceil_mode;
  int32_t count_include_pad;
} ie_pool2d_desc;

/* Effective pads and output extent (resolve_pool_geometry, pool_ops.cpp:24-61):
 * SAME pads split like convolution, ceil_mode drops a last window that would
 * start in the padding; IE_INVALID_ARGUMENT for a window larger than the
 * padded input or an empty output. */
int ie_pool2d_resolve(const ie_pool2d_desc* desc, ie_conv2d_shape* out);

/* Max (max_pool = 1) or average pooling, NCHW fp32 -> [n, c, out_h, out_w]
 * (pool2d_forward, pool_ops.cpp:111-215, behind MaxPool2DOp / AvgPool2DOp,
 * pool_ops.h:37-68).  Same window order and arithmetic as the reference:
 * results equal it bit for bit. */
int ie_cuda_pool2d_f32(const ie_pool2d_desc* desc, int32_t max_pool, const float* x, float* y,
                       void* stream);

/* Max pooling of 8-bit activations in the int8 activation layout (NHWC with
 * c_store = round_up(desc->c, 16) bytes per pixel; padding channels carry no
 * data) under the same configurations as ie_cuda_pool2d_f32: the MaxPool2D
 * node of a quantized graph.  The maximum of quantized values is the
 * quantized maximum (the quantization is monotonic and the output keeps the
 * input's scale and zero point), so the result equals the reference
 * MaxPool2DOp run on the same integers as floats, bit for bit; a window with
 * no in-image position (possible only when a pad reaches the kernel size)
 * gives the storage type's minimum where the fp32 pool gives -inf.
 * x, y 16-byte aligned; y holds [n, out_h, out_w, c_store]. */
int ie_cuda_q8_maxpool2d_nhwc(const ie_pool2d_desc* desc, int32_t is_signed, const void* x,
                              void* y, void* stream);

/* [n, c, h, w] -> [n, c, 1, 1] mean over each plane (global_avg_pool_forward,
 * pool_ops.cpp:217-270, behind GlobalAvgPoolOp): one sequential fp32 sum per
 * plane, bit-exact with the reference. */
int ie_cuda_global_avg_pool_f32(const float* x, float* y, int64_t n, int64_t c, int64_t h,
                                int64_t w, void* stream);

/* Global average pooling of an 8-bit activation into dequantized fp32: the
 * GlobalAvgPool node at the head of a quantized graph, ahead of the fp32 Gemm
 * (the reference GlobalAvgPoolOp is fp32-only; this rule is the backend's
 * own).  x [n, h, w, c_store] (c_store = round_up(c, 16), the int8 activation
 * layout), y [n, c] fp32:
 *   y = fp32((sum over the plane of q - zp * h * w) * scale / (h * w))
 * with the sum exact in integers and the rest in double, rounded once.
 * h * w * 255 must fit int32 (IE_UNSUPPORTED otherwise). */
int ie_cuda_q8_global_avg_pool_nhwc(const void* x, float* y, int64_t n, int64_t c, int64_t h,
                                    int64_t w, int32_t is_signed, int32_t zp, double scale,
                                    void* stream);

/* C broadcast of Gemm (gemm_op.cpp:103-139). */
enum {
  IE_GEMM_C_NONE = 0,   /* no C */
  IE_GEMM_C_SCALAR = 1, /* one value */
  IE_GEMM_C_ROW = 2,    /* [M] or [M, 1]: C(i, j) = c[i] */
  IE_GEMM_C_COLUMN = 3, /* [N] or [1, N]: C(i, j) = c[j] */
  IE_GEMM_C_FULL = 4    /* [M, N] */
};

/* Y[M, N] = alpha * A' * B' + beta * C, A' = A [M, K] or A^T (trans_a, A is
 * [K, M]), B' = B [K, N] or B^T (trans_b, B is [N, K]) — the drop-in for
 * GemmOp::forward (gemm_op.cpp:76-221).  The product runs on the tensor cores
 * as bf16x3 (a 1x1 convolution over M "pixels" of K channels), accurate to
 * about 1e-5 relative; a column C with alpha = beta = 1 is fused as the
 * convolution's bias, anything else goes through a separate epilogue.
 * workspace must hold ie_cuda_gemm_f32_workspace_bytes(...) bytes. */
size_t ie_cuda_gemm_f32_workspace_bytes(int64_t m, int64_t n, int64_t k, int32_t trans_a,
                                        int32_t trans_b);
int ie_cuda_gemm_f32(int64_t m, int64_t n, int64_t k, int32_t trans_a, int32_t trans_b,
                     float alpha, float beta, const float* a, const float* b, const float* c,
                     int32_t c_mode, float* y, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Tile plan of the last implicit-GEMM launch issued on the calling host thread
 * (performance introspection; no counterpart in the reference).  row_band is 1
 * when the stride-1 row-band mode ran: tiles of whole output rows, one input
 * band load per channel block, filter taps as shifted operand reads. */
typedef struct {
  int32_t bn;             /* output channels per tile */
  int32_t bk_bytes;       /* K bytes per pipeline step */
  int32_t m_sub;          /* 128-row sub-tiles per tile */
  int32_t stages;         /* pipeline depth */
  int32_t resident_weights;
  int32_t out_bufs;       /* staged output tiles (int8 requantized output) */
  int32_t row_band;
  int32_t grid;           /* CTAs launched */
  int32_t a_tiled;        /* 1x1 stride-1 unpadded: A loaded as a 2D [pixels, channels] tile */
} ie_conv_plan;
int ie_cuda_last_plan(ie_conv_plan* out);

/* Tile choice of the implicit GEMM (int8 and bf16x3), process-wide
 * (performance control; no counterpart in the reference).  Every plan gives
 * the same results: the int8 bytes, and for fp32 the same products summed in
 * the same K order.
 *   IE_TILE_FILL     (default) a launch whose default tiles cannot fill the
 *                    GPU and carry enough MMA work each (deep K) takes
 *                    narrower (64 / 128 channel) or shorter (128 position)
 *                    tiles when a cycle estimate says they finish at least
 *                    10% sooner
 *   IE_TILE_DEFAULT  always the default tiles: the widest channel tile that
 *                    wastes least (int8: 256 positions below 256 channels)
 * *previous (may be NULL) receives the policy that was in force. */
enum { IE_TILE_FILL = 0, IE_TILE_DEFAULT = 1 };
int ie_cuda_set_tile_policy(int32_t policy, int32_t* previous);

#ifdef __cplusplus
}
#endif

#endif /* IE_CUDA_CONV_H */
