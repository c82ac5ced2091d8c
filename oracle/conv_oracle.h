/*
 * CPU oracle for the Conv2D forward path: TEST INFRASTRUCTURE ONLY.
 *
 * This header declares a plain-C restatement of the reference engine's
 * convolution (grayondream/ComputeEngine, src/ops/traditional/conv2d_op.cpp)
 * plus the int8-quantized form that the reference only plans.  Only the test
 * suite, the smoke check and the CPU-baseline leg of the benchmark load it, as
 * the checker.  Nothing in the shipped library links or calls it.
 *
 * Parity status:
 *  - fp32: pinned against the reference's own golden vectors
 *    (tests/data/traditional_reference.h) and against the reference's
 *    Conv2DOp compiled from its sources (oracle/_ref).
 *  - int8 integer accumulation: pinned against the reference Conv2DOp run on
 *    integer-valued fp32 data (exact while every partial sum stays below
 *    2^24).
 *  - int8 requantize: unpinned by the reference, which has no int8 conv
 *    (src/converter/quantization/quant_plugins.h:7-22 returns Unsupported);
 *    the rounding and saturation rules below are this project's scheme.
 */
#ifndef CONV_ORACLE_H
#define CONV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes mirror ie::Error::Code (src/core/base/error.h:10-17), plus 0
 * for success. */
enum {
    ORC_OK = 0,
    ORC_INVALID_ARGUMENT = 1,
    ORC_UNSUPPORTED = 2,
    ORC_NOT_FOUND = 3,
    ORC_ALREADY_EXISTS = 4,
    ORC_OUT_OF_MEMORY = 5,
    ORC_RUNTIME = 6,
};

/* auto_pad values (src/ops/traditional/attrs_util.h:18). */
enum { ORC_PAD_NOTSET = 0, ORC_PAD_VALID = 1, ORC_PAD_SAME_UPPER = 2,
       ORC_PAD_SAME_LOWER = 3 };

/* Resolved convolution geometry. */
typedef struct orc_conv_geom {
    int64_t n, c, h, w;          /* input NCHW */
    int64_t m, cg, kh, kw;       /* weight [M, C/group, kH, kW] */
    int64_t stride_h, stride_w;
    int64_t dil_h, dil_w;
    int64_t pad_t, pad_l, pad_b, pad_r;  /* resolved pads */
    int64_t group;
    int64_t out_h, out_w;
} orc_conv_geom;

/* Validates shapes and resolves padding and output size exactly as
 * conv2d_forward does (conv2d_op.cpp:77-165).  pads_attr is
 * {top, left, bottom, right}; auto_pad one of ORC_PAD_*.  bias_len < 0 means
 * "no bias input".  Returns ORC_OK or ORC_INVALID_ARGUMENT. */
int orc_conv_resolve(int64_t n, int64_t c, int64_t h, int64_t w,
                     int64_t m, int64_t cg, int64_t kh, int64_t kw,
                     int64_t stride_h, int64_t stride_w,
                     int64_t dil_h, int64_t dil_w,
                     const int64_t pads_attr[4], int64_t group, int auto_pad,
                     int depthwise, int64_t bias_len, orc_conv_geom* out);

/* SAME padding for one axis (attrs_util.h:185-197). */
void orc_same_padding(int64_t input, int64_t kernel, int64_t dilation,
                      int64_t stride, int lower, int64_t* before,
                      int64_t* after);

/* fp32 NCHW convolution following conv2d_op.cpp:189-241: im2col per image and
 * group, then one ascending-t dot product per output element, then the bias
 * add (skipped when the bias value is 0, as the reference does).  act: 0 none,
 * 1 ReLU, 2 ReLU6 (applied after the bias; the reference runs these as
 * separate Relu/Clip nodes).  nthreads <= 1 runs serially; more threads split
 * the batch. */
int orc_conv2d_f32(const orc_conv_geom* g, const float* x, const float* wt,
                   const float* bias, int act, float* y, int nthreads);

/* int8 NCHW convolution.
 *   acc[n,m,p] = sum over (c, ky, kx) of (xq - zp_x) * wq   (int32; taps that
 *                fall in the padding contribute 0, i.e. real 0.0)
 *   t          = acc + bias[m]                             (int32, wraps)
 *   r          = round_half_away_from_zero(t * mult[m])    (exact: the fp32
 *                multiplier is mant * 2^-shift, the product is taken in
 *                64-bit integers and rounded once)
 *   yq         = clamp(r + zp_y, qmin, qmax)
 * x_signed selects int8 (1) or uint8 (0) storage for x; y_signed likewise for
 * y.  bias may be NULL.  acc_out (optional) receives acc before the bias. */
int orc_conv2d_q8(const orc_conv_geom* g, const void* x, int x_signed,
                  int32_t zp_x, const int8_t* wt, const int32_t* bias,
                  const float* mult, int32_t zp_y, int32_t qmin, int32_t qmax,
                  int y_signed, void* y, int32_t* acc_out, int nthreads);

/* The requantize step alone, for exhaustive edge tests. */
int32_t orc_requantize(int32_t acc, int32_t bias, float mult, int32_t zp_y,
                       int32_t qmin, int32_t qmax);

/* int8 addition of two quantized tensors of the same shape (the shortcut Add
 * of a quantized ResNet block; the reference has no int8 Add, so the rule is
 * this project's, in the style of the requantize above):
 *   v  = (a - zp_a) * mult_a + (b - zp_b) * mult_b   exact: both fp32
 *        multipliers are dyadic rationals mant * 2^-shift, summed over the
 *        common shift in 128-bit integers
 *   yq = clamp(round_half_away_from_zero(v) + zp_y, qmin, qmax)
 * mult_a = s_a / s_y and mult_b = s_b / s_y, each rounded once to fp32.
 * ORC_UNSUPPORTED when the two nonzero multipliers' shifts differ by more
 * than 60 (one term below 2^-60 of the other). */
int orc_qadd(const void* a, int a_signed, int32_t zp_a, float mult_a, const void* b,
             int b_signed, int32_t zp_b, float mult_b, int32_t zp_y, int32_t qmin,
             int32_t qmax, int y_signed, void* y, int64_t count);

#ifdef __cplusplus
}
#endif

#endif
