/*
 * CPU oracle for the Conv2D forward path: TEST INFRASTRUCTURE ONLY.
 * See conv_oracle.h for the contract and the parity status of each part.
 *
 * Reference algorithm followed here (grayondream/ComputeEngine):
 *   src/ops/traditional/conv2d_op.cpp:77-165  validation, pads, output size
 *   src/ops/traditional/attrs_util.h:185-197  SAME_UPPER / SAME_LOWER split
 *   src/ops/traditional/conv2d_op.cpp:189-220 im2col rows (c_local, ky, kx)
 *   src/ops/traditional/conv2d_op.cpp:13-22   ascending-t row dot product
 *   src/ops/traditional/conv2d_op.cpp:223-238 per-channel row, bias after dot
 *
 * The int8 requantize is exact integer arithmetic (see orc_requantize), so it
 * does not depend on floating-point build flags.
 */
#include "conv_oracle.h"

#include <math.h>
#include <stdint.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

void orc_same_padding(int64_t input, int64_t kernel, int64_t dilation,
                      int64_t stride, int lower, int64_t* before,
                      int64_t* after) {
    /* attrs_util.h:188-195: output = ceil(input / stride); the odd pad goes
     * after the window for SAME_UPPER and before it for SAME_LOWER. */
    const int64_t output = (input + stride - 1) / stride;
    int64_t total = (output - 1) * stride + dilation * (kernel - 1) + 1 - input;
    if (total < 0) total = 0;
    int64_t b = total / 2;
    int64_t a = total - b;
    if (lower) {
        const int64_t t = b;
        b = a;
        a = t;
    }
    *before = b;
    *after = a;
}

int orc_conv_resolve(int64_t n, int64_t c, int64_t h, int64_t w,
                     int64_t m, int64_t cg, int64_t kh, int64_t kw,
                     int64_t stride_h, int64_t stride_w,
                     int64_t dil_h, int64_t dil_w,
                     const int64_t pads_attr[4], int64_t group, int auto_pad,
                     int depthwise, int64_t bias_len, orc_conv_geom* out) {
    /* conv2d_op.cpp:102-106 */
    if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || m <= 0 || cg <= 0 ||
        kh <= 0 || kw <= 0) {
        return ORC_INVALID_ARGUMENT;
    }
    if (stride_h <= 0 || stride_w <= 0 || dil_h <= 0 || dil_w <= 0) {
        return ORC_INVALID_ARGUMENT;
    }
    /* conv2d_op.cpp:107-119 */
    if (group <= 0 || c % group != 0 || m % group != 0) {
        return ORC_INVALID_ARGUMENT;
    }
    if (cg != c / group) return ORC_INVALID_ARGUMENT;
    if (depthwise && group != c) return ORC_INVALID_ARGUMENT;
    /* conv2d_op.cpp:128-136 */
    if (bias_len >= 0 && bias_len != m) return ORC_INVALID_ARGUMENT;

    int64_t pt = pads_attr[0], pl = pads_attr[1], pb = pads_attr[2],
            pr = pads_attr[3];
    if (pt < 0 || pl < 0 || pb < 0 || pr < 0) return ORC_INVALID_ARGUMENT;
    /* conv2d_op.cpp:138-149 */
    if (auto_pad == ORC_PAD_VALID) {
        pt = pl = pb = pr = 0;
    } else if (auto_pad == ORC_PAD_SAME_UPPER ||
               auto_pad == ORC_PAD_SAME_LOWER) {
        const int lower = auto_pad == ORC_PAD_SAME_LOWER;
        orc_same_padding(h, kh, dil_h, stride_h, lower, &pt, &pb);
        orc_same_padding(w, kw, dil_w, stride_w, lower, &pl, &pr);
    } else if (auto_pad != ORC_PAD_NOTSET) {
        return ORC_INVALID_ARGUMENT;
    }
    /* conv2d_op.cpp:151-165 */
    const int64_t eff_h = dil_h * (kh - 1) + 1;
    const int64_t eff_w = dil_w * (kw - 1) + 1;
    if (h + pt + pb < eff_h || w + pl + pr < eff_w) return ORC_INVALID_ARGUMENT;
    const int64_t oh = (h + pt + pb - eff_h) / stride_h + 1;
    const int64_t ow = (w + pl + pr - eff_w) / stride_w + 1;
    if (oh <= 0 || ow <= 0) return ORC_INVALID_ARGUMENT;

    out->n = n; out->c = c; out->h = h; out->w = w;
    out->m = m; out->cg = cg; out->kh = kh; out->kw = kw;
    out->stride_h = stride_h; out->stride_w = stride_w;
    out->dil_h = dil_h; out->dil_w = dil_w;
    out->pad_t = pt; out->pad_l = pl; out->pad_b = pb; out->pad_r = pr;
    out->group = group;
    out->out_h = oh; out->out_w = ow;
    return ORC_OK;
}

/* ---------------------------------------------------------------- threads */

typedef void (*orc_image_fn)(void* ctx, int64_t image, void* scratch);

typedef struct {
    orc_image_fn fn;
    void* ctx;
    int64_t begin, end;
    size_t scratch_bytes;
    int failed;
} orc_worker;

static void* orc_worker_main(void* arg) {
    orc_worker* wk = (orc_worker*)arg;
    void* scratch = malloc(wk->scratch_bytes ? wk->scratch_bytes : 1);
    if (scratch == NULL) {
        wk->failed = 1;
        return NULL;
    }
    for (int64_t i = wk->begin; i < wk->end; ++i) wk->fn(wk->ctx, i, scratch);
    free(scratch);
    return NULL;
}

/* Runs fn over images [0, n) on up to nthreads threads, each with its own
 * scratch buffer.  Images are independent, so the split changes nothing in
 * the results. */
static int orc_for_images(int64_t n, int nthreads, size_t scratch_bytes,
                          orc_image_fn fn, void* ctx) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > n) nthreads = (int)n;
    if (nthreads > 256) nthreads = 256;
    orc_worker workers[256];
    pthread_t threads[256];
    int started[256];
    for (int t = 0; t < nthreads; ++t) {
        workers[t].fn = fn;
        workers[t].ctx = ctx;
        workers[t].begin = n * t / nthreads;
        workers[t].end = n * (t + 1) / nthreads;
        workers[t].scratch_bytes = scratch_bytes;
        workers[t].failed = 0;
        started[t] = 0;
    }
    if (nthreads == 1) {
        orc_worker_main(&workers[0]);
        return workers[0].failed ? ORC_OUT_OF_MEMORY : ORC_OK;
    }
    for (int t = 0; t < nthreads; ++t) {
        started[t] = pthread_create(&threads[t], NULL, orc_worker_main,
                                    &workers[t]) == 0;
        if (!started[t]) orc_worker_main(&workers[t]);
    }
    int rc = ORC_OK;
    for (int t = 0; t < nthreads; ++t) {
        if (started[t]) pthread_join(threads[t], NULL);
        if (workers[t].failed) rc = ORC_OUT_OF_MEMORY;
    }
    return rc;
}

/* ------------------------------------------------------------------- fp32 */

typedef struct {
    const orc_conv_geom* g;
    const float* x;
    const float* wt;
    const float* bias;
    int act;
    float* y;
} orc_f32_ctx;

static void orc_f32_image(void* vctx, int64_t b, void* scratch) {
    const orc_f32_ctx* k = (const orc_f32_ctx*)vctx;
    const orc_conv_geom* g = k->g;
    const int64_t spatial = g->out_h * g->out_w;
    const int64_t reduction = g->cg * g->kh * g->kw;
    const int64_t m_per_group = g->m / g->group;
    float* columns = (float*)scratch; /* [reduction][spatial] as the reference */
    for (int64_t grp = 0; grp < g->group; ++grp) {
        /* im2col, conv2d_op.cpp:191-220 */
        int64_t row = 0;
        for (int64_t cl = 0; cl < g->cg; ++cl) {
            const int64_t ch = grp * g->cg + cl;
            const float* xc = k->x + (b * g->c + ch) * g->h * g->w;
            for (int64_t ky = 0; ky < g->kh; ++ky) {
                for (int64_t kx = 0; kx < g->kw; ++kx) {
                    float* col = columns + row * spatial;
                    for (int64_t oy = 0; oy < g->out_h; ++oy) {
                        const int64_t iy = oy * g->stride_h - g->pad_t + ky * g->dil_h;
                        for (int64_t ox = 0; ox < g->out_w; ++ox) {
                            const int64_t ix = ox * g->stride_w - g->pad_l + kx * g->dil_w;
                            float v = 0.0f;
                            if (iy >= 0 && iy < g->h && ix >= 0 && ix < g->w) {
                                v = xc[iy * g->w + ix];
                            }
                            col[oy * g->out_w + ox] = v;
                        }
                    }
                    ++row;
                }
            }
        }
        /* row dot products, conv2d_op.cpp:13-22 and :223-238 */
        for (int64_t ml = 0; ml < m_per_group; ++ml) {
            const int64_t mo = grp * m_per_group + ml;
            const float* wrow = k->wt + mo * reduction;
            float* out = k->y + (b * g->m + mo) * spatial;
            for (int64_t p = 0; p < spatial; ++p) {
                float acc = 0.0f;
                for (int64_t t = 0; t < reduction; ++t) {
                    acc += wrow[t] * columns[t * spatial + p];
                }
                out[p] = acc;
            }
            if (k->bias != NULL && k->bias[mo] != 0.0f) {
                const float bv = k->bias[mo];
                for (int64_t p = 0; p < spatial; ++p) out[p] += bv;
            }
            if (k->act == 1 || k->act == 2) {
                for (int64_t p = 0; p < spatial; ++p) {
                    float v = out[p];
                    v = v > 0.0f ? v : 0.0f;
                    if (k->act == 2 && v > 6.0f) v = 6.0f;
                    out[p] = v;
                }
            }
        }
    }
}

int orc_conv2d_f32(const orc_conv_geom* g, const float* x, const float* wt,
                   const float* bias, int act, float* y, int nthreads) {
    if (g == NULL || x == NULL || wt == NULL || y == NULL) {
        return ORC_INVALID_ARGUMENT;
    }
    orc_f32_ctx ctx = {g, x, wt, bias, act, y};
    const size_t scratch = (size_t)(g->cg * g->kh * g->kw) *
                           (size_t)(g->out_h * g->out_w) * sizeof(float);
    return orc_for_images(g->n, nthreads, scratch, orc_f32_image, &ctx);
}

/* ------------------------------------------------------------------- int8 */

/* Exact requantize: the fp32 multiplier is a dyadic rational mant * 2^-shift
 * (mant the 24-bit significand scaled to 31 bits), so t * mult is computed
 * exactly in 64-bit integers and rounded half away from zero once. */
static void orc_split_multiplier(float mult, int64_t* mant, int* shift) {
    if (mult == 0.0f || !isfinite(mult)) {
        *mant = 0;
        *shift = 32;
        return;
    }
    int e = 0;
    const double f = frexp((double)mult, &e);      /* mult = f * 2^e, 0.5 <= |f| < 1 */
    *mant = (int64_t)ldexp(f, 31);                  /* exact: f has 24 significant bits */
    *shift = 31 - e;                                /* mult = mant * 2^-shift */
}

int32_t orc_requantize(int32_t acc, int32_t bias, float mult, int32_t zp_y,
                       int32_t qmin, int32_t qmax) {
    const int32_t t = (int32_t)((uint32_t)acc + (uint32_t)bias);
    int64_t mant;
    int shift;
    orc_split_multiplier(mult, &mant, &shift);
    const int64_t p = (int64_t)t * mant;            /* |p| < 2^62 */
    int64_t r;
    if (shift >= 63) {
        r = 0;                                      /* |t * mult| < 1/2 */
    } else if (shift <= 0) {
        r = p == 0 ? 0 : (p > 0 ? INT64_C(1) << 40 : -(INT64_C(1) << 40));  /* saturates */
    } else {
        const int64_t half = INT64_C(1) << (shift - 1);
        /* floor((p + half - [p < 0]) / 2^shift) = round half away from zero */
        r = (p + half - (p < 0 ? 1 : 0)) >> shift;
    }
    int64_t q = r + zp_y;
    if (q < qmin) q = qmin;
    if (q > qmax) q = qmax;
    return (int32_t)q;
}

typedef struct {
    const orc_conv_geom* g;
    const void* x;
    int x_signed;
    int32_t zp_x;
    const int8_t* wt;
    const int32_t* bias;
    const float* mult;
    int32_t zp_y, qmin, qmax;
    int y_signed;
    void* y;
    int32_t* acc_out;
} orc_q8_ctx;

static void orc_q8_image(void* vctx, int64_t b, void* scratch) {
    const orc_q8_ctx* k = (const orc_q8_ctx*)vctx;
    const orc_conv_geom* g = k->g;
    const int64_t spatial = g->out_h * g->out_w;
    const int64_t reduction = g->cg * g->kh * g->kw;
    const int64_t m_per_group = g->m / g->group;
    /* Same im2col rows as conv2d_op.cpp:191-220, stored transposed
     * ([spatial][reduction]) so that each dot product runs over contiguous
     * memory; integer sums do not depend on the order. */
    int16_t* cols = (int16_t*)scratch;
    const uint8_t* xu = (const uint8_t*)k->x;
    const int8_t* xs = (const int8_t*)k->x;
    for (int64_t grp = 0; grp < g->group; ++grp) {
        int64_t row = 0;
        for (int64_t cl = 0; cl < g->cg; ++cl) {
            const int64_t ch = grp * g->cg + cl;
            const int64_t base = (b * g->c + ch) * g->h * g->w;
            for (int64_t ky = 0; ky < g->kh; ++ky) {
                for (int64_t kx = 0; kx < g->kw; ++kx) {
                    for (int64_t oy = 0; oy < g->out_h; ++oy) {
                        const int64_t iy = oy * g->stride_h - g->pad_t + ky * g->dil_h;
                        for (int64_t ox = 0; ox < g->out_w; ++ox) {
                            const int64_t ix = ox * g->stride_w - g->pad_l + kx * g->dil_w;
                            int32_t v = 0; /* padding is real 0.0 */
                            if (iy >= 0 && iy < g->h && ix >= 0 && ix < g->w) {
                                const int64_t at = base + iy * g->w + ix;
                                const int32_t q = k->x_signed ? (int32_t)xs[at]
                                                              : (int32_t)xu[at];
                                v = q - k->zp_x;
                            }
                            cols[(oy * g->out_w + ox) * reduction + row] = (int16_t)v;
                        }
                    }
                    ++row;
                }
            }
        }
        for (int64_t ml = 0; ml < m_per_group; ++ml) {
            const int64_t mo = grp * m_per_group + ml;
            const int8_t* wrow = k->wt + mo * reduction;
            const int64_t out_base = (b * g->m + mo) * spatial;
            const int32_t bv = k->bias != NULL ? k->bias[mo] : 0;
            const float mult = k->mult[mo];
            for (int64_t p = 0; p < spatial; ++p) {
                const int16_t* col = cols + p * reduction;
                int32_t acc = 0;
                for (int64_t t = 0; t < reduction; ++t) {
                    acc += (int32_t)col[t] * (int32_t)wrow[t];
                }
                if (k->acc_out != NULL) k->acc_out[out_base + p] = acc;
                const int32_t q = orc_requantize(acc, bv, mult, k->zp_y, k->qmin,
                                                 k->qmax);
                if (k->y_signed) {
                    ((int8_t*)k->y)[out_base + p] = (int8_t)q;
                } else {
                    ((uint8_t*)k->y)[out_base + p] = (uint8_t)q;
                }
            }
        }
    }
}

int orc_conv2d_q8(const orc_conv_geom* g, const void* x, int x_signed,
                  int32_t zp_x, const int8_t* wt, const int32_t* bias,
                  const float* mult, int32_t zp_y, int32_t qmin, int32_t qmax,
                  int y_signed, void* y, int32_t* acc_out, int nthreads) {
    if (g == NULL || x == NULL || wt == NULL || mult == NULL || y == NULL) {
        return ORC_INVALID_ARGUMENT;
    }
    const int32_t lo = y_signed ? -128 : 0;
    const int32_t hi = y_signed ? 127 : 255;
    if (qmin < lo || qmax > hi || qmin > qmax || zp_y < lo || zp_y > hi) {
        return ORC_INVALID_ARGUMENT;
    }
    orc_q8_ctx ctx = {g, x, x_signed, zp_x, wt, bias, mult, zp_y, qmin, qmax,
                      y_signed, y, acc_out};
    const size_t scratch = (size_t)(g->cg * g->kh * g->kw) *
                           (size_t)(g->out_h * g->out_w) * sizeof(int16_t);
    return orc_for_images(g->n, nthreads, scratch, orc_q8_image, &ctx);
}

int orc_qadd(const void* a, int a_signed, int32_t zp_a, float mult_a, const void* b,
             int b_signed, int32_t zp_b, float mult_b, int32_t zp_y, int32_t qmin,
             int32_t qmax, int y_signed, void* y, int64_t count) {
    if (count < 0 || (count > 0 && (a == NULL || b == NULL || y == NULL))) {
        return ORC_INVALID_ARGUMENT;
    }
    int64_t ma, mb;
    int sa, sb;
    orc_split_multiplier(mult_a, &ma, &sa);
    orc_split_multiplier(mult_b, &mb, &sb);
    if (ma == 0) sa = sb;  /* a vanishing term puts no constraint on the shift */
    if (mb == 0) sb = sa;
    const int s = sa > sb ? sa : sb;
    if (s - (sa < sb ? sa : sb) > 60) return ORC_UNSUPPORTED;
    for (int64_t i = 0; i < count; ++i) {
        const int32_t av = a_signed ? ((const int8_t*)a)[i] : ((const uint8_t*)a)[i];
        const int32_t bv = b_signed ? ((const int8_t*)b)[i] : ((const uint8_t*)b)[i];
        const __int128 v = ((__int128)(av - zp_a) * ma) * ((__int128)1 << (s - sa)) +
                           ((__int128)(bv - zp_b) * mb) * ((__int128)1 << (s - sb));
        int64_t r;
        if (s >= 127) {
            r = 0;                                   /* |v| < 2^103 <= 2^(s-1) */
        } else if (s <= 0) {
            r = v == 0 ? 0 : (v > 0 ? INT64_C(1) << 40 : -(INT64_C(1) << 40));
        } else {
            const __int128 half = (__int128)1 << (s - 1);
            r = (int64_t)((v + half - (v < 0 ? 1 : 0)) >> s);
        }
        int64_t q = r + zp_y;
        if (q < qmin) q = qmin;
        if (q > qmax) q = qmax;
        if (y_signed) {
            ((int8_t*)y)[i] = (int8_t)q;
        } else {
            ((uint8_t*)y)[i] = (uint8_t)q;
        }
    }
    return ORC_OK;
}
