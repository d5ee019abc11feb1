/*
 * C restatement of the reference's W8A8 accumulation loops (TEST INFRASTRUCTURE ONLY).
 *
 * Used by oracle/w8a8.py to make the CPU oracle fast enough for BASELINE-sized
 * parity cases and for the timed CPU baseline of bench.py.  Nothing in the
 * product links or loads this library.
 *
 * oracle_conv_acc_i32 restates the integer part of the prequant conv kernels
 * (reference native/aexrt_d3d12_runtime.cpp:4614-4762: acc = sum over input
 * channels and taps of int8 activation code x int8 weight code, zero padding),
 * with the activation in NCHW int8 and the weight in layout-8 order
 * [oc][ic][kh][kw] (src/aexrt/engine.py:2458).  Integer addition is exact and
 * associative, so the loop order here is free.
 *
 * oracle_conv_f32 is a plain fp32 convolution (no bias) for the fp16 stem and
 * detect head of the model-level oracle.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void oracle_conv_acc_i32(const int8_t* x, const int8_t* w, int32_t* out,
                         int n, int c, int h, int wd, int oc, int oh, int ow,
                         int k, int s, int p) {
    const int kk = k * k;
    const int kdim = c * kk;
    /* weights re-ordered to [oc][kh][kw][ic] so the inner loop runs over ic */
    int16_t* wt = (int16_t*)malloc(sizeof(int16_t) * (size_t)oc * kdim);
    for (int o = 0; o < oc; ++o)
        for (int ic = 0; ic < c; ++ic)
            for (int t = 0; t < kk; ++t)
                wt[(size_t)o * kdim + (size_t)t * c + ic] = w[(size_t)o * kdim + (size_t)ic * kk + t];
    /* activation widened to NHWC int16 with a zero border of p pixels */
    const int hp = h + 2 * p, wp = wd + 2 * p;
    int16_t* xp = (int16_t*)calloc((size_t)n * hp * wp * c, sizeof(int16_t));
    for (int b = 0; b < n; ++b)
        for (int ic = 0; ic < c; ++ic)
            for (int y = 0; y < h; ++y)
                for (int xx = 0; xx < wd; ++xx)
                    xp[(((size_t)b * hp + y + p) * wp + xx + p) * c + ic] =
                        x[(((size_t)b * c + ic) * h + y) * wd + xx];
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < n; ++b) {
        for (int y = 0; y < oh; ++y) {
            for (int xx = 0; xx < ow; ++xx) {
                for (int o = 0; o < oc; ++o) {
                    int32_t acc = 0;
                    const int16_t* wo = wt + (size_t)o * kdim;
                    for (int kh = 0; kh < k; ++kh) {
                        const int iy = y * s + kh;
                        for (int kw = 0; kw < k; ++kw) {
                            const int ix = xx * s + kw;
                            const int16_t* xv = xp + (((size_t)b * hp + iy) * wp + ix) * c;
                            const int16_t* wv = wo + (size_t)(kh * k + kw) * c;
                            int32_t part = 0;
                            for (int ic = 0; ic < c; ++ic) part += (int32_t)xv[ic] * (int32_t)wv[ic];
                            acc += part;
                        }
                    }
                    out[(((size_t)b * oc + o) * oh + y) * ow + xx] = acc;
                }
            }
        }
    }
    (void)clampi;
    free(xp);
    free(wt);
}

void oracle_conv_f32(const float* x, const float* w, float* out,
                     int n, int c, int h, int wd, int oc, int oh, int ow,
                     int k, int s, int p) {
    const int kk = k * k;
    const int kdim = c * kk;
    float* wt = (float*)malloc(sizeof(float) * (size_t)oc * kdim);
    for (int o = 0; o < oc; ++o)
        for (int ic = 0; ic < c; ++ic)
            for (int t = 0; t < kk; ++t)
                wt[(size_t)o * kdim + (size_t)t * c + ic] = w[(size_t)o * kdim + (size_t)ic * kk + t];
    const int hp = h + 2 * p, wp = wd + 2 * p;
    float* xp = (float*)calloc((size_t)n * hp * wp * c, sizeof(float));
    for (int b = 0; b < n; ++b)
        for (int ic = 0; ic < c; ++ic)
            for (int y = 0; y < h; ++y)
                for (int xx = 0; xx < wd; ++xx)
                    xp[(((size_t)b * hp + y + p) * wp + xx + p) * c + ic] =
                        x[(((size_t)b * c + ic) * h + y) * wd + xx];
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < n; ++b) {
        for (int y = 0; y < oh; ++y) {
            for (int xx = 0; xx < ow; ++xx) {
                for (int o = 0; o < oc; ++o) {
                    float acc = 0.0f;
                    const float* wo = wt + (size_t)o * kdim;
                    for (int kh = 0; kh < k; ++kh) {
                        for (int kw = 0; kw < k; ++kw) {
                            const float* xv = xp + (((size_t)b * hp + y * s + kh) * wp + xx * s + kw) * c;
                            const float* wv = wo + (size_t)(kh * k + kw) * c;
                            for (int ic = 0; ic < c; ++ic) acc += xv[ic] * wv[ic];
                        }
                    }
                    out[(((size_t)b * oc + o) * oh + y) * ow + xx] = acc;
                }
            }
        }
    }
    free(xp);
    free(wt);
}
