/*
 * c2s_oracle.c -- CPU restatement of the c2slm token loop (TEST INFRASTRUCTURE).
 *
 * This file is the parity checker for c2slm_b200; the product never links it.
 * Each function restates a scalar function of hazyhaar/c2slm in the
 * reference's own statement order (file:line cited).  Build flags: -O2
 * -ffp-contract=off, no -ffast-math: every float expression below rounds
 * exactly like the Go code on amd64 (which never fuses multiply-add).
 */
#define _GNU_SOURCE
#include "c2s_oracle.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* little-endian helpers                                                     */
/* ------------------------------------------------------------------------ */
static inline uint16_t rd_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline int16_t rd_i16(const uint8_t *p) { return (int16_t)rd_u16(p); }
static inline uint32_t rd_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* tensor/fp16.go:44-73 (computeFP16ToF32) */
float c2o_fp16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h >> 15)) << 31;
    uint32_t exp = (uint32_t)((h >> 10) & 0x1F);
    uint32_t mant = (uint32_t)(h & 0x3FF);
    if (exp == 0) {
        if (mant == 0) return f32_from_bits(sign);
        while ((mant & 0x400) == 0) { mant <<= 1; exp--; }
        exp++;
        mant &= 0x3FF;
        exp = (exp + (127 - 15)) << 23;
        mant <<= 13;
        return f32_from_bits(sign | exp | mant);
    }
    if (exp == 31) {
        if (mant == 0) return f32_from_bits(sign | 0x7F800000u);
        return f32_from_bits(sign | 0x7F800000u | (mant << 13));
    }
    exp = (exp + (127 - 15)) << 23;
    mant <<= 13;
    return f32_from_bits(sign | exp | mant);
}
#define FP16(p) c2o_fp16_to_f32(rd_u16(p))

/* ------------------------------------------------------------------------ */
/* Q8_K activation quantisation                                              */
/* internal/simd/c2_quantize_q8_k_gen.go:11-91                               */
/* Block (292 B): f32 d @0, int8 q[256] @4, int16 bsum[16] @260.             */
/* ------------------------------------------------------------------------ */
void c2o_quantize_row_q8_k(const float *x, uint8_t *y, int cols) {
    for (int b = 0; b < cols / 256; b++) {
        const float *xb = x + (size_t)b * 256;
        uint8_t *yb = y + (size_t)b * 292;
        float amax = 0;
        for (int i = 0; i < 256; i++) {
            float v = xb[i];
            float a = v < 0.0f ? -v : v;
            if (a > amax) amax = a;
        }
        if (amax == 0.0f) {
            /* the reference clears from this block to the end of the buffer;
             * later blocks are rewritten by their own iterations, so only this
             * block's bytes matter (:38-47) */
            memset(yb, 0, 292);
            continue;
        }
        uint32_t db = f32_to_bits(amax / 127.0f);
        yb[0] = (uint8_t)(db & 0xff);
        yb[1] = (uint8_t)((db >> 8) & 0xff);
        yb[2] = (uint8_t)((db >> 16) & 0xff);
        yb[3] = (uint8_t)((db >> 24) & 0xff);
        for (int i = 0; i < 256; i++) {
            float v = xb[i] * (127.0f / amax);
            float r = (v >= 0.0f) ? (v + 0.5f) : (v - 0.5f);
            int q = (int)r; /* Go int(float32) truncates toward zero */
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            yb[4 + i] = (uint8_t)(int8_t)q;
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int k = 0; k < 16; k++) s += (int)(int8_t)yb[4 + g * 16 + k];
            yb[260 + g * 2] = (uint8_t)(s & 255);
            yb[260 + g * 2 + 1] = (uint8_t)((s >> 8) & 255);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q4_K x Q8_K                                                               */
/* internal/simd/c2_tensor_dot_q4_k_q8_k_nosimd_gen.go:15-74 (single row) and */
/* c2_tensor_gemv2_q4_k_q8_k_nosimd_gen.go:7-106 (row pair).  Both evaluate   */
/* the same per-row expression tree, so one helper serves both.               */
/* ------------------------------------------------------------------------ */
static inline void q4k_unpack_scales(const uint8_t *s, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (uint8_t)((s[j + 8] & 15) | ((s[j] >> 6) << 4));
        mn[j + 4] = (uint8_t)((s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4));
    }
}

static float q4k_q8k_row(const uint8_t *w, const uint8_t *q8k, int cols,
                         int32_t *dots_out /* nsb*8 or NULL */) {
    float acc = 0;
    for (int b = 0; b < cols / 256; b++) {
        const uint8_t *wb = w + (size_t)b * 144;
        const uint8_t *qb = q8k + (size_t)b * 292;
        float d8 = f32_from_bits(rd_u32(qb));
        float dd = FP16(wb) * d8;       /* v428 */
        float dm = FP16(wb + 2) * d8;   /* v442 */
        uint8_t sc[8], mn[8];
        q4k_unpack_scales(wb + 4, sc, mn);
        for (int j = 0; j < 4; j++) {
            int32_t lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                uint8_t v = wb[16 + j * 32 + l];
                lo += (int32_t)(v & 15) * (int32_t)(int8_t)qb[4 + j * 64 + l];
                hi += (int32_t)(v >> 4) * (int32_t)(int8_t)qb[4 + j * 64 + 32 + l];
            }
            if (dots_out) { dots_out[b * 8 + 2 * j] = lo; dots_out[b * 8 + 2 * j + 1] = hi; }
            const uint8_t *bs = qb + 260;
            float bs01 = (float)((int32_t)rd_i16(bs + (4 * j) * 2) + (int32_t)rd_i16(bs + (4 * j + 1) * 2));
            float bs23 = (float)((int32_t)rd_i16(bs + (4 * j + 2) * 2) + (int32_t)rd_i16(bs + (4 * j + 3) * 2));
            acc += (((float)lo * (dd * (float)sc[2 * j])) - (bs01 * (dm * (float)mn[2 * j]))) +
                   (((float)hi * (dd * (float)sc[2 * j + 1])) - (bs23 * (dm * (float)mn[2 * j + 1])));
        }
    }
    return acc;
}

float c2o_dot_q4_k_q8_k(const uint8_t *w, const uint8_t *q8k, int cols) {
    return q4k_q8k_row(w, q8k, cols, NULL);
}

void c2o_gemv2_q4_k_q8_k(const uint8_t *w0, const uint8_t *w1, const uint8_t *q8k,
                         int cols, float *out0, float *out1) {
    *out0 = q4k_q8k_row(w0, q8k, cols, NULL);
    *out1 = q4k_q8k_row(w1, q8k, cols, NULL);
}

/* ------------------------------------------------------------------------ */
/* Q6_K x Q8_K: internal/simd/c2_tensor_gemv2_q6_k_q8_k_nosimd_gen.go:12-246 */
/* Block (210 B): ql[128] @0, qh[64] @128, int8 sc[16] @192, fp16 d @208.    */
/* ------------------------------------------------------------------------ */
static inline int q6k_val(const uint8_t *ql, const uint8_t *qh, int k, int l) {
    uint8_t qlb = (k == 0 || k == 2) ? ql[l] : ql[32 + l];
    uint8_t qhb = qh[l];
    switch (k) {
    case 0: return (qlb & 15) | ((qhb & 3) << 4);
    case 1: return (qlb & 15) | (((qhb >> 2) & 3) << 4);
    case 2: return (qlb >> 4) | (((qhb >> 4) & 3) << 4);
    default: return (qlb >> 4) | (((qhb >> 6) & 3) << 4);
    }
}

static float q6k_q8k_row(const uint8_t *w, const uint8_t *q8k, int cols, int32_t *isum_out) {
    float acc = 0;
    for (int b = 0; b < cols / 256; b++) {
        const uint8_t *wb = w + (size_t)b * 210;
        const uint8_t *qb = q8k + (size_t)b * 292;
        float d8 = f32_from_bits(rd_u32(qb));
        float d6 = FP16(wb + 208);
        int32_t isum = 0;
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = wb + n * 64;
            const uint8_t *qh = wb + 128 + n * 32;
            const int8_t *sc = (const int8_t *)(wb + 192 + n * 8);
            const uint8_t *q8 = qb + 4 + n * 128;
            const uint8_t *bs = qb + 260 + n * 16;
            for (int k = 0; k < 4; k++) {
                int32_t s0 = 0, s1 = 0;
                for (int l = 0; l < 16; l++)
                    s0 += (int32_t)q6k_val(ql, qh, k, l) * (int32_t)(int8_t)q8[k * 32 + l];
                for (int l = 16; l < 32; l++)
                    s1 += (int32_t)q6k_val(ql, qh, k, l) * (int32_t)(int8_t)q8[k * 32 + l];
                int32_t sc0 = sc[2 * k], sc1 = sc[2 * k + 1];
                int32_t b0 = 32 * (int32_t)rd_i16(bs + (2 * k) * 2);
                int32_t b1 = 32 * (int32_t)rd_i16(bs + (2 * k + 1) * 2);
                isum += ((s0 - b0) * sc0) + ((s1 - b1) * sc1);
            }
        }
        if (isum_out) isum_out[b] = isum;
        acc += (float)isum * (d6 * d8);
    }
    return acc;
}

void c2o_gemv2_q6_k_q8_k(const uint8_t *w0, const uint8_t *w1, const uint8_t *q8k,
                         int cols, float *out0, float *out1) {
    *out0 = q6k_q8k_row(w0, q8k, cols, NULL);
    *out1 = q6k_q8k_row(w1, q8k, cols, NULL);
}

void c2o_q4k_q8k_partials(const uint8_t *w, const uint8_t *q8k, int rows, int cols,
                          int32_t *dots, int32_t *bsum_pairs) {
    int nsb = cols / 256;
    size_t rb = (size_t)nsb * 144;
    for (int r = 0; r < rows; r++) q4k_q8k_row(w + r * rb, q8k, cols, dots + (size_t)r * nsb * 8);
    for (int b = 0; b < nsb; b++) {
        const uint8_t *bs = q8k + (size_t)b * 292 + 260;
        for (int j = 0; j < 4; j++)
            bsum_pairs[b * 4 + j] = (int32_t)rd_i16(bs + (2 * j) * 2) + (int32_t)rd_i16(bs + (2 * j + 1) * 2);
    }
}

void c2o_q6k_q8k_partials(const uint8_t *w, const uint8_t *q8k, int rows, int cols, int32_t *isum) {
    int nsb = cols / 256;
    size_t rb = (size_t)nsb * 210;
    for (int r = 0; r < rows; r++) q6k_q8k_row(w + r * rb, q8k, cols, isum + (size_t)r * nsb);
}

/* ------------------------------------------------------------------------ */
/* f32-activation dots                                                      */
/* ------------------------------------------------------------------------ */
/* tensor/ops.go:40-74 (DotQ5_0, plain scalar Go; no SIMD twin) */
float c2o_dot_q5_0(const uint8_t *w, const float *x, int cols) {
    float total = 0;
    for (int b = 0; b < cols / 32; b++) {
        const uint8_t *wb = w + (size_t)b * 22;
        float d = FP16(wb);
        uint32_t qh = rd_u32(wb + 2);
        const uint8_t *qs = wb + 6;
        const float *xb = x + (size_t)b * 32;
        float sum = 0;
        for (int i = 0; i < 16; i++) {
            uint8_t x0 = qs[i] & 0x0F, x1 = qs[i] >> 4;
            uint8_t h0 = (uint8_t)((qh >> i) & 1), h1 = (uint8_t)((qh >> (i + 16)) & 1);
            float q0 = (float)((int32_t)(x0 | (h0 << 4)) - 16);
            float q1 = (float)((int32_t)(x1 | (h1 << 4)) - 16);
            sum += q0 * xb[i];
            sum += q1 * xb[i + 16];
        }
        total += d * sum;
    }
    return total;
}

/* internal/simd/c2_tensor_dot_q8_0_nosimd_gen.go:68-91 (8 lane accumulators) */
float c2o_dot_q8_0(const uint8_t *w, const float *x, int cols) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < cols / 32; b++) {
        const uint8_t *wb = w + (size_t)b * 34;
        float d = FP16(wb);
        const int8_t *q = (const int8_t *)(wb + 2);
        const float *xb = x + (size_t)b * 32;
        for (int k = 0; k < 8; k++) {
            lane[k] += ((((float)q[k] * xb[k]) + ((float)q[k + 8] * xb[k + 8])) +
                        (((float)q[k + 16] * xb[k + 16]) + ((float)q[k + 24] * xb[k + 24]))) * d;
        }
    }
    return ((((((lane[0] + lane[1]) + lane[2]) + lane[3]) + lane[4]) + lane[5]) + lane[6]) + lane[7];
}

/* internal/simd/c2_tensor_dot_q4_k_nosimd_gen.go:7-74 */
float c2o_dot_q4_k(const uint8_t *w, const float *x, int cols) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < cols / 256; b++) {
        const uint8_t *wb = w + (size_t)b * 144;
        float d = FP16(wb), dmin = FP16(wb + 2);
        uint8_t sc[8], mn[8];
        q4k_unpack_scales(wb + 4, sc, mn);
        for (int j = 0; j < 4; j++) {
            const float *xl = x + (size_t)b * 256 + j * 64;
            const float *xh = xl + 32;
            const uint8_t *qs = wb + 16 + j * 32;
            for (int t = 0; t < 8; t++) {
                uint8_t b0 = qs[t], b1 = qs[t + 8], b2 = qs[t + 16], b3 = qs[t + 24];
                float x0 = xl[t], x1 = xl[t + 8], x2 = xl[t + 16], x3 = xl[t + 24];
                float y0 = xh[t], y1 = xh[t + 8], y2 = xh[t + 16], y3 = xh[t + 24];
                lane[t] += (((((float)(b0 & 15) * x0) + ((float)(b1 & 15) * x1)) +
                             (((float)(b2 & 15) * x2) + ((float)(b3 & 15) * x3))) * (d * (float)sc[2 * j])) -
                           (((x0 + x1) + (x2 + x3)) * (dmin * (float)mn[2 * j]));
                lane[t] += (((((float)(b0 >> 4) * y0) + ((float)(b1 >> 4) * y1)) +
                             (((float)(b2 >> 4) * y2) + ((float)(b3 >> 4) * y3))) * (d * (float)sc[2 * j + 1])) -
                           (((y0 + y1) + (y2 + y3)) * (dmin * (float)mn[2 * j + 1]));
            }
        }
    }
    return ((((((lane[0] + lane[1]) + lane[2]) + lane[3]) + lane[4]) + lane[5]) + lane[6]) + lane[7];
}

/* internal/simd/c2_tensor_dot_q6_k_nosimd_gen.go:7-84 */
float c2o_dot_q6_k(const uint8_t *w, const float *x, int cols) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < cols / 256; b++) {
        const uint8_t *wb = w + (size_t)b * 210;
        float d = FP16(wb + 208);
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = wb + n * 64;
            const uint8_t *qh = wb + 128 + n * 32;
            const int8_t *sc = (const int8_t *)(wb + 192 + n * 8);
            const float *xb = x + (size_t)b * 256 + n * 128;
            float a0[8] = {0}, a1[8] = {0}, a2[8] = {0}, a3[8] = {0};
            for (int t2 = 0; t2 < 2; t2++) {
                float ds0 = d * (float)sc[t2], ds1 = d * (float)sc[t2 + 2];
                float ds2 = d * (float)sc[t2 + 4], ds3 = d * (float)sc[t2 + 6];
                for (int t = 0; t < 8; t++) {
                    int i0 = t2 * 16 + t, i1 = t2 * 16 + 8 + t;
                    uint8_t h0 = qh[i0], h1 = qh[i1];
                    uint8_t l0 = ql[i0], l1 = ql[i1], l0b = ql[i0 + 32], l1b = ql[i1 + 32];
                    a0[t] += (((float)((int)((l0 & 15) | ((h0 & 3) << 4)) - 32) * ds0) * xb[i0]) +
                             (((float)((int)((l1 & 15) | ((h1 & 3) << 4)) - 32) * ds0) * xb[i1]);
                    a1[t] += (((float)((int)((l0b & 15) | (((h0 >> 2) & 3) << 4)) - 32) * ds1) * xb[i0 + 32]) +
                             (((float)((int)((l1b & 15) | (((h1 >> 2) & 3) << 4)) - 32) * ds1) * xb[i1 + 32]);
                    a2[t] += (((float)((int)((l0 >> 4) | (((h0 >> 4) & 3) << 4)) - 32) * ds2) * xb[i0 + 64]) +
                             (((float)((int)((l1 >> 4) | (((h1 >> 4) & 3) << 4)) - 32) * ds2) * xb[i1 + 64]);
                    a3[t] += (((float)((int)((l0b >> 4) | (((h0 >> 6) & 3) << 4)) - 32) * ds3) * xb[i0 + 96]) +
                             (((float)((int)((l1b >> 4) | (((h1 >> 6) & 3) << 4)) - 32) * ds3) * xb[i1 + 96]);
                }
            }
            for (int t = 0; t < 8; t++) lane[t] += ((a0[t] + a1[t]) + (a2[t] + a3[t]));
        }
    }
    return ((((((lane[0] + lane[1]) + lane[2]) + lane[3]) + lane[4]) + lane[5]) + lane[6]) + lane[7];
}

/* ------------------------------------------------------------------------ */
/* Row dequantisation (token embedding), tensor/ops.go:342-424               */
/* ------------------------------------------------------------------------ */
static void dequant_q4_k(const uint8_t *data, float *dst, int cols) {  /* ops.go:342-380 */
    for (int b = 0; b < cols / 256; b++) {
        const uint8_t *wb = data + (size_t)b * 144;
        float d = FP16(wb), dmin = FP16(wb + 2);
        uint8_t sc[8], mn[8];
        q4k_unpack_scales(wb + 4, sc, mn);
        const uint8_t *qs = wb + 16;
        for (int sb = 0; sb < 4; sb++) {
            float d0 = d * (float)sc[2 * sb], m0 = dmin * (float)mn[2 * sb];
            float d1 = d * (float)sc[2 * sb + 1], m1 = dmin * (float)mn[2 * sb + 1];
            float *o = dst + (size_t)b * 256 + sb * 64;
            for (int l = 0; l < 32; l++) {
                uint8_t v = qs[sb * 32 + l];
                o[l] = d0 * (float)(v & 0x0F) - m0;
                o[l + 32] = d1 * (float)(v >> 4) - m1;
            }
        }
    }
}

static void dequant_q5_0(const uint8_t *data, float *dst, int cols) {  /* ops.go:383-409 */
    for (int b = 0; b < cols / 32; b++) {
        const uint8_t *wb = data + (size_t)b * 22;
        float d = FP16(wb);
        uint32_t qh = rd_u32(wb + 2);
        const uint8_t *qs = wb + 6;
        for (int i = 0; i < 16; i++) {
            uint8_t x0 = qs[i] & 0x0F, x1 = qs[i] >> 4;
            uint8_t h0 = (uint8_t)((qh >> i) & 1), h1 = (uint8_t)((qh >> (i + 16)) & 1);
            dst[b * 32 + i] = d * (float)((int32_t)(x0 | (h0 << 4)) - 16);
            dst[b * 32 + i + 16] = d * (float)((int32_t)(x1 | (h1 << 4)) - 16);
        }
    }
}

static void dequant_q8_0(const uint8_t *data, float *dst, int cols) {  /* ops.go:412-424 */
    for (int b = 0; b < cols / 32; b++) {
        const uint8_t *wb = data + (size_t)b * 34;
        float d = FP16(wb);
        for (int i = 0; i < 32; i++) dst[b * 32 + i] = d * (float)(int8_t)wb[2 + i];
    }
}

/* Q6_K row dequant: the reference has no Q6_K embedding case
 * (engine/model.go:221-247).  This follows the dequant written in the
 * reference's own test oracle, tensor/oracle_q6_k_test.go:62-94:
 * dst = d * (float)sc * (float)q, evaluated left to right.                  */
static void dequant_q6_k(const uint8_t *data, float *dst, int cols) {
    for (int b = 0; b < cols / 256; b++) {
        const uint8_t *wb = data + (size_t)b * 210;
        float d = FP16(wb + 208);
        for (int n = 0; n < 2; n++) {
            const uint8_t *ql = wb + n * 64, *qh = wb + 128 + n * 32;
            const int8_t *sc = (const int8_t *)(wb + 192 + n * 8);
            float *o = dst + (size_t)b * 256 + n * 128;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                uint8_t h = qh[l];
                int8_t q0 = (int8_t)((ql[l] & 0xF) | (((h >> 0) & 3) << 4)) - 32;
                int8_t q1 = (int8_t)((ql[l + 32] & 0xF) | (((h >> 2) & 3) << 4)) - 32;
                int8_t q2 = (int8_t)((ql[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
                int8_t q3 = (int8_t)((ql[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
                o[l] = d * (float)sc[is + 0] * (float)q0;
                o[l + 32] = d * (float)sc[is + 2] * (float)q1;
                o[l + 64] = d * (float)sc[is + 4] * (float)q2;
                o[l + 96] = d * (float)sc[is + 6] * (float)q3;
            }
        }
    }
}

int c2o_dequant_row(int type, const uint8_t *row, float *out, int cols) {
    switch (type) {
    case C2O_Q4_K: dequant_q4_k(row, out, cols); return 0;
    case C2O_Q5_0: dequant_q5_0(row, out, cols); return 0;
    case C2O_Q8_0: dequant_q8_0(row, out, cols); return 0;
    case C2O_Q6_K: dequant_q6_k(row, out, cols); return 0;
    case C2O_F32:  /* engine/model.go:238-245 */
        for (int i = 0; i < cols; i++) out[i] = f32_from_bits(rd_u32(row + 4 * i));
        return 0;
    default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* Elementwise / normalisation / attention                                  */
/* ------------------------------------------------------------------------ */
/* tensor/ops.go:207-218 */
void c2o_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    float sumsq = 0;
    for (int i = 0; i < n; i++) sumsq += x[i] * x[i];
    float inv = (float)(1.0 / sqrt((double)(sumsq / (float)n + eps)));
    for (int i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* tensor/ops.go:221-225 */
void c2o_add_bias(float *x, const float *bias, int n) {
    for (int i = 0; i < n; i++) x[i] += bias[i];
}

/* tensor/ops.go:237-257 (angles in float64, stored as float32) */
void c2o_rope_table(float *cos_t, float *sin_t, int max_len, int head_dim, float theta) {
    int half = head_dim / 2;
    for (int p = 0; p < max_len; p++) {
        for (int i = 0; i < half; i++) {
            double freq = 1.0 / pow((double)theta, (double)(2 * i) / (double)head_dim);
            double val = (double)p * freq;
            cos_t[(size_t)p * half + i] = (float)cos(val);
            sin_t[(size_t)p * half + i] = (float)sin(val);
        }
    }
}

/* tensor/ops.go:262-286 (guards reject out-of-range pos and oversized heads) */
void c2o_rope_apply(const float *cos_t, const float *sin_t, int max_len, int head_dim,
                    float *vec, int vec_len, int num_heads, int pos) {
    if (pos < 0 || pos >= max_len) return;
    if (num_heads <= 0 || num_heads * head_dim > vec_len) return;
    int half = head_dim / 2;
    const float *c = cos_t + (size_t)pos * half;
    const float *s = sin_t + (size_t)pos * half;
    for (int h = 0; h < num_heads; h++) {
        float *v = vec + h * head_dim;
        for (int i = 0; i < half; i++) {
            float x0 = v[i], x1 = v[i + half];
            v[i] = x0 * c[i] - x1 * s[i];
            v[i + half] = x0 * s[i] + x1 * c[i];
        }
    }
}

/* tensor/ops.go:292-309 */
void c2o_rope_neox(float *vec, int num_heads, int head_dim, int pos, float theta) {
    int half = head_dim / 2;
    for (int h = 0; h < num_heads; h++) {
        float *v = vec + h * head_dim;
        for (int i = 0; i < half; i++) {
            double freq = 1.0 / pow((double)theta, (double)(2 * i) / (double)head_dim);
            double val = (double)pos * freq;
            float c = (float)cos(val), s = (float)sin(val);
            float x0 = v[i], x1 = v[i + half];
            v[i] = x0 * c - x1 * s;
            v[i + half] = x0 * s + x1 * c;
        }
    }
}

/* tensor/ops.go:317-339 */
void c2o_softmax(float *x, int n) {
    if (n <= 0) return;
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0;
    for (int i = 0; i < n; i++) {
        float e = (float)exp((double)(x[i] - mx));
        x[i] = e;
        sum += e;
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* internal/simd/c2_tensor_swiglu_nosimd_gen.go:11-19 */
void c2o_swiglu(float *out, const float *gate, const float *up, int n) {
    for (int i = 0; i < n; i++) {
        double g = (double)gate[i];
        float silu = (float)(g / (1.0 + exp(-g)));
        out[i] = silu * up[i];
    }
}

/* internal/simd/c2_tensor_attn_nosimd_gen.go:7-24 */
void c2o_attn_qk(const float *q, const float *kbase, int pos, int stride, float scale,
                 float *scores, int hd) {
    for (int p = 0; p <= pos; p++) {
        float acc = 0;
        for (int d = 0; d < hd; d++) acc += q[d] * kbase[(size_t)p * stride + d];
        scores[p] = acc * scale;
    }
}

/* internal/simd/c2_tensor_attn_nosimd_gen.go:26-39 */
void c2o_attn_av(const float *scores, const float *vbase, int pos, int stride,
                 float *out, int hd) {
    for (int d = 0; d < hd; d++) {
        float acc = 0;
        for (int p = 0; p <= pos; p++) acc += scores[p] * vbase[(size_t)p * stride + d];
        out[d] = acc;
    }
}

/* ------------------------------------------------------------------------ */
/* The reference's AVX2 build (GOEXPERIMENT=simd) evaluates three kernels of  */
/* the 0.5B path in a different float order than the scalar twins above:     */
/* attention QK and AV use fused multiply-add, SwiGLU uses a polynomial exp.  */
/* Restated here so the scalar and SIMD builds of the reference can be        */
/* compared with each other.                                                  */
/* ------------------------------------------------------------------------ */
/* internal/simd/c2_tensor_attn_gen.go:9-58 (AVX2 branch; hd % 8 == 0) */
void c2o_attn_qk_simd(const float *q, const float *kbase, int pos, int stride, float scale,
                      float *scores, int hd) {
    for (int p = 0; p <= pos; p++) {
        const float *k = kbase + (size_t)p * stride;
        float a[8] = {0}, b[8] = {0};
        int d = 0;
        for (; d + 16 <= hd; d += 16)
            for (int i = 0; i < 8; i++) {
                a[i] = fmaf(q[d + i], k[d + i], a[i]);
                b[i] = fmaf(q[d + 8 + i], k[d + 8 + i], b[i]);
            }
        for (; d + 8 <= hd; d += 8)
            for (int i = 0; i < 8; i++) a[i] = fmaf(q[d + i], k[d + i], a[i]);
        float v[8];
        for (int i = 0; i < 8; i++) v[i] = a[i] + b[i];
        float acc = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        for (; d < hd; d++) acc += q[d] * k[d];
        scores[p] = acc * scale;
    }
}

/* internal/simd/c2_tensor_attn_gen.go:68-112 (AVX2 branch): per output
 * element, sequential over positions with fused multiply-add. */
void c2o_attn_av_simd(const float *scores, const float *vbase, int pos, int stride,
                      float *out, int hd) {
    const int dv = hd - hd % 8;  /* 8-wide vector columns; the rest is scalar */
    for (int d = 0; d < hd; d++) {
        float acc = 0;
        if (d < dv)
            for (int p = 0; p <= pos; p++) acc = fmaf(scores[p], vbase[(size_t)p * stride + d], acc);
        else
            for (int p = 0; p <= pos; p++) acc += scores[p] * vbase[(size_t)p * stride + d];
        out[d] = acc;
    }
}

/* internal/simd/c2_tensor_swiglu_gen.go:11-57 (AVX2 branch, 8 at a time;
 * tail in float64 like the scalar twin).  Truncating float->int conversion. */
static float bitsf(uint32_t u) { return f32_from_bits(u); }
void c2o_swiglu_simd(float *out, const float *gate, const float *up, int n) {
    const float half = bitsf(0x3f000000u), one = bitsf(0x3f800000u);
    const float inv_ln2 = bitsf(0x3fb8aa3bu), ln2 = bitsf(0x3f317218u);
    const float c5 = bitsf(0x3c088888u), c4 = bitsf(0x3d2aaaabu), c3 = bitsf(0x3e2aaaabu);
    const int nv = n - n % 8;  /* 8-wide vector part; the tail is scalar */
    int i = 0;
    for (; i < nv; i++) {
        float x = gate[i];
        float nx = -x;
        float nf = nx * inv_ln2;
        /* x86 cvttps2dq returns INT32_MIN for out-of-range input */
        float fp = nf + half, fn = nf - half;
        int npos = (fp >= -2147483648.0f && fp < 2147483648.0f) ? (int)fp : INT32_MIN;
        int nneg = (fn >= -2147483648.0f && fn < 2147483648.0f) ? (int)fn : INT32_MIN;
        int ni = nf >= 0.0f ? npos : nneg;
        if (ni < -126) ni = -126;
        if (ni > 127) ni = 127;
        float nif = (float)ni;
        float r = nx - nif * ln2;
        float p = ((((c5 * r + c4) * r + c3) * r + half) * r + one) * r + one;
        float scl = f32_from_bits((uint32_t)(ni + 127) << 23);
        float ev = p * scl;
        float den = one + ev;
        float sig = one / den;
        float silu = x * sig;
        out[i] = silu * up[i];
    }
    for (; i < n; i++) {
        double g = (double)gate[i];
        float silu = (float)(g / (1.0 + exp(-g)));
        out[i] = silu * up[i];
    }
}

/* ------------------------------------------------------------------------ */
/* Worker pool: engine/pool.go:16-154,180-208.                              */
/* n persistent workers; the caller publishes a task and waits.              */
/* ------------------------------------------------------------------------ */
typedef struct {
    int n;
    pthread_t *tid;
    pthread_mutex_t mu;
    pthread_cond_t cv_start, cv_done;
    unsigned long gen;
    int pending;
    int quit;
    void (*fn)(void *arg, int worker, int nworkers);
    void *arg;
} c2o_pool;

typedef struct { c2o_pool *p; int id; } c2o_worker_arg;

static void *pool_main(void *varg) {
    c2o_worker_arg *wa = (c2o_worker_arg *)varg;
    c2o_pool *p = wa->p;
    int id = wa->id;
    free(wa);
    unsigned long seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        while (!p->quit && p->gen == seen) pthread_cond_wait(&p->cv_start, &p->mu);
        if (p->quit) { pthread_mutex_unlock(&p->mu); return NULL; }
        seen = p->gen;
        void (*fn)(void *, int, int) = p->fn;
        void *arg = p->arg;
        pthread_mutex_unlock(&p->mu);
        fn(arg, id, p->n);
        pthread_mutex_lock(&p->mu);
        if (--p->pending == 0) pthread_cond_signal(&p->cv_done);
        pthread_mutex_unlock(&p->mu);
    }
}

static c2o_pool *pool_new(int n) {
    if (n <= 1) return NULL;
    if (n > 32) n = 32;  /* engine/pool.go:51-53 */
    c2o_pool *p = (c2o_pool *)calloc(1, sizeof(*p));
    p->n = n;
    p->tid = (pthread_t *)calloc((size_t)n, sizeof(pthread_t));
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv_start, NULL);
    pthread_cond_init(&p->cv_done, NULL);
    for (int i = 0; i < n; i++) {
        c2o_worker_arg *wa = (c2o_worker_arg *)malloc(sizeof(*wa));
        wa->p = p;
        wa->id = i;
        pthread_create(&p->tid[i], NULL, pool_main, wa);
    }
    return p;
}

static void pool_run(c2o_pool *p, void (*fn)(void *, int, int), void *arg) {
    pthread_mutex_lock(&p->mu);
    p->fn = fn;
    p->arg = arg;
    p->pending = p->n;
    p->gen++;
    pthread_cond_broadcast(&p->cv_start);
    while (p->pending > 0) pthread_cond_wait(&p->cv_done, &p->mu);
    pthread_mutex_unlock(&p->mu);
}

static void pool_free(c2o_pool *p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->quit = 1;
    pthread_cond_broadcast(&p->cv_start);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->n; i++) pthread_join(p->tid[i], NULL);
    free(p->tid);
    free(p);
}

/* ------------------------------------------------------------------------ */
/* GEMV dispatch: engine/pool.go:122-154 + tensor/ops.go range drivers       */
/* ------------------------------------------------------------------------ */
static size_t row_bytes(int type, int cols) {
    switch (type) {
    case C2O_Q5_0: return (size_t)(cols / 32) * 22;
    case C2O_Q8_0: return (size_t)(cols / 32) * 34;
    case C2O_Q4_K: return (size_t)(cols / 256) * 144;
    case C2O_Q6_K: return (size_t)(cols / 256) * 210;
    case C2O_F32:  return (size_t)cols * 4;
    default: return 0;
    }
}

/* rows [r0, r1); the K-quant drivers go pairwise (tensor/ops.go:120-141,
 * 182-198) -- each row's value is the same expression in the pair and the
 * single-row kernel, so the result is computed per row.                   */
static void gemv_range(int type, const uint8_t *w, const float *x, const uint8_t *q8k,
                       float *y, int r0, int r1, int cols) {
    size_t rb = row_bytes(type, cols);
    for (int r = r0; r < r1; r++) {
        const uint8_t *row = w + (size_t)r * rb;
        switch (type) {
        case C2O_Q8_0: y[r] = c2o_dot_q8_0(row, x, cols); break;
        case C2O_Q5_0: y[r] = c2o_dot_q5_0(row, x, cols); break;
        case C2O_Q6_K: y[r] = q6k_q8k_row(row, q8k, cols, NULL); break;
        case C2O_Q4_K: y[r] = q4k_q8k_row(row, q8k, cols, NULL); break;
        default: break;  /* unknown types leave y untouched (engine/pool.go:318-327) */
        }
    }
}

typedef struct {
    int type; const uint8_t *w; const float *x; const uint8_t *q8k; float *y; int rows, cols;
} gemv_task;

static void gemv_worker(void *arg, int wid, int nw) {
    gemv_task *t = (gemv_task *)arg;
    int r0 = (int)(((long)wid * t->rows) / nw);           /* engine/pool.go:98-99 */
    int r1 = (int)(((long)(wid + 1) * t->rows) / nw);
    if (r0 < r1 && r0 < t->rows) {
        if (r1 > t->rows) r1 = t->rows;
        gemv_range(t->type, t->w, t->x, t->q8k, t->y, r0, r1, t->cols);
    }
}

static int gemv_pool(c2o_pool *pool, int type, const uint8_t *w, const float *x, float *y,
                     int rows, int cols, uint8_t *q8k) {
    if (type == C2O_Q4_K || type == C2O_Q6_K) {
        if (!q8k) return -1;
        c2o_quantize_row_q8_k(x, q8k, cols);              /* engine/pool.go:123-125 */
    }
    if (!pool || rows < 256) {                             /* engine/pool.go:127-139 */
        gemv_range(type, w, x, q8k, y, 0, rows, cols);
        return 0;
    }
    gemv_task t = {type, w, x, q8k, y, rows, cols};
    pool_run(pool, gemv_worker, &t);
    return 0;
}

int c2o_gemv(int type, const uint8_t *w, const float *x, float *y, int rows, int cols,
             uint8_t *q8k_scratch, int nthreads) {
    c2o_pool *pool = pool_new(nthreads);
    int rc = gemv_pool(pool, type, w, x, y, rows, cols, q8k_scratch);
    pool_free(pool);
    return rc;
}

/* engine/model.go:255-269 (pool-less DispatchGEMV: f32-x dots for every type) */
int c2o_gemv_f32x(int type, const uint8_t *w, const float *x, float *y, int rows, int cols) {
    size_t rb = row_bytes(type, cols);
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = w + (size_t)r * rb;
        switch (type) {
        case C2O_Q5_0: y[r] = c2o_dot_q5_0(row, x, cols); break;
        case C2O_Q8_0: y[r] = c2o_dot_q8_0(row, x, cols); break;
        case C2O_Q6_K: y[r] = c2o_dot_q6_k(row, x, cols); break;
        case C2O_Q4_K: y[r] = c2o_dot_q4_k(row, x, cols); break;
        default: y[r] = 0; break;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* GGUF parsing: gguf/reader.go:394-546                                      */
/* ------------------------------------------------------------------------ */
typedef struct {
    char name[96];
    uint64_t dims[4];
    uint32_t n_dims;
    uint32_t type;
    uint64_t offset;
    const uint8_t *data;
    uint64_t nbytes;
} c2o_tensor;

typedef struct {
    char key[96];
    uint32_t vtype;
    union { uint64_t u; int64_t i; double f; } v;
} c2o_kv;

typedef struct {
    const uint8_t *map;
    size_t size;
    size_t pos;
    int bad;
} rd_t;

static int rd_need(rd_t *r, size_t n) { if (r->pos + n > r->size) { r->bad = 1; return 0; } return 1; }
static uint8_t rd8(rd_t *r) { if (!rd_need(r, 1)) return 0; return r->map[r->pos++]; }
static uint32_t rd32(rd_t *r) { if (!rd_need(r, 4)) return 0; uint32_t v = rd_u32(r->map + r->pos); r->pos += 4; return v; }
static uint64_t rd64(rd_t *r) {
    if (!rd_need(r, 8)) return 0;
    uint64_t v = (uint64_t)rd_u32(r->map + r->pos) | ((uint64_t)rd_u32(r->map + r->pos + 4) << 32);
    r->pos += 8;
    return v;
}
static const uint8_t *rdstr(rd_t *r, uint64_t *len) {
    *len = rd64(r);
    if (r->bad || !rd_need(r, *len)) return NULL;
    const uint8_t *s = r->map + r->pos;
    r->pos += *len;
    return s;
}

struct c2o_model {
    /* mapping */
    uint8_t *map; size_t map_size;
    c2o_tensor *tensors; int n_tensors;
    c2o_kv *kvs; int n_kvs;
    /* hyper-parameters (engine/model.go:64-148) */
    int embd, n_layers, n_heads, n_kv, hd, ffn, vocab;
    float rope_base, eps;
    int max_tokens;
    int32_t im_end, eos;
    /* weights */
    const c2o_tensor *tok_embd, *output;
    const float *out_norm;
    struct {
        const float *attn_norm, *q_b, *k_b, *v_b, *q_norm, *k_norm, *ffn_norm;
        int n_q_b, n_k_b, n_v_b;            /* AddBias iterates over len(bias) */
        const c2o_tensor *q, *k, *v, *o, *gate, *up, *down;
    } *layers;
    float *rope_cos, *rope_sin; int rope_len;
    /* KV cache [2][L][KVH][max_tokens][hd] (engine/kvcache.go:31,127-140) */
    float *kv;
    int32_t *token_ids;
    int seq_len;
    /* arena (engine/forward.go:12-43) */
    float *X, *NormX, *Q, *K, *V, *scores, *AttnOut, *Gate, *Up, *Down, *Logits;
    uint8_t *q8k;
    float *attn_scratch; /* per worker scores for parallel heads */
    c2o_pool *pool;
    int nthreads;
    int simd_order;      /* 1: restate the reference's AVX2 build */
};

static void set_err(char *err, int errlen, const char *fmt, ...) {
    if (!err || errlen <= 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
}

static int skip_value(rd_t *r, uint32_t vt, c2o_kv *kv, int depth);

static int skip_value(rd_t *r, uint32_t vt, c2o_kv *kv, int depth) {
    uint64_t len;
    switch (vt) {
    case 0: kv->v.u = rd8(r); break;
    case 1: kv->v.i = (int8_t)rd8(r); break;
    case 2: if (rd_need(r, 2)) { kv->v.u = rd_u16(r->map + r->pos); r->pos += 2; } break;
    case 3: if (rd_need(r, 2)) { kv->v.i = rd_i16(r->map + r->pos); r->pos += 2; } break;
    case 4: kv->v.u = rd32(r); break;
    case 5: kv->v.i = (int32_t)rd32(r); break;
    case 6: { uint32_t b = rd32(r); kv->v.f = (double)f32_from_bits(b); } break;
    case 7: kv->v.u = rd8(r); break;
    case 8: rdstr(r, &len); break;
    case 9: {
        if (depth > 4) { r->bad = 1; return -1; }
        uint32_t et = rd32(r);
        uint64_t n = rd64(r);
        c2o_kv tmp;
        for (uint64_t i = 0; i < n && !r->bad; i++) skip_value(r, et, &tmp, depth + 1);
    } break;
    case 10: kv->v.u = rd64(r); break;
    case 11: kv->v.i = (int64_t)rd64(r); break;
    case 12: { uint64_t b = rd64(r); double d; memcpy(&d, &b, 8); kv->v.f = d; } break;
    default: r->bad = 1; return -1;
    }
    return r->bad ? -1 : 0;
}

static uint64_t tensor_nbytes(uint32_t type, const uint64_t *dims, uint32_t nd) {
    if (nd == 0) return 0;
    uint64_t n = 1;
    for (uint32_t i = 0; i < nd; i++) n *= dims[i];
    switch (type) {  /* gguf/reader.go:513-546 */
    case 0: return n * 4;
    case 1: return n * 2;
    case 2: return (n / 32) * 18;
    case 6: return (n / 32) * 22;
    case 8: return (n / 32) * 34;
    case 12: return (n / 256) * 144;
    case 14: return (n / 256) * 210;
    default: return n * 4;
    }
}

/* GetUint32 (gguf/reader.go:559-576): u32, u64, i32, i64 accepted */
static int kv_u32(const c2o_model *m, const char *key, uint32_t *out) {
    for (int i = 0; i < m->n_kvs; i++) {
        if (strcmp(m->kvs[i].key, key) != 0) continue;
        switch (m->kvs[i].vtype) {
        case 4: case 10: *out = (uint32_t)m->kvs[i].v.u; return 1;
        case 5: case 11: *out = (uint32_t)m->kvs[i].v.i; return 1;
        default: return 0;
        }
    }
    return 0;
}

/* GetFloat32 (gguf/reader.go:579-592): f32 and f64 accepted */
static int kv_f32(const c2o_model *m, const char *key, float *out) {
    for (int i = 0; i < m->n_kvs; i++) {
        if (strcmp(m->kvs[i].key, key) != 0) continue;
        if (m->kvs[i].vtype == 6 || m->kvs[i].vtype == 12) { *out = (float)m->kvs[i].v.f; return 1; }
        return 0;
    }
    return 0;
}

static const c2o_tensor *find_tensor(const c2o_model *m, const char *name) {
    for (int i = 0; i < m->n_tensors; i++)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

static int parse_gguf(c2o_model *m, char *err, int errlen) {
    rd_t r = {m->map, m->map_size, 0, 0};
    uint32_t magic = rd32(&r);
    if (magic != 0x46554747u) { set_err(err, errlen, "invalid GGUF magic 0x%08x", magic); return -1; }
    uint32_t version = rd32(&r);
    if (version < 2 || version > 3) { set_err(err, errlen, "unsupported GGUF version %u", version); return -1; }
    uint64_t n_t = rd64(&r), n_kv = rd64(&r);
    if (r.bad || n_t > 1000000 || n_kv > 1000000) { set_err(err, errlen, "bad GGUF header"); return -1; }
    m->kvs = (c2o_kv *)calloc(n_kv ? n_kv : 1, sizeof(c2o_kv));
    m->n_kvs = (int)n_kv;
    m->im_end = 0;
    m->eos = 0;
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; i++) {
        uint64_t klen;
        const uint8_t *k = rdstr(&r, &klen);
        if (!k) { set_err(err, errlen, "metadata[%llu] key truncated", (unsigned long long)i); return -1; }
        c2o_kv *kv = &m->kvs[i];
        size_t cl = klen < sizeof(kv->key) - 1 ? klen : sizeof(kv->key) - 1;
        memcpy(kv->key, k, cl);
        kv->key[cl] = 0;
        kv->vtype = rd32(&r);
        if (kv->vtype == 9 && strcmp(kv->key, "tokenizer.ggml.tokens") == 0) {
            /* special ids: tokenizer/bpe.go:50-58 indexes "<|...|>" tokens;
             * SpecialTokenIDs (:284-289) returns 0 for an absent name */
            uint32_t et = rd32(&r);
            uint64_t n = rd64(&r);
            if (et != 8) { set_err(err, errlen, "tokenizer.ggml.tokens is not a string array"); return -1; }
            for (uint64_t t = 0; t < n && !r.bad; t++) {
                uint64_t sl;
                const uint8_t *s = rdstr(&r, &sl);
                if (!s) break;
                if (sl == 10 && memcmp(s, "<|im_end|>", 10) == 0) m->im_end = (int32_t)t;
                if (sl == 13 && memcmp(s, "<|endoftext|>", 13) == 0) m->eos = (int32_t)t;
            }
        } else if (skip_value(&r, kv->vtype, kv, 0) != 0) {
            set_err(err, errlen, "metadata[%s] value unreadable", kv->key);
            return -1;
        }
        if (strcmp(kv->key, "general.alignment") == 0) {
            if (kv->vtype == 4 || kv->vtype == 10) alignment = kv->v.u;
        }
        if (r.bad) { set_err(err, errlen, "metadata truncated"); return -1; }
    }
    if (alignment == 0) alignment = 32;
    m->tensors = (c2o_tensor *)calloc(n_t ? n_t : 1, sizeof(c2o_tensor));
    m->n_tensors = (int)n_t;
    for (uint64_t i = 0; i < n_t; i++) {
        c2o_tensor *t = &m->tensors[i];
        uint64_t nl;
        const uint8_t *nm = rdstr(&r, &nl);
        if (!nm) { set_err(err, errlen, "tensor[%llu] name truncated", (unsigned long long)i); return -1; }
        size_t cl = nl < sizeof(t->name) - 1 ? nl : sizeof(t->name) - 1;
        memcpy(t->name, nm, cl);
        t->name[cl] = 0;
        t->n_dims = rd32(&r);
        if (t->n_dims > 4) { set_err(err, errlen, "tensor[%s] has %u dims", t->name, t->n_dims); return -1; }
        for (uint32_t d = 0; d < t->n_dims; d++) t->dims[d] = rd64(&r);
        t->type = rd32(&r);
        t->offset = rd64(&r);
        if (r.bad) { set_err(err, errlen, "tensor infos truncated"); return -1; }
    }
    size_t pad = r.pos % alignment;
    if (pad) r.pos += alignment - pad;
    size_t data_off = r.pos;
    for (int i = 0; i < m->n_tensors; i++) {
        c2o_tensor *t = &m->tensors[i];
        t->nbytes = tensor_nbytes(t->type, t->dims, t->n_dims);
        if (data_off + t->offset + t->nbytes > m->map_size) {
            set_err(err, errlen, "tensor[%s] data out of range", t->name);
            return -1;
        }
        t->data = m->map + data_off + t->offset;
    }
    return 0;
}

static const float *f32_data(const c2o_tensor *t) { return t ? (const float *)t->data : NULL; }
static uint64_t tensor_len(const c2o_tensor *t) { return t ? t->nbytes / 4 : 0; }

c2o_model *c2o_model_open(const char *path, int max_tokens, int nthreads, char *err, int errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { set_err(err, errlen, "open %s: %s", path, strerror(errno)); return NULL; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        set_err(err, errlen, "gguf: file too small");
        close(fd);
        return NULL;
    }
    void *mp = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_SHARED | MAP_POPULATE, fd, 0);
    close(fd);
    if (mp == MAP_FAILED) { set_err(err, errlen, "mmap failed"); return NULL; }
    c2o_model *m = (c2o_model *)calloc(1, sizeof(*m));
    m->map = (uint8_t *)mp;
    m->map_size = (size_t)st.st_size;
    if (parse_gguf(m, err, errlen) != 0) { c2o_model_close(m); return NULL; }

    /* engine/model.go:64-112: qwen2.* then qwen3.* then defaults */
    uint32_t u;
#define HP(field, k2, k3, dflt) \
    do { u = 0; kv_u32(m, k2, &u); if (u == 0) kv_u32(m, k3, &u); if (u == 0) u = dflt; m->field = (int)u; } while (0)
    HP(embd, "qwen2.embedding_length", "qwen3.embedding_length", 896);
    HP(n_layers, "qwen2.block_count", "qwen3.block_count", 24);
    HP(n_heads, "qwen2.attention.head_count", "qwen3.attention.head_count", 14);
    HP(n_kv, "qwen2.attention.head_count_kv", "qwen3.attention.head_count_kv", 2);
    HP(ffn, "qwen2.feed_forward_length", "qwen3.feed_forward_length", 4864);
#undef HP
    float f = 0;
    kv_f32(m, "qwen2.rope.freq_base", &f);
    if (f == 0) kv_f32(m, "qwen3.rope.freq_base", &f);
    if (f == 0) f = 1000000.0f;
    m->rope_base = f;
    f = 0;
    kv_f32(m, "qwen2.attention.layer_norm_rms_epsilon", &f);
    if (f == 0) kv_f32(m, "qwen3.attention.layer_norm_rms_epsilon", &f);
    if (f == 0) f = 1e-6f;
    m->eps = f;

    m->tok_embd = find_tensor(m, "token_embd.weight");
    if (!m->tok_embd || m->tok_embd->n_dims < 2) { set_err(err, errlen, "missing token_embd.weight"); c2o_model_close(m); return NULL; }
    m->vocab = (int)m->tok_embd->dims[1];
    const c2o_tensor *on = find_tensor(m, "output_norm.weight");
    if (!on) { set_err(err, errlen, "missing output_norm.weight"); c2o_model_close(m); return NULL; }
    m->out_norm = f32_data(on);
    m->output = find_tensor(m, "output.weight");
    if (!m->output) m->output = m->tok_embd;           /* tied fallback, model.go:126-130 */
    m->hd = m->embd / m->n_heads;

    m->layers = calloc((size_t)m->n_layers, sizeof(*m->layers));
    char nm[96];
    for (int i = 0; i < m->n_layers; i++) {
#define T(name) (snprintf(nm, sizeof nm, "blk.%d." name, i), find_tensor(m, nm))
        const c2o_tensor *an = T("attn_norm.weight");
        if (!an) { set_err(err, errlen, "missing blk.%d.attn_norm.weight", i); c2o_model_close(m); return NULL; }
        m->layers[i].attn_norm = f32_data(an);
        m->layers[i].q = T("attn_q.weight");
        m->layers[i].q_b = f32_data(T("attn_q.bias"));
        m->layers[i].n_q_b = (int)tensor_len(T("attn_q.bias"));
        m->layers[i].q_norm = f32_data(T("attn_q_norm.weight"));
        m->layers[i].k = T("attn_k.weight");
        m->layers[i].k_b = f32_data(T("attn_k.bias"));
        m->layers[i].n_k_b = (int)tensor_len(T("attn_k.bias"));
        m->layers[i].k_norm = f32_data(T("attn_k_norm.weight"));
        m->layers[i].v = T("attn_v.weight");
        m->layers[i].v_b = f32_data(T("attn_v.bias"));
        m->layers[i].n_v_b = (int)tensor_len(T("attn_v.bias"));
        m->layers[i].o = T("attn_output.weight");
        m->layers[i].ffn_norm = f32_data(T("ffn_norm.weight"));
        m->layers[i].gate = T("ffn_gate.weight");
        m->layers[i].up = T("ffn_up.weight");
        m->layers[i].down = T("ffn_down.weight");
#undef T
        if (!m->layers[i].q || !m->layers[i].k || !m->layers[i].v || !m->layers[i].o ||
            !m->layers[i].gate || !m->layers[i].up || !m->layers[i].down || !m->layers[i].ffn_norm) {
            set_err(err, errlen, "blk.%d is missing a projection or norm tensor", i);
            c2o_model_close(m);
            return NULL;
        }
    }
    /* RoPE table over MaxContextLen positions (engine/model.go:145) */
    m->rope_len = 16384;
    size_t rt = (size_t)m->rope_len * (m->hd / 2);
    m->rope_cos = (float *)malloc(rt * sizeof(float));
    m->rope_sin = (float *)malloc(rt * sizeof(float));
    c2o_rope_table(m->rope_cos, m->rope_sin, m->rope_len, m->hd, m->rope_base);

    if (max_tokens <= 0) max_tokens = 16384;
    m->max_tokens = max_tokens;
    size_t kvn = (size_t)2 * m->n_layers * m->n_kv * (size_t)max_tokens * m->hd;
    m->kv = (float *)calloc(kvn, sizeof(float));
    m->token_ids = (int32_t *)calloc((size_t)max_tokens, sizeof(int32_t));
    if (!m->kv || !m->token_ids) { set_err(err, errlen, "KV cache allocation failed"); c2o_model_close(m); return NULL; }
    int kvd = m->n_kv * m->hd;
    m->X = calloc((size_t)m->embd, 4);
    m->NormX = calloc((size_t)m->embd, 4);
    m->Q = calloc((size_t)(m->embd > m->n_heads * m->hd ? m->embd : m->n_heads * m->hd), 4);
    m->K = calloc((size_t)kvd, 4);
    m->V = calloc((size_t)kvd, 4);
    m->scores = calloc((size_t)max_tokens, 4);
    m->AttnOut = calloc((size_t)(m->embd > m->n_heads * m->hd ? m->embd : m->n_heads * m->hd), 4);
    m->Gate = calloc((size_t)m->ffn, 4);
    m->Up = calloc((size_t)m->ffn, 4);
    m->Down = calloc((size_t)m->embd, 4);
    m->Logits = calloc((size_t)m->vocab, 4);
    int maxcols = m->ffn > m->embd ? m->ffn : m->embd;
    m->q8k = calloc((size_t)(maxcols / 256 + 1) * 292, 1);   /* sized from cols */
    m->nthreads = nthreads < 1 ? 1 : (nthreads > 32 ? 32 : nthreads);
    m->attn_scratch = calloc((size_t)m->nthreads * max_tokens, 4);
    m->pool = pool_new(m->nthreads);
    return m;
}

void c2o_model_close(c2o_model *m) {
    if (!m) return;
    pool_free(m->pool);
    if (m->map) munmap(m->map, m->map_size);
    free(m->tensors); free(m->kvs); free(m->layers);
    free(m->rope_cos); free(m->rope_sin);
    free(m->kv); free(m->token_ids);
    free(m->X); free(m->NormX); free(m->Q); free(m->K); free(m->V); free(m->scores);
    free(m->AttnOut); free(m->Gate); free(m->Up); free(m->Down); free(m->Logits);
    free(m->q8k); free(m->attn_scratch);
    free(m);
}

void c2o_model_get_info(const c2o_model *m, c2o_model_info *info) {
    info->embd = m->embd; info->n_layers = m->n_layers; info->n_heads = m->n_heads;
    info->n_kv_heads = m->n_kv; info->head_dim = m->hd; info->ffn = m->ffn; info->vocab = m->vocab;
    info->rope_base = m->rope_base; info->eps = m->eps; info->max_tokens = m->max_tokens;
    info->im_end = m->im_end; info->eos = m->eos; info->tied_output = (m->output == m->tok_embd);
}

/* engine/kvcache.go:127-140 */
static size_t kv_off(const c2o_model *m, int is_v, int layer, int kvh, int pos) {
    size_t head_group = (size_t)m->max_tokens * m->hd;
    size_t layer_stride = (size_t)m->n_kv * head_group;
    size_t kv_stride = (size_t)m->n_layers * layer_stride;
    return (is_v ? kv_stride : 0) + (size_t)layer * layer_stride + (size_t)kvh * head_group + (size_t)pos * m->hd;
}

/* engine/kvcache.go:143-158 (out-of-range pos is ignored) */
static void store_kv(c2o_model *m, int layer, int pos, const float *k, const float *v) {
    if (pos < 0 || pos >= m->max_tokens) return;
    for (int h = 0; h < m->n_kv; h++) {
        memcpy(m->kv + kv_off(m, 0, layer, h, pos), k + h * m->hd, (size_t)m->hd * 4);
        memcpy(m->kv + kv_off(m, 1, layer, h, pos), v + h * m->hd, (size_t)m->hd * 4);
    }
}

/* engine/model.go:221-247 (+ Q6_K) */
static void embed_token(c2o_model *m, float *out, int32_t tok) {
    if (tok >= m->vocab || tok < 0) tok = 0;
    size_t rb = row_bytes((int)m->tok_embd->type, m->embd);
    c2o_dequant_row((int)m->tok_embd->type, m->tok_embd->data + (size_t)tok * rb, out, m->embd);
}

typedef struct { c2o_model *m; int layer, pos; float scale; } attn_task;

/* engine/forward.go:143-155 */
static void attention_head(c2o_model *m, int layer, int pos, int h, float scale, float *scores) {
    int qperkv = m->n_heads / m->n_kv;
    int kvh = h / qperkv;
    const float *q = m->Q + h * m->hd;
    const float *kb = m->kv + kv_off(m, 0, layer, kvh, 0);
    const float *vb = m->kv + kv_off(m, 1, layer, kvh, 0);
    if (m->simd_order) c2o_attn_qk_simd(q, kb, pos, m->hd, scale, scores, m->hd);
    else c2o_attn_qk(q, kb, pos, m->hd, scale, scores, m->hd);
    c2o_softmax(scores, pos + 1);
    if (m->simd_order) c2o_attn_av_simd(scores, vb, pos, m->hd, m->AttnOut + h * m->hd, m->hd);
    else c2o_attn_av(scores, vb, pos, m->hd, m->AttnOut + h * m->hd, m->hd);
}

static void attn_worker(void *arg, int wid, int nw) {  /* engine/pool.go:159-175 */
    attn_task *t = (attn_task *)arg;
    c2o_model *m = t->m;
    int h0 = (wid * m->n_heads) / nw, h1 = ((wid + 1) * m->n_heads) / nw;
    if (h0 >= m->n_heads) return;
    if (h1 > m->n_heads) h1 = m->n_heads;
    float *scr = m->attn_scratch + (size_t)wid * m->max_tokens;
    for (int h = h0; h < h1; h++) attention_head(m, t->layer, t->pos, h, t->scale, scr);
}

/* engine/pool.go:180-208 (heads in parallel only when pos >= 256) */
static void dispatch_attention(c2o_model *m, int layer, int pos, float scale) {
    if (!m->pool || m->n_heads < 2 || pos < 256) {
        for (int h = 0; h < m->n_heads; h++) attention_head(m, layer, pos, h, scale, m->scores);
        return;
    }
    attn_task t = {m, layer, pos, scale};
    pool_run(m->pool, attn_worker, &t);
}

static void gemv_t(c2o_model *m, float *y, const c2o_tensor *t, const float *x, int rows, int cols) {
    gemv_pool(m->pool, (int)t->type, t->data, x, y, rows, cols, m->q8k);
}

/* engine/forward.go:54-138 */
void c2o_forward(c2o_model *m, int32_t token, int pos, float *normx_out) {
    embed_token(m, m->X, token);
    int hd = m->hd, kvh = m->n_kv, H = m->embd;
    float scale = (float)(1.0 / sqrt((double)hd));
    for (int l = 0; l < m->n_layers; l++) {
        c2o_rmsnorm(m->NormX, m->X, m->layers[l].attn_norm, H, m->eps);
        gemv_t(m, m->Q, m->layers[l].q, m->NormX, H, H);
        if (m->layers[l].q_b) c2o_add_bias(m->Q, m->layers[l].q_b, m->layers[l].n_q_b);
        gemv_t(m, m->K, m->layers[l].k, m->NormX, kvh * hd, H);
        if (m->layers[l].k_b) c2o_add_bias(m->K, m->layers[l].k_b, m->layers[l].n_k_b);
        gemv_t(m, m->V, m->layers[l].v, m->NormX, kvh * hd, H);
        if (m->layers[l].v_b) c2o_add_bias(m->V, m->layers[l].v_b, m->layers[l].n_v_b);
        if (m->layers[l].q_norm)
            for (int h = 0; h < m->n_heads; h++) c2o_rmsnorm(m->Q + h * hd, m->Q + h * hd, m->layers[l].q_norm, hd, m->eps);
        if (m->layers[l].k_norm)
            for (int h = 0; h < kvh; h++) c2o_rmsnorm(m->K + h * hd, m->K + h * hd, m->layers[l].k_norm, hd, m->eps);
        c2o_rope_apply(m->rope_cos, m->rope_sin, m->rope_len, hd, m->Q, H, m->n_heads, pos);
        c2o_rope_apply(m->rope_cos, m->rope_sin, m->rope_len, hd, m->K, kvh * hd, kvh, pos);
        store_kv(m, l, pos, m->K, m->V);
        dispatch_attention(m, l, pos, scale);
        gemv_t(m, m->Down, m->layers[l].o, m->AttnOut, H, H);
        for (int i = 0; i < H; i++) m->X[i] += m->Down[i];
        c2o_rmsnorm(m->NormX, m->X, m->layers[l].ffn_norm, H, m->eps);
        gemv_t(m, m->Gate, m->layers[l].gate, m->NormX, m->ffn, H);
        gemv_t(m, m->Up, m->layers[l].up, m->NormX, m->ffn, H);
        if (m->simd_order) c2o_swiglu_simd(m->Gate, m->Gate, m->Up, m->ffn);
        else c2o_swiglu(m->Gate, m->Gate, m->Up, m->ffn);
        gemv_t(m, m->Down, m->layers[l].down, m->Gate, H, m->ffn);
        for (int i = 0; i < H; i++) m->X[i] += m->Down[i];
    }
    c2o_rmsnorm(m->NormX, m->X, m->out_norm, H, m->eps);
    if (normx_out) memcpy(normx_out, m->NormX, (size_t)H * 4);
}

/* engine/forward.go:171-212 */
void c2o_compute_logits(c2o_model *m, const float *normx, float *out,
                        const int32_t *targets, int n_targets) {
    int cols = m->embd;
    if (n_targets > 0) {
        size_t rb = row_bytes((int)m->output->type, cols);
        for (int i = 0; i < n_targets; i++) {
            int32_t t = targets[i];
            if (t >= m->vocab || t < 0) continue;
            const uint8_t *row = m->output->data + (size_t)t * rb;
            float v = 0;
            switch (m->output->type) {  /* computeSingleTokenLogit, :193-212 */
            case C2O_Q8_0: v = c2o_dot_q8_0(row, normx, cols); break;
            case C2O_Q5_0: v = c2o_dot_q5_0(row, normx, cols); break;
            case C2O_Q6_K: v = c2o_dot_q6_k(row, normx, cols); break;
            case C2O_Q4_K: v = c2o_dot_q4_k(row, normx, cols); break;
            default: v = 0; break;
            }
            out[t] = v;
        }
        return;
    }
    gemv_t(m, out, m->output, normx, m->vocab, cols);
}

/* c2slm.go:156-180: penalty over TokenIDs[cur_pos-window, cur_pos) skipping
 * imEnd/eos, then strict-> argmax from id 0 (ties keep the lowest id).     */
int32_t c2o_select(c2o_model *m, float *logits, int cur_pos, float penalty, int window) {
    int start = cur_pos - window;
    if (start < 0) start = 0;
    for (int p = start; p < cur_pos; p++) {
        int32_t tok = m->token_ids[p];
        if (tok >= 0 && tok < m->vocab && tok != m->im_end && tok != m->eos) {
            if (logits[tok] > 0) logits[tok] /= penalty;
            else logits[tok] *= penalty;
        }
    }
    int32_t best = 0;
    float bv = logits[0];
    for (int id = 1; id < m->vocab; id++)
        if (logits[id] > bv) { bv = logits[id]; best = id; }
    return best;
}

void c2o_model_set_simd_order(c2o_model *m, int on) { m->simd_order = on ? 1 : 0; }

int c2o_kv_seq_len(const c2o_model *m) { return m->seq_len; }
void c2o_kv_set_seq_len(c2o_model *m, int n) { m->seq_len = n; }
void c2o_kv_reset(c2o_model *m) { m->seq_len = 0; }                 /* kvcache.go:101-103 */
void c2o_kv_rewind(c2o_model *m, int n) {                           /* kvcache.go:109-117 */
    if (n < 0) n = 0;
    if (n > m->seq_len) n = m->seq_len;
    m->seq_len -= n;
}
void c2o_kv_store_token_id(c2o_model *m, int pos, int32_t tok) {    /* kvcache.go:120-125 */
    if (pos < 0 || pos >= m->max_tokens) return;
    m->token_ids[pos] = tok;
}
int32_t c2o_kv_token_id(const c2o_model *m, int pos) {
    if (pos < 0 || pos >= m->max_tokens) return -1;
    return m->token_ids[pos];
}
void c2o_kv_get(const c2o_model *m, int is_v, int layer, int kv_head, int pos, float *out) {
    memcpy(out, m->kv + kv_off(m, is_v, layer, kv_head, pos), (size_t)m->hd * 4);
}

/* c2slm.go:92-115 */
int c2o_ingest_from(c2o_model *m, int pos, const int32_t *tokens, int n, float *normx_out) {
    if (n <= 0) return 0;
    if (pos < 0) pos = 0;
    if (pos > m->seq_len) pos = m->seq_len;
    if (pos < m->seq_len) c2o_kv_rewind(m, m->seq_len - pos);
    int done = 0;
    for (int i = 0; i < n; i++) {
        int p = pos + i;
        if (p >= m->max_tokens) break;
        c2o_forward(m, tokens[i], p, normx_out);
        c2o_kv_store_token_id(m, p, tokens[i]);
        m->seq_len = p + 1;
        done++;
    }
    return done;
}

/* c2slm.go:144-223 on token ids (decode/callback/stop strings stay host-side) */
int c2o_generate(c2o_model *m, const float *last_normx, int max_new, float penalty,
                 int window, int stop_on_special, int32_t *tokens_out,
                 float *margins_out, float *maxabs_out) {
    int cur = m->seq_len;
    float *normx = (float *)malloc((size_t)m->embd * 4);
    memcpy(normx, last_normx, (size_t)m->embd * 4);
    int n = 0;
    for (int step = 0; step < max_new; step++) {
        if (cur >= m->max_tokens) break;
        c2o_compute_logits(m, normx, m->Logits, NULL, 0);
        int32_t best = c2o_select(m, m->Logits, cur, penalty, window);
        if (margins_out || maxabs_out) {
            float b1 = m->Logits[best], b2 = -INFINITY, mx = 0;
            for (int i = 0; i < m->vocab; i++) {
                float a = fabsf(m->Logits[i]);
                if (a > mx) mx = a;
                if (i != best && m->Logits[i] > b2) b2 = m->Logits[i];
            }
            if (margins_out) margins_out[n] = b1 - b2;
            if (maxabs_out) maxabs_out[n] = mx;
        }
        tokens_out[n++] = best;
        if (stop_on_special && (best == m->im_end || best == m->eos)) {
            c2o_forward(m, best, cur, normx);
            c2o_kv_store_token_id(m, cur, best);
            cur++;
            m->seq_len = cur;
            break;
        }
        c2o_forward(m, best, cur, normx);
        c2o_kv_store_token_id(m, cur, best);
        cur++;
        m->seq_len = cur;
    }
    free(normx);
    return n;
}
