/*
 * vxo_kquant.c — CPU oracle for the K-quant weight types (TEST
 * INFRASTRUCTURE ONLY; see vxo.h).
 *
 * Restates, in plain C, the reference's K-quant block decoding
 * (src/quantize.c:116-250 and :423-437) and its GEMV dispatch for these
 * types (src/model.c:222-233 -> src/quantize.c:439-576):
 *
 *   vxo_dequant_kquant  the reference's vx_dequantize_row_* per type
 *   vxo_gemv_kquant     y = dequant(W) . x, one sequential fp32 sum per row
 *                       over 256-element super-blocks: the reference's
 *                       blockwise GEMV (src/quantize.c:486-505), which is
 *                       what it runs for Q5_K, Q6_K and Q8_K
 *   vxo_gemv_kquant_shipped  the reference's primary path for Q2_K, Q3_K and
 *                       Q4_K: activations quantised to Q8_K blocks
 *                       (src/quantize.c:252-287), integer dot products per
 *                       super-block (:289-421), sequential fp32 sum per row
 *
 * The two GEMVs differ for the same inputs: the Q8_K path rounds the
 * activations to int8, its Q4_K dot accumulates only 16 of every 32 elements
 * per scale (128 of 256 per super-block), and its Q2_K dot decodes the GGML
 * Q2_K layout, not the one vx_dequantize_row_q2_K decodes.  The device path
 * targets vxo_gemv_kquant; tests/test_kquant_cpu.py pins both restatements
 * bit for bit against the reference build.
 *
 * Block layouts are the reference's (include/quantize.h:47-93), restated
 * here as byte offsets.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "vxo.h"

#define QK 256

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

size_t vxo_kquant_block_bytes(int type) {
    switch (type) {
    case 10: return 84;    /* Q2_K: scales[16] qs[64] d dmin */
    case 11: return 110;   /* Q3_K: hmask[32] qs[64] scales[12] d */
    case 12: return 144;   /* Q4_K: d dmin scales[12] qs[128] */
    case 13: return 176;   /* Q5_K: d dmin scales[12] qh[32] qs[128] */
    case 14: return 210;   /* Q6_K: ql[128] qh[64] scales[16] d */
    case 15: return 292;   /* Q8_K: float d, qs[256], int16 bsums[16] */
    default: return 0;
    }
}

/* 6-bit scale and min j of a Q4_K / Q5_K super-block (src/quantize.c:180-188). */
static void scale_min_k4(int j, const uint8_t *s, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Signed 6-bit scale j of a Q3_K super-block: low nibble from bytes 0..7,
 * two high bits from bytes 8..11 (the unpacking of src/quantize.c:150-155). */
static int scale_q3k(int j, const uint8_t *s) {
    const int lo = j < 8 ? (s[j] & 0xF) : (s[j - 8] >> 4);
    const int hi = (s[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
    return (int)(int8_t)(uint8_t)(lo | (hi << 4)) - 32;
}

/* ---- dequantisation, one super-block of 256 ---- */

/* src/quantize.c:116-135 (not the GGML Q2_K layout: signed 4-bit scales
 * sc - 8, values v - 0.5, and every sub-block reads qs[0..3]). */
static void deq_q2k(const uint8_t *b, float *y) {
    const uint8_t *scales = b, *qs = b + 16;
    const float d = vxo_fp16_to_fp32(rd16(b + 80)) * 1.0f, dmin = vxo_fp16_to_fp32(rd16(b + 82)) * 1.0f;
    for (int j = 0; j < 16; j++) {
        const int sv = (j & 1) ? (scales[j / 2] >> 4) : (scales[j / 2] & 0xF);
        const float dl = d * (float)(sv - 8), ml = dmin * (float)(sv - 8);
        for (int l = 0; l < 16; l++) {
            const int v = (qs[l / 4] >> (2 * (l % 4))) & 3;
            y[j * 16 + l] = dl * ((float)v - 0.5f) + ml;
        }
    }
}

/* src/quantize.c:137-178: element n0 + 32j + l of each 128-half takes bits
 * 2j of qs[32 * half + l], minus 4 unless hmask bit 4 * half + j is set. */
static void deq_q3k(const uint8_t *b, float *y) {
    const uint8_t *hm = b, *qs = b + 32, *sc = b + 96;
    const float d = vxo_fp16_to_fp32(rd16(b + 108));
    for (int half = 0; half < 2; half++)
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 32; l++) {
                const int is = half * 8 + 2 * j + (l >= 16);
                const float dl = d * (float)(scale_q3k(is, sc));
                const int q = (qs[half * 32 + l] >> (2 * j)) & 3;
                const int hbit = (hm[l] >> (4 * half + j)) & 1;
                y[half * 128 + j * 32 + l] = dl * (float)(q - (hbit ? 0 : 4));
            }
}

/* src/quantize.c:190-212: four groups of 64; low nibbles with scale/min 2g,
 * high nibbles with 2g + 1. */
static void deq_q4k(const uint8_t *b, float *y) {
    const float d = vxo_fp16_to_fp32(rd16(b)), mn = vxo_fp16_to_fp32(rd16(b + 2));
    const uint8_t *s = b + 4, *q = b + 16;
    for (int g = 0; g < 4; g++) {
        int sc, m;
        scale_min_k4(2 * g, s, &sc, &m);
        const float d1 = d * (float)sc, m1 = mn * (float)m;
        scale_min_k4(2 * g + 1, s, &sc, &m);
        const float d2 = d * (float)sc, m2 = mn * (float)m;
        for (int l = 0; l < 32; l++) y[64 * g + l] = d1 * (float)(q[32 * g + l] & 0xF) - m1;
        for (int l = 0; l < 32; l++) y[64 * g + 32 + l] = d2 * (float)(q[32 * g + l] >> 4) - m2;
    }
}

/* src/quantize.c:214-240: Q4_K plus a fifth bit from qh (bits 2g, 2g + 1). */
static void deq_q5k(const uint8_t *b, float *y) {
    const float d = vxo_fp16_to_fp32(rd16(b)), mn = vxo_fp16_to_fp32(rd16(b + 2));
    const uint8_t *s = b + 4, *qh = b + 16, *ql = b + 48;
    for (int g = 0; g < 4; g++) {
        int sc, m;
        scale_min_k4(2 * g, s, &sc, &m);
        const float d1 = d * (float)sc, m1 = mn * (float)m;
        scale_min_k4(2 * g + 1, s, &sc, &m);
        const float d2 = d * (float)sc, m2 = mn * (float)m;
        for (int l = 0; l < 32; l++)
            y[64 * g + l] = d1 * (float)((ql[32 * g + l] & 0xF) + (((qh[l] >> (2 * g)) & 1) ? 16 : 0)) - m1;
        for (int l = 0; l < 32; l++)
            y[64 * g + 32 + l] = d2 * (float)((ql[32 * g + l] >> 4) + (((qh[l] >> (2 * g + 1)) & 1) ? 16 : 0)) - m2;
    }
}

/* src/quantize.c:423-437 (the reference's own layout, not GGML's Q6_K):
 * element j = low nibble j % 2 of ql[j / 2] | 2 bits j % 4 of qh[j / 4],
 * scale scales[j / 16], value - 32. */
static void deq_q6k(const uint8_t *b, float *y) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    const float d = vxo_fp16_to_fp32(rd16(b + 208));
    for (int j = 0; j < QK; j++) {
        const int lo = (ql[j / 2] >> ((j % 2) * 4)) & 0xF, hi = (qh[j / 4] >> ((j % 4) * 2)) & 3;
        y[j] = d * (float)sc[j / 16] * (float)(((hi << 4) | lo) - 32);
    }
}

/* src/quantize.c:242-250 */
static void deq_q8k(const uint8_t *b, float *y) {
    float d;
    memcpy(&d, b, 4);
    const int8_t *qs = (const int8_t *)(b + 4);
    for (int j = 0; j < QK; j++) y[j] = d * (float)qs[j];
}

typedef void (*deq_fn)(const uint8_t *, float *);

static deq_fn deq_of(int type) {
    switch (type) {
    case 10: return deq_q2k;
    case 11: return deq_q3k;
    case 12: return deq_q4k;
    case 13: return deq_q5k;
    case 14: return deq_q6k;
    case 15: return deq_q8k;
    default: return NULL;
    }
}

int vxo_dequant_kquant(int type, const void *blocks, float *y, int n) {
    deq_fn f = deq_of(type);
    if (!f || n % QK) return -1;
    const size_t bb = vxo_kquant_block_bytes(type);
    for (int i = 0; i < n / QK; i++) f((const uint8_t *)blocks + (size_t)i * bb, y + (size_t)i * QK);
    return 0;
}

/* y[r] = sum over super-blocks and their elements, in order, of
 * dequant(W)[r][k] * x[k] (src/quantize.c:486-505; cols % 256 == 0). */
int vxo_gemv_kquant(int type, const void *w, const float *x, float *y, int rows, int cols) {
    deq_fn f = deq_of(type);
    if (!f || cols % QK) return -1;
    const size_t bb = vxo_kquant_block_bytes(type);
    const int nb = cols / QK;
    for (int r = 0; r < rows; r++) {
        float sum = 0.0f, tmp[QK];
        const uint8_t *row = (const uint8_t *)w + (size_t)r * nb * bb;
        for (int b = 0; b < nb; b++) {
            f(row + (size_t)b * bb, tmp);
            for (int j = 0; j < QK; j++) sum += tmp[j] * x[b * QK + j];
        }
        y[r] = sum;
    }
    return 0;
}

/* ---- the reference's Q8_K path for Q2_K / Q3_K / Q4_K ---- */

typedef struct {
    float d;
    int8_t qs[QK];
    int16_t bsums[QK / 16];
} q8k;

/* src/quantize.c:252-287: per 256 activations, iscale = -127 / (the value of
 * largest magnitude), q = lrintf(iscale * x) clamped to [-128, 127], sums of
 * 16, d = 1 / iscale; an all-zero block gets d = 0. */
static void quantize_q8k(const float *x, q8k *y, int n) {
    for (int i = 0; i < n / QK; i++, x += QK) {
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; j++) {
            const float ax = fabsf(x[j]);
            if (ax > amax) { amax = ax; max = x[j]; }
        }
        if (amax == 0.0f) {
            memset(&y[i], 0, sizeof y[i]);
            continue;
        }
        const float iscale = -127.f / max;
        for (int j = 0; j < QK; j++) {
            int v = (int)lrintf(iscale * x[j]);
            y[i].qs[j] = (int8_t)(v > 127 ? 127 : v < -128 ? -128 : v);
        }
        for (int j = 0; j < QK / 16; j++) {
            int s = 0;
            for (int k = 0; k < 16; k++) s += y[i].qs[16 * j + k];
            y[i].bsums[j] = (int16_t)s;
        }
        y[i].d = 1.0f / iscale;
    }
}

/* src/quantize.c:339-371: GGML Q2_K decoding (scale = low nibble, min =
 * high nibble of scales[16]; four 2-bit planes of qs per 128-half). */
static float dot_q2k(const uint8_t *b, const q8k *y) {
    const uint8_t *sc = b, *q2 = b + 16;
    int summs = 0;
    for (int j = 0; j < 16; j++) summs += y->bsums[j] * (sc[j] >> 4);
    const float dall = y->d * vxo_fp16_to_fp32(rd16(b + 80));
    const float dmin = y->d * vxo_fp16_to_fp32(rd16(b + 82));
    int isum = 0, is = 0;
    const int8_t *q8 = y->qs;
    for (int half = 0; half < 2; half++, q2 += 32)
        for (int shift = 0; shift < 8; shift += 2, q8 += 32)
            for (int part = 0; part < 2; part++) {
                const int dsc = sc[is++] & 0xF;
                int s = 0;
                for (int l = 16 * part; l < 16 * part + 16; l++) s += q8[l] * ((q2[l] >> shift) & 3);
                isum += dsc * s;
            }
    return dall * (float)isum - dmin * (float)summs;
}

/* src/quantize.c:289-337: Q3_K values against int8 activations; eight int32
 * lanes (element % 8) accumulate scale * product, then d * lane summed in
 * lane order. */
static float dot_q3k(const uint8_t *b, const q8k *y) {
    int8_t a[QK];
    /* the signed 3-bit values of deq_q3k without the scale */
    const uint8_t *hm = b, *qs = b + 32, *sc = b + 96;
    for (int half = 0; half < 2; half++)
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 32; l++) {
                const int q = (qs[half * 32 + l] >> (2 * j)) & 3;
                const int hbit = (hm[l] >> (4 * half + j)) & 1;
                a[half * 128 + j * 32 + l] = (int8_t)(q - (hbit ? 0 : 4));
            }
    int32_t lane[8] = {0};
    for (int j = 0; j < QK / 16; j++)
        for (int l = 0; l < 16; l++) lane[l % 8] += scale_q3k(j, sc) * (int)(int16_t)(y->qs[16 * j + l] * a[16 * j + l]);
    const float d = vxo_fp16_to_fp32(rd16(b + 108)) * y->d;
    float sumf = 0.0f;
    for (int l = 0; l < 8; l++) sumf += d * (float)lane[l];
    return sumf;
}

/* src/quantize.c:373-421 as shipped: nibbles in element order, but each of
 * the 8 scale steps takes only 16 elements (elements 16s..16s+15 with scale
 * s), so elements 128..255 do not contribute; mins use all 16 bsums. */
static float dot_q4k_shipped(const uint8_t *b, const q8k *y) {
    int8_t a[QK];
    const uint8_t *q4 = b + 16, *s = b + 4;
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) {
            a[64 * g + l] = (int8_t)(q4[32 * g + l] & 0xF);
            a[64 * g + 32 + l] = (int8_t)(q4[32 * g + l] >> 4);
        }
    int scales[8], mins[8];
    for (int j = 0; j < 8; j++) scale_min_k4(j, s, &scales[j], &mins[j]);
    int sumi = 0;
    for (int j = 0; j < QK / 16; j++) sumi += y->bsums[j] * mins[j / 2];
    int32_t lane[8] = {0};
    for (int st = 0; st < 8; st++)
        for (int l = 0; l < 16; l++)
            lane[l % 8] += scales[st] * (int)(int16_t)(y->qs[16 * st + l] * a[16 * st + l]);
    const float d = vxo_fp16_to_fp32(rd16(b)) * y->d, dmin = vxo_fp16_to_fp32(rd16(b + 2)) * y->d;
    float sumf = 0.0f;
    for (int l = 0; l < 8; l++) sumf += d * (float)lane[l];
    sumf -= dmin * (float)sumi;
    return sumf;
}

int vxo_gemv_kquant_shipped(int type, const void *w, const float *x, float *y, int rows, int cols) {
    if (type != 10 && type != 11 && type != 12) return vxo_gemv_kquant(type, w, x, y, rows, cols);
    if (cols % QK) return -1;
    const int nb = cols / QK;
    q8k *qx = (q8k *)malloc((size_t)nb * sizeof(q8k));
    if (!qx) return -1;
    quantize_q8k(x, qx, cols);
    const size_t bb = vxo_kquant_block_bytes(type);
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = (const uint8_t *)w + (size_t)r * nb * bb;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * bb;
            sum += type == 10 ? dot_q2k(blk, &qx[b]) : type == 11 ? dot_q3k(blk, &qx[b]) : dot_q4k_shipped(blk, &qx[b]);
        }
        y[r] = sum;
    }
    free(qx);
    return 0;
}
