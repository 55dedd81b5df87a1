// vxc_kquant.cuh — decoding of the reference's K-quant super-blocks (Q2_K,
// Q3_K, Q4_K, Q5_K, Q6_K, Q8_K; 256 weights each), shared by the K-quant
// GEMVs (vxc_kquant.cu) and the embedding lookup (vxc_model.cu).
//
// Every weight is decoded with the reference's fp32 steps for its type
// (src/quantize.c:116-250, :423-437), written as explicitly rounded
// multiplies and adds so that no step is contracted: the value is the
// reference's bit for bit.  Byte offsets restate the block structs of
// include/quantize.h:47-93.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#define VXC_QK_K 256

__host__ __device__ constexpr int vxc_kq_block_bytes(int t) {
    return t == 10 ? 84 : t == 11 ? 110 : t == 12 ? 144 : t == 13 ? 176 : t == 14 ? 210 : t == 15 ? 292 : 0;
}

__device__ __forceinline__ float vxc_kq_h2f(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__device__ __forceinline__ void vxc_kq_scale_min_k4(int j, const uint8_t *s, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Weight e (0..255) of super-block b, as the reference decodes it.
template <int T>
__device__ __forceinline__ float vxc_kq_decode(const uint8_t *b, int e) {
    if (T == 10) {   // src/quantize.c:116-135 (its own layout, not GGML's Q2_K)
        const int j = e >> 4, l = e & 15;
        const int sv = (j & 1) ? (b[j >> 1] >> 4) : (b[j >> 1] & 0xF);
        const float d = __fmul_rn(vxc_kq_h2f(b + 80), 1.0f), dmin = __fmul_rn(vxc_kq_h2f(b + 82), 1.0f);
        const float dl = __fmul_rn(d, (float)(sv - 8)), ml = __fmul_rn(dmin, (float)(sv - 8));
        const int v = (b[16 + (l >> 2)] >> (2 * (l & 3))) & 3;
        return __fadd_rn(__fmul_rn(dl, (float)v - 0.5f), ml);
    } else if (T == 11) {   // src/quantize.c:137-178
        const int half = e >> 7, j = (e >> 5) & 3, l = e & 31;
        const int is = half * 8 + 2 * j + (l >> 4);
        const uint8_t *sc = b + 96;
        const int lo = is < 8 ? (sc[is] & 0xF) : (sc[is - 8] >> 4);
        const int hi = (sc[8 + (is & 3)] >> (2 * (is >> 2))) & 3;
        const float dl = __fmul_rn(vxc_kq_h2f(b + 108), (float)((lo | (hi << 4)) - 32));
        const int q = (b[32 + half * 32 + l] >> (2 * j)) & 3;
        const int hbit = (b[l] >> (4 * half + j)) & 1;
        return __fmul_rn(dl, (float)(q - (hbit ? 0 : 4)));
    } else if (T == 12 || T == 13) {   // src/quantize.c:190-240
        const int g = e >> 6, hiq = (e >> 5) & 1, l = e & 31;
        int sc, m;
        vxc_kq_scale_min_k4(2 * g + hiq, b + 4, sc, m);
        const float d1 = __fmul_rn(vxc_kq_h2f(b), (float)sc), m1 = __fmul_rn(vxc_kq_h2f(b + 2), (float)m);
        const uint8_t *ql = b + (T == 12 ? 16 : 48);
        int q = hiq ? (ql[32 * g + l] >> 4) : (ql[32 * g + l] & 0xF);
        if (T == 13) q += ((b[16 + l] >> (2 * g + hiq)) & 1) ? 16 : 0;
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    } else if (T == 14) {   // src/quantize.c:423-437 (its own layout, not GGML's Q6_K)
        const int lo = (b[e >> 1] >> ((e & 1) * 4)) & 0xF, hi = (b[128 + (e >> 2)] >> ((e & 3) * 2)) & 3;
        const float ds = __fmul_rn(vxc_kq_h2f(b + 208), (float)(int8_t)b[192 + (e >> 4)]);
        return __fmul_rn(ds, (float)(((hi << 4) | lo) - 32));
    } else {   // Q8_K, src/quantize.c:242-250
        const float d = __uint_as_float((unsigned)b[0] | ((unsigned)b[1] << 8) | ((unsigned)b[2] << 16) |
                                        ((unsigned)b[3] << 24));
        return __fmul_rn(d, (float)(int8_t)b[4 + e]);
    }
}

// The same for a type known only at run time (10..15).
__device__ __forceinline__ float vxc_kq_decode_any(int type, const uint8_t *b, int e) {
    switch (type) {
    case 10: return vxc_kq_decode<10>(b, e);
    case 11: return vxc_kq_decode<11>(b, e);
    case 12: return vxc_kq_decode<12>(b, e);
    case 13: return vxc_kq_decode<13>(b, e);
    case 14: return vxc_kq_decode<14>(b, e);
    default: return vxc_kq_decode<15>(b, e);
    }
}
