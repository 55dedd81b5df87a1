// vxc_kquant.cu — K-quant weight matrices (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K,
// Q8_K: the types the reference's GEMV dispatches, src/model.c:222-233).
//
// The matrix keeps the GGUF super-blocks of 256 weights as they are.  Every
// weight is decoded with the reference's fp32 steps for its type
// (src/quantize.c:116-250, :423-437), written as explicitly rounded
// multiplies and adds so that no step is contracted: the decoded value is
// the reference's bit for bit.  The GEMV is y = decoded(W) . x with fp32
// accumulation, the reference's blockwise GEMV (src/quantize.c:486-505) up
// to the order of the sum.  The reference's Q8_K-activation path for
// Q2_K/Q3_K/Q4_K is not reproduced: it rounds the activations to int8 and its
// Q4_K dot leaves out half of every super-block.
//
// One warp per output row, each lane decoding every 32nd weight of a
// super-block; up to 8 activation rows share each decoded weight.
#include "vxc_common.cuh"
#include "vxc_internal.h"
#include "vxc_qmat.cuh"

#include <cuda_fp16.h>
#include <stdlib.h>

namespace {

constexpr int QK = 256;

__host__ __device__ constexpr int kq_block_bytes(int t) {
    return t == 10 ? 84 : t == 11 ? 110 : t == 12 ? 144 : t == 13 ? 176 : t == 14 ? 210 : t == 15 ? 292 : 0;
}

__device__ __forceinline__ float h2f(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *s, int &sc, int &m) {
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
__device__ __forceinline__ float decode(const uint8_t *b, int e) {
    if (T == 10) {   // src/quantize.c:116-135 (its own layout, not GGML's Q2_K)
        const int j = e >> 4, l = e & 15;
        const int sv = (j & 1) ? (b[j >> 1] >> 4) : (b[j >> 1] & 0xF);
        const float d = __fmul_rn(h2f(b + 80), 1.0f), dmin = __fmul_rn(h2f(b + 82), 1.0f);
        const float dl = __fmul_rn(d, (float)(sv - 8)), ml = __fmul_rn(dmin, (float)(sv - 8));
        const int v = (b[16 + (l >> 2)] >> (2 * (l & 3))) & 3;
        return __fadd_rn(__fmul_rn(dl, (float)v - 0.5f), ml);
    } else if (T == 11) {   // src/quantize.c:137-178
        const int half = e >> 7, j = (e >> 5) & 3, l = e & 31;
        const int is = half * 8 + 2 * j + (l >> 4);
        const uint8_t *sc = b + 96;
        const int lo = is < 8 ? (sc[is] & 0xF) : (sc[is - 8] >> 4);
        const int hi = (sc[8 + (is & 3)] >> (2 * (is >> 2))) & 3;
        const float dl = __fmul_rn(h2f(b + 108), (float)((lo | (hi << 4)) - 32));
        const int q = (b[32 + half * 32 + l] >> (2 * j)) & 3;
        const int hbit = (b[l] >> (4 * half + j)) & 1;
        return __fmul_rn(dl, (float)(q - (hbit ? 0 : 4)));
    } else if (T == 12 || T == 13) {   // src/quantize.c:190-240
        const int g = e >> 6, hiq = (e >> 5) & 1, l = e & 31;
        int sc, m;
        scale_min_k4(2 * g + hiq, b + 4, sc, m);
        const float d1 = __fmul_rn(h2f(b), (float)sc), m1 = __fmul_rn(h2f(b + 2), (float)m);
        const uint8_t *ql = b + (T == 12 ? 16 : 48);
        int q = hiq ? (ql[32 * g + l] >> 4) : (ql[32 * g + l] & 0xF);
        if (T == 13) q += ((b[16 + l] >> (2 * g + hiq)) & 1) ? 16 : 0;
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    } else if (T == 14) {   // src/quantize.c:423-437 (its own layout, not GGML's Q6_K)
        const int lo = (b[e >> 1] >> ((e & 1) * 4)) & 0xF, hi = (b[128 + (e >> 2)] >> ((e & 3) * 2)) & 3;
        const float ds = __fmul_rn(h2f(b + 208), (float)(int8_t)b[192 + (e >> 4)]);
        return __fmul_rn(ds, (float)(((hi << 4) | lo) - 32));
    } else {   // Q8_K, src/quantize.c:242-250
        const float d = __uint_as_float((unsigned)b[0] | ((unsigned)b[1] << 8) | ((unsigned)b[2] << 16) |
                                        ((unsigned)b[3] << 24));
        return __fmul_rn(d, (float)(int8_t)b[4 + e]);
    }
}

template <int T>
__global__ void __launch_bounds__(256) k_dequant_kq(const uint8_t *__restrict__ w, long long n, float *__restrict__ y) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = decode<T>(w + (size_t)(i / QK) * kq_block_bytes(T), (int)(i % QK));
}

// y[m][r] = sum_k decoded(W)[r][k] x[m][k] for m < M; one warp per row r.
template <int T>
__global__ void __launch_bounds__(256) k_gemv_kq(const uint8_t *__restrict__ w, int R, int nb,
                                                 const float *__restrict__ x, int M, float *__restrict__ y) {
    constexpr int BB = kq_block_bytes(T);
    const int r = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (r >= R) return;
    const int K = nb * QK;
    const uint8_t *row = w + (size_t)r * nb * BB;
    for (int m0 = 0; m0 < M; m0 += 8) {
        const int mc = min(8, M - m0);
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = row + (size_t)b * BB;
#pragma unroll 2
            for (int i = 0; i < QK / 32; i++) {
                const int e = lane + 32 * i;
                const float wv = decode<T>(blk, e);
                const float *xc = x + (size_t)m0 * K + (size_t)b * QK + e;
#pragma unroll
                for (int mm = 0; mm < 8; mm++)
                    if (mm < mc) acc[mm] = fmaf(wv, xc[(size_t)mm * K], acc[mm]);
            }
        }
#pragma unroll
        for (int mm = 0; mm < 8; mm++) {
            float v = acc[mm];
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && mm < mc) y[(size_t)(m0 + mm) * R + r] = v;
        }
    }
}

}  // namespace

bool vxc_is_kquant(int type) { return type >= 10 && type <= 15; }

int vxc_kquant_create(int type, const void *host_blocks, int rows, int cols, vxc_qmat **out) {
    if (!out || !host_blocks || !vxc_is_kquant(type) || rows <= 0 || cols <= 0 || cols % QK) {
        vxc_set_error("vxc_qmat_create: bad K-quant arguments (type %d, %d x %d; cols %% 256 == 0)", type, rows,
                      cols);
        return -4;
    }
    vxc_qmat *w = (vxc_qmat *)calloc(1, sizeof(vxc_qmat));
    if (!w) { vxc_set_error("vxc_qmat_create: out of host memory"); return -3; }
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->nblk = cols / QK;   // super-blocks per row
    w->rec = kq_block_bytes(type);
    w->wscale = 1.0f;
    w->qs_bytes = (size_t)rows * w->nblk * w->rec;
    cudaError_t e = cudaMalloc((void **)&w->qs, w->qs_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(w->qs, host_blocks, w->qs_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        vxc_set_error("vxc_qmat_create: %s", cudaGetErrorString(e));
        vxc_qmat_destroy(w);
        return -3;
    }
    *out = w;
    return 0;
}

int vxc_kquant_gemv(const vxc_qmat *w, const float *x, int M, float *y, cudaStream_t st) {
    const unsigned grid = (unsigned)(((size_t)w->rows * 32 + 255) / 256);
    switch (w->type) {
    case 10: k_gemv_kq<10><<<grid, 256, 0, st>>>(w->qs, w->rows, w->nblk, x, M, y); break;
    case 11: k_gemv_kq<11><<<grid, 256, 0, st>>>(w->qs, w->rows, w->nblk, x, M, y); break;
    case 12: k_gemv_kq<12><<<grid, 256, 0, st>>>(w->qs, w->rows, w->nblk, x, M, y); break;
    case 13: k_gemv_kq<13><<<grid, 256, 0, st>>>(w->qs, w->rows, w->nblk, x, M, y); break;
    case 14: k_gemv_kq<14><<<grid, 256, 0, st>>>(w->qs, w->rows, w->nblk, x, M, y); break;
    default: k_gemv_kq<15><<<grid, 256, 0, st>>>(w->qs, w->rows, w->nblk, x, M, y); break;
    }
    vxc_count_launches(1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        vxc_set_error("vxc_qgemv: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}

extern "C" int vxc_kquant_dequant(const vxc_qmat *w, float *y, void *stream) {
    if (!w || !y || !vxc_is_kquant(w->type)) {
        vxc_set_error("vxc_kquant_dequant: bad arguments");
        return -4;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const long long n = (long long)w->rows * w->cols;
    const long long want = (n + 255) / 256;
    const unsigned grid = (unsigned)(want < 148 * 8 ? want : 148 * 8);
    switch (w->type) {
    case 10: k_dequant_kq<10><<<grid, 256, 0, st>>>(w->qs, n, y); break;
    case 11: k_dequant_kq<11><<<grid, 256, 0, st>>>(w->qs, n, y); break;
    case 12: k_dequant_kq<12><<<grid, 256, 0, st>>>(w->qs, n, y); break;
    case 13: k_dequant_kq<13><<<grid, 256, 0, st>>>(w->qs, n, y); break;
    case 14: k_dequant_kq<14><<<grid, 256, 0, st>>>(w->qs, n, y); break;
    default: k_dequant_kq<15><<<grid, 256, 0, st>>>(w->qs, n, y); break;
    }
    vxc_count_launches(1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        vxc_set_error("vxc_kquant_dequant: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}
