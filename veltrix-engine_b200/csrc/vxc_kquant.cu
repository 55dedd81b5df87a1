// vxc_kquant.cu — K-quant weight matrices (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K,
// Q8_K: the types the reference's GEMV dispatches, src/model.c:222-233).
//
// The matrix keeps the GGUF super-blocks of 256 weights as they are, and
// every weight is decoded bit for bit as the reference does (vxc_kquant.cuh).
// The GEMV is y = decoded(W) . x with fp32
// accumulation, the reference's blockwise GEMV (src/quantize.c:486-505) up
// to the order of the sum.  The reference's Q8_K-activation path for
// Q2_K/Q3_K/Q4_K is not reproduced: it rounds the activations to int8 and its
// Q4_K dot leaves out half of every super-block.
//
// One warp per output row, each lane decoding every 32nd weight of a
// super-block; up to 8 activation rows share each decoded weight.
#include "vxc_common.cuh"
#include "vxc_internal.h"
#include "vxc_kquant.cuh"
#include "vxc_ptx.cuh"
#include "vxc_qmat.cuh"

#include <cuda_fp16.h>
#include <stdlib.h>

namespace {

constexpr int QK = VXC_QK_K;

template <int T>
__global__ void __launch_bounds__(256) k_dequant_kq(const uint8_t *__restrict__ w, long long n, float *__restrict__ y) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = vxc_kq_decode<T>(w + (size_t)(i / QK) * vxc_kq_block_bytes(T), (int)(i % QK));
}

// y[m][r] = sum_k decoded(W)[r][k] x[m][k] for m < M; one warp per row r.
template <int T>
__global__ void __launch_bounds__(256) k_gemv_kq(const uint8_t *__restrict__ w, int R, int nb,
                                                 const float *__restrict__ x, int M, float *__restrict__ y) {
    constexpr int BB = vxc_kq_block_bytes(T);
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
                const float wv = vxc_kq_decode<T>(blk, e);
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

// Forward-pass variant: the activations are the GEMV image of one chunk of
// up to 64 rows (layout in vxc_qmat.cuh): element k of row m is
// (hi + lo) / xs[m], where hi + lo is exact in fp32 and xs[m] a power of two.
// out[m * ldo + r] for m < M, one slice (no split-K).
template <int T>
__global__ void __launch_bounds__(256) k_gemv_kq_img(const uint8_t *__restrict__ w, int R, int nb,
                                                     const uint8_t *__restrict__ img, int N,
                                                     const float *__restrict__ xs, int M, float *__restrict__ out,
                                                     int ldo) {
    pdl_trigger();
    pdl_wait();
    constexpr int BB = vxc_kq_block_bytes(T);
    const int r = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (r >= R) return;
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
                const int e = lane + 32 * i, k = b * QK + e;
                const float wv = vxc_kq_decode<T>(blk, e);
                // 16-byte row of chunk (k / 8) of the image, element k % 8
                const uint8_t *ph = img + (size_t)(((k >> 5) * 4 + ((k >> 3) & 3)) * 2 * N + m0) * 16 + (k & 7) * 2;
#pragma unroll
                for (int mm = 0; mm < 8; mm++)
                    if (mm < mc) {
                        const float hi = __half2float(*reinterpret_cast<const __half *>(ph + (size_t)mm * 16));
                        const float lo = __half2float(*reinterpret_cast<const __half *>(ph + (size_t)(N + mm) * 16));
                        acc[mm] = fmaf(wv, hi + lo, acc[mm]);
                    }
            }
        }
#pragma unroll
        for (int mm = 0; mm < 8; mm++) {
            float v = acc[mm];
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && mm < mc) out[(size_t)(m0 + mm) * ldo + r] = v / xs[m0 + mm];
        }
    }
}

template <int T>
cudaError_t launch_img(const vxc_qmat *w, const uint8_t *img, int N, const float *xs, int M, float *out, int ldo,
                       cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((size_t)w->rows * 32 + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const uint8_t *q = w->qs;
    return cudaLaunchKernelEx(&cfg, k_gemv_kq_img<T>, q, w->rows, w->nblk, img, N, xs, M, out, ldo);
}

}  // namespace

static int gemv_image_one(const vxc_qmat *w, const uint8_t *img, int N, const float *xs, int M, float *out, int ldo,
                          cudaStream_t st) {
    cudaError_t e;
    switch (w->type) {
    case 10: e = launch_img<10>(w, img, N, xs, M, out, ldo, st); break;
    case 11: e = launch_img<11>(w, img, N, xs, M, out, ldo, st); break;
    case 12: e = launch_img<12>(w, img, N, xs, M, out, ldo, st); break;
    case 13: e = launch_img<13>(w, img, N, xs, M, out, ldo, st); break;
    case 14: e = launch_img<14>(w, img, N, xs, M, out, ldo, st); break;
    default: e = launch_img<15>(w, img, N, xs, M, out, ldo, st); break;
    }
    vxc_count_launches(1);
    if (e != cudaSuccess) {
        vxc_set_error("vxc_forward: K-quant GEMV: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}

int vxc_kquant_gemv_image(const vxc_qmat *w, const uint8_t *img, int N, const float *xs, int M, float *out,
                          cudaStream_t st) {
    if (w->type != VXC_QMAT_STACK) return gemv_image_one(w, img, N, xs, M, out, w->rows, st);
    for (int i = 0; i < w->nparts; i++) {
        int rc = gemv_image_one(w->parts[i], img, N, xs, M, out + w->part_row0[i], w->rows, st);
        if (rc) return rc;
    }
    return 0;
}

int vxc_kquant_stack(vxc_qmat **parts, int n, vxc_qmat **out) {
    if (n < 1 || n > 3) { vxc_set_error("vxc_net_create: 1 to 3 stacked parts"); return -4; }
    vxc_qmat *w = (vxc_qmat *)calloc(1, sizeof(vxc_qmat));
    if (!w) { vxc_set_error("vxc_net_create: out of host memory"); return -3; }
    w->type = VXC_QMAT_STACK;
    w->cols = parts[0]->cols;
    w->nparts = n;
    for (int i = 0; i < n; i++) {
        w->parts[i] = parts[i];
        w->part_row0[i] = w->rows;
        w->rows += parts[i]->rows;
        w->qs_bytes += parts[i]->qs_bytes;
    }
    *out = w;
    return 0;
}

int vxc_kquant_from_device(int type, const uint8_t *dev_blocks, int rows, int cols, vxc_qmat **out) {
    if (!out || !dev_blocks || !vxc_is_kquant(type) || rows <= 0 || cols <= 0 || cols % QK) {
        vxc_set_error("vxc_net_create: K-quant matrices need a multiple of 256 columns (type %d, %d x %d)", type,
                      rows, cols);
        return -7;
    }
    vxc_qmat *w = (vxc_qmat *)calloc(1, sizeof(vxc_qmat));
    if (!w) { vxc_set_error("vxc_net_create: out of host memory"); return -3; }
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->nblk = cols / QK;
    w->rec = vxc_kq_block_bytes(type);
    w->wscale = 1.0f;
    w->qs_bytes = (size_t)rows * w->nblk * w->rec;
    cudaError_t e = cudaMalloc((void **)&w->qs, w->qs_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(w->qs, dev_blocks, w->qs_bytes, cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) {
        vxc_set_error("vxc_net_create: %s", cudaGetErrorString(e));
        vxc_qmat_destroy(w);
        return -3;
    }
    *out = w;
    return 0;
}

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
    w->rec = vxc_kq_block_bytes(type);
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
