// vxc_gemv.cu — GGUF Q4_0 / Q8_0 weight upload (repack) and the exact
// CUDA-core GEMV, plus the split-K reduction shared with the tensor-core
// kernel (vxc_gemv_tc.cu).
//
// Math (reference src/quantize.c:728-750 for Q4_0, src/model.c:234-244 for
// Q8_0):  y[m][r] = sum_b d[r][b] * sum_{j<32} (q[r][32b+j] - off) x[m][32b+j]
// with off = 8 for Q4_0 (nibbles 0..15) and 0 for Q8_0 (int8).  The inner
// 32-term sums are exact-integer weights times fp32 activations, accumulated
// in fp32; only the summation order differs from the reference.
#include "vxc_common.cuh"
#include "vxc_qmat.cuh"
#include "vxc_internal.h"

#include <stdio.h>
#include <stdlib.h>

// ---------------------------------------------------------------------------
// Repack: GGUF blocks (row-major, one row = nblk blocks) -> tiled planes.
// ---------------------------------------------------------------------------
__global__ void k_repack_q4_0(const uint8_t *__restrict__ src, uint8_t *__restrict__ qs,
                              uint16_t *__restrict__ sc, int R, int nblk) {
    long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)R * nblk;
    if (id >= total) return;
    int r = (int)(id / nblk), b = (int)(id % nblk);
    const uint8_t *blk = src + (size_t)id * 18;
    int tile = r / VXC_TILE_ROWS, tr = r % VXC_TILE_ROWS;
    size_t slot = ((size_t)tile * nblk + b) * VXC_TILE_ROWS + tr;
    sc[slot] = (uint16_t)(blk[0] | (blk[1] << 8));
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint32_t v = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int e0 = 8 * j + 2 * i, e1 = e0 + 1;           // GGUF: element e in byte e/2
            uint32_t n0 = (blk[2 + e0 / 2] >> (4 * (e0 & 1))) & 0xF;
            uint32_t n1 = (blk[2 + e1 / 2] >> (4 * (e1 & 1))) & 0xF;
            v |= n0 << (4 * i);
            v |= n1 << (16 + 4 * i);
        }
        w[j] = v;
    }
    *reinterpret_cast<uint4 *>(qs + slot * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void k_repack_q8_0(const uint8_t *__restrict__ src, uint8_t *__restrict__ qs,
                              uint16_t *__restrict__ sc, int R, int nblk) {
    long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)R * nblk;
    if (id >= total) return;
    int r = (int)(id / nblk), b = (int)(id % nblk);
    const uint8_t *blk = src + (size_t)id * 34;
    int tile = r / VXC_TILE_ROWS, tr = r % VXC_TILE_ROWS;
    size_t slot = ((size_t)tile * nblk + b) * VXC_TILE_ROWS + tr;
    sc[slot] = (uint16_t)(blk[0] | (blk[1] << 8));
    uint8_t *dst = qs + slot * 32;
#pragma unroll
    for (int j = 0; j < 32; j++) dst[j] = blk[2 + j];
}

extern "C" int vxc_qmat_create(int type, const void *host_blocks, int rows, int cols, vxc_qmat **out) {
    if (!out || !host_blocks || rows <= 0 || cols <= 0 || (cols % 32) != 0 || (type != 2 && type != 8)) {
        vxc_set_error("vxc_qmat_create: bad arguments (type %d, %d x %d)", type, rows, cols);
        return -4;
    }
    int rc = vxc_require_device();
    if (rc) return rc;
    vxc_qmat *w = (vxc_qmat *)calloc(1, sizeof(vxc_qmat));
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->nblk = cols / 32;
    w->ntile = (rows + VXC_TILE_ROWS - 1) / VXC_TILE_ROWS;
    w->qb = type == 2 ? 16 : 32;
    size_t nslot = (size_t)w->ntile * w->nblk * VXC_TILE_ROWS;
    w->qs_bytes = nslot * w->qb;
    w->sc_bytes = nslot * 2;
    size_t src_bytes = (size_t)rows * w->nblk * (type == 2 ? 18 : 34);
    uint8_t *staging = NULL;
    cudaError_t e = cudaMalloc((void **)&w->qs, w->qs_bytes);
    if (e == cudaSuccess) e = cudaMalloc((void **)&w->sc, w->sc_bytes);
    if (e == cudaSuccess) e = cudaMalloc((void **)&staging, src_bytes);
    if (e == cudaSuccess) e = cudaMemset(w->qs, 0, w->qs_bytes);
    if (e == cudaSuccess) e = cudaMemset(w->sc, 0, w->sc_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(staging, host_blocks, src_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        long long total = (long long)rows * w->nblk;
        int th = 256;
        unsigned gb = (unsigned)((total + th - 1) / th);
        if (type == 2) (k_repack_q4_0<<<gb, th>>>(staging, w->qs, w->sc, rows, w->nblk), vxc_count_launches(1));
        else (k_repack_q8_0<<<gb, th>>>(staging, w->qs, w->sc, rows, w->nblk), vxc_count_launches(1));
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        vxc_set_error("vxc_qmat_create: %s", cudaGetErrorString(e));
        vxc_qmat_destroy(w);
        return -3;
    }
    *out = w;
    return 0;
}

extern "C" void vxc_qmat_destroy(vxc_qmat *w) {
    if (!w) return;
    if (w->qs) cudaFree(w->qs);
    if (w->sc) cudaFree(w->sc);
    free(w);
}

extern "C" int vxc_qmat_shape(const vxc_qmat *w, int *type, int *rows, int *cols) {
    if (!w) return -4;
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    return 0;
}

// ---------------------------------------------------------------------------
// Exact CUDA-core kernel: one thread per weight row of a 128-row tile, one
// CTA per (tile, K-slice).  The CTA stages x[m][slice] in shared memory in
// chunks of 8 rows; each block's 32 weights are dequantised once per chunk.
// ---------------------------------------------------------------------------
#define SIMT_MC 8

template <int QT>
__global__ void __launch_bounds__(128) k_qgemv_simt(const uint8_t *__restrict__ qs, const uint16_t *__restrict__ sc,
                                                    int R, int nblk, const float *__restrict__ x, int M,
                                                    float *__restrict__ out, int bps) {
    extern __shared__ float xs[];   // [SIMT_MC][bps*32]
    const int tile = blockIdx.x, s = blockIdx.y;
    const int b0 = s * bps;
    const int b1 = min(nblk, b0 + bps);
    const int nb = b1 - b0;
    const int K = nblk * 32;
    const int t = threadIdx.x;
    const int row = tile * VXC_TILE_ROWS + t;
    const int slice_len = nb * 32;
    float *dst = gridDim.y == 1 ? out : out + (size_t)s * M * R;
    for (int m0 = 0; m0 < M; m0 += SIMT_MC) {
        const int mc = min(SIMT_MC, M - m0);
        __syncthreads();
        for (int i = t; i < mc * slice_len; i += blockDim.x) {
            int m = i / slice_len, j = i % slice_len;
            xs[m * bps * 32 + j] = x[(size_t)(m0 + m) * K + (size_t)b0 * 32 + j];
        }
        __syncthreads();
        float acc[SIMT_MC];
#pragma unroll
        for (int m = 0; m < SIMT_MC; m++) acc[m] = 0.0f;
        for (int b = b0; b < b1; b++) {
            size_t slot = ((size_t)tile * nblk + b) * VXC_TILE_ROWS + t;
            float d = vxc_h2f(sc[slot]);
            float wv[32];
            if (QT == 2) {
                uint4 q = *reinterpret_cast<const uint4 *>(qs + slot * 16);
                uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        wv[8 * j + 2 * i] = (float)((int)((wd[j] >> (4 * i)) & 0xF) - 8);
                        wv[8 * j + 2 * i + 1] = (float)((int)((wd[j] >> (16 + 4 * i)) & 0xF) - 8);
                    }
            } else {
                const int4 *p = reinterpret_cast<const int4 *>(qs + slot * 32);
                int4 q0 = p[0], q1 = p[1];
                int wd[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int j = 0; j < 8; j++)
#pragma unroll
                    for (int i = 0; i < 4; i++) wv[4 * j + i] = (float)(int8_t)((wd[j] >> (8 * i)) & 0xFF);
            }
            const float *xb = xs + (b - b0) * 32;
#pragma unroll
            for (int m = 0; m < SIMT_MC; m++) {
                if (m < mc) {
                    const float *xm = xb + m * bps * 32;
                    float sacc = 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; j++) sacc = fmaf(wv[j], xm[j], sacc);
                    acc[m] = fmaf(d, sacc, acc[m]);
                }
            }
        }
        if (row < R) {
#pragma unroll
            for (int m = 0; m < SIMT_MC; m++)
                if (m < mc) dst[(size_t)(m0 + m) * R + row] = acc[m];
        }
    }
}

// Deterministic split-K reduction: y[m][r] = sum_{s<ks} ws[s][m][r] in order.
__global__ void k_splitk_reduce(const float *__restrict__ ws, int ks, int MR, float *__restrict__ y) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= MR) return;
    float acc = ws[i];
    for (int s = 1; s < ks; s++) acc += ws[(size_t)s * MR + i];
    y[i] = acc;
}

int vxc_launch_splitk_reduce(const float *ws, int ks, int M, int R, float *y, cudaStream_t st) {
    int MR = M * R;
    (k_splitk_reduce<<<(MR + 255) / 256, 256, 0, st>>>(ws, ks, MR, y), vxc_count_launches(1));
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

static void simt_split(const vxc_qmat *w, int *ks, int *bps) {
    int want = (2 * 148 + w->ntile - 1) / w->ntile;   // about two CTAs per SM
    int b = (w->nblk + want - 1) / want;
    if (b < 4) b = 4;
    if (b > 32) b = 32;
    if (b > w->nblk) b = w->nblk;
    *bps = b;
    *ks = (w->nblk + b - 1) / b;
}

size_t vxc_qgemv_simt_ws(const vxc_qmat *w, int M) {
    int ks, bps;
    simt_split(w, &ks, &bps);
    return ks > 1 ? (size_t)ks * M * w->rows * sizeof(float) : 0;
}

extern "C" int vxc_qgemv_simt(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
                              size_t workspace_bytes, void *stream) {
    if (!w || !x || !y || M <= 0) { vxc_set_error("vxc_qgemv_simt: bad arguments"); return -4; }
    int ks, bps;
    simt_split(w, &ks, &bps);
    size_t need = ks > 1 ? (size_t)ks * M * w->rows * sizeof(float) : 0;
    if (need > workspace_bytes || (need && !workspace)) {
        vxc_set_error("vxc_qgemv_simt: workspace %zu < %zu bytes", workspace_bytes, need);
        return -4;
    }
    cudaStream_t st = (cudaStream_t)stream;
    dim3 grid(w->ntile, ks);
    size_t smem = (size_t)SIMT_MC * bps * 32 * sizeof(float);
    float *dst = ks > 1 ? (float *)workspace : y;
    if (w->type == 2)
        (k_qgemv_simt<2><<<grid, 128, smem, st>>>(w->qs, w->sc, w->rows, w->nblk, x, M, dst, bps), vxc_count_launches(1));
    else
        (k_qgemv_simt<8><<<grid, 128, smem, st>>>(w->qs, w->sc, w->rows, w->nblk, x, M, dst, bps), vxc_count_launches(1));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { vxc_set_error("vxc_qgemv_simt: %s", cudaGetErrorString(e)); return -3; }
    if (ks > 1) return vxc_launch_splitk_reduce(dst, ks, M, w->rows, y, st);
    return 0;
}
