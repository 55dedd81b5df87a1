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
#include "vxc_image.cuh"
#include "vxc_ptx.cuh"
#include "vxc_qmat.cuh"
#include "vxc_internal.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>

// ---------------------------------------------------------------------------
// Repack: GGUF blocks (row-major, one row = nblk blocks) -> tile records
// (layout in vxc_qmat.cuh), scales multiplied by 2^wshift.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint16_t scaled_scale(const uint8_t *blk, float mul) {
    const float d = vxc_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    return __half_as_ushort(__float2half_rn(d * mul));   // exact: mul is a power of two
}

__global__ void k_repack_q4_0(const uint8_t *__restrict__ src, uint8_t *__restrict__ qs, int R, int nblk,
                              float mul) {
    long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)R * nblk;
    if (id >= total) return;
    int r = (int)(id / nblk), b = (int)(id % nblk);
    const uint8_t *blk = src + (size_t)id * 18;
    int tile = r / VXC_TILE_ROWS, tr = r % VXC_TILE_ROWS;
    uint8_t *rec = qs + ((size_t)tile * nblk + b) * (VXC_TILE_ROWS * 16 + 256);
    reinterpret_cast<uint16_t *>(rec + VXC_TILE_ROWS * 16)[tr] = scaled_scale(blk, mul);
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
    *reinterpret_cast<uint4 *>(rec + tr * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void k_repack_q8_0(const uint8_t *__restrict__ src, uint8_t *__restrict__ qs, int R, int nblk,
                              float mul) {
    long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)R * nblk;
    if (id >= total) return;
    int r = (int)(id / nblk), b = (int)(id % nblk);
    const uint8_t *blk = src + (size_t)id * 34;
    int tile = r / VXC_TILE_ROWS, tr = r % VXC_TILE_ROWS;
    uint8_t *rec = qs + ((size_t)tile * nblk + b) * (VXC_TILE_ROWS * 32 + 256);
    reinterpret_cast<uint16_t *>(rec + VXC_TILE_ROWS * 32)[tr] = scaled_scale(blk, mul);
    uint8_t *dst = rec + tr * 32;
#pragma unroll
    for (int j = 0; j < 32; j++) dst[j] = blk[2 + j];
}

// Largest finite |d| of a matrix's blocks, as fp16 bits (finite magnitudes
// order like their bits).
__global__ void k_max_scale_bits(const uint8_t *__restrict__ blocks, long long nblocks, int bs,
                                 unsigned int *__restrict__ out) {
    unsigned int mx = 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nblocks;
         i += (long long)gridDim.x * blockDim.x) {
        const uint8_t *b = blocks + (size_t)i * bs;
        const unsigned int h = (unsigned int)(b[0] | (b[1] << 8)) & 0x7FFFu;
        if (h < 0x7C00u && h > mx) mx = h;
    }
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    if ((threadIdx.x & 31) == 0 && mx) atomicMax(out, mx);
}

// wshift such that max|d| * qmax * 2^wshift <= 2^14 over the whole matrix.
static int wshift_of(int type, unsigned int mx) {
    if (mx == 0) return 0;
    const float maxd = __half2float(__ushort_as_half((unsigned short)mx));
    int e;
    frexpf(maxd * (type == 2 ? 8.0f : 128.0f), &e);
    int S = 14 - e;
    return S < -60 ? -60 : S > 60 ? 60 : S;
}

int vxc_qmat_from_device(int type, const uint8_t *dev_blocks, int rows, int cols, vxc_qmat **out) {
    if (!out || !dev_blocks || rows <= 0 || cols <= 0 || (cols % 32) != 0 || (type != 2 && type != 8)) {
        vxc_set_error("vxc_qmat_create: bad arguments (type %d, %d x %d)", type, rows, cols);
        return -4;
    }
    vxc_qmat *w = (vxc_qmat *)calloc(1, sizeof(vxc_qmat));
    if (!w) { vxc_set_error("vxc_qmat_create: out of host memory"); return -3; }
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->nblk = cols / 32;
    w->ntile = (rows + VXC_TILE_ROWS - 1) / VXC_TILE_ROWS;
    w->qb = type == 2 ? 16 : 32;
    w->rec = VXC_TILE_ROWS * w->qb + 256;
    w->qs_bytes = (size_t)w->ntile * w->nblk * w->rec;
    const long long total = (long long)rows * w->nblk;
    unsigned int *d_mx = NULL, mx = 0;
    cudaError_t e = cudaMalloc((void **)&d_mx, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemset(d_mx, 0, sizeof(unsigned int));
    if (e == cudaSuccess) {
        const long long want = (total + 255) / 256;
        k_max_scale_bits<<<(unsigned)(want < 4 * 148 ? want : 4 * 148), 256>>>(dev_blocks, total,
                                                                                type == 2 ? 18 : 34, d_mx);
        vxc_count_launches(1);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(&mx, d_mx, sizeof mx, cudaMemcpyDeviceToHost);
    if (d_mx) cudaFree(d_mx);
    w->wshift = wshift_of(type, mx);
    w->wscale = ldexpf(1.0f, -w->wshift);
    if (e == cudaSuccess) e = cudaMalloc((void **)&w->qs, w->qs_bytes);
    if (e == cudaSuccess) e = cudaMemset(w->qs, 0, w->qs_bytes);
    if (e == cudaSuccess) {
        int th = 256;
        unsigned gb = (unsigned)((total + th - 1) / th);
        const float mul = ldexpf(1.0f, w->wshift);
        if (type == 2) (k_repack_q4_0<<<gb, th>>>(dev_blocks, w->qs, rows, w->nblk, mul), vxc_count_launches(1));
        else (k_repack_q8_0<<<gb, th>>>(dev_blocks, w->qs, rows, w->nblk, mul), vxc_count_launches(1));
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        vxc_set_error("vxc_qmat_create: %s", cudaGetErrorString(e));
        vxc_qmat_destroy(w);
        return -3;
    }
    *out = w;
    return 0;
}

extern "C" int vxc_qmat_create(int type, const void *host_blocks, int rows, int cols, vxc_qmat **out) {
    if (vxc_is_kquant(type)) {
        int rc = vxc_require_device();
        return rc ? rc : vxc_kquant_create(type, host_blocks, rows, cols, out);
    }
    if (!out || !host_blocks || rows <= 0 || cols <= 0 || (cols % 32) != 0 || (type != 2 && type != 8)) {
        vxc_set_error("vxc_qmat_create: bad arguments (type %d, %d x %d)", type, rows, cols);
        return -4;
    }
    int rc = vxc_require_device();
    if (rc) return rc;
    const size_t src_bytes = (size_t)rows * (cols / 32) * (type == 2 ? 18 : 34);
    uint8_t *staging = NULL;
    cudaError_t e = cudaMalloc((void **)&staging, src_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(staging, host_blocks, src_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (staging) cudaFree(staging);
        vxc_set_error("vxc_qmat_create: %s", cudaGetErrorString(e));
        return -3;
    }
    rc = vxc_qmat_from_device(type, staging, rows, cols, out);
    cudaFree(staging);
    return rc;
}

extern "C" void vxc_qmat_destroy(vxc_qmat *w) {
    if (!w) return;
    if (w->type == VXC_QMAT_STACK)
        for (int i = 0; i < w->nparts; i++) vxc_qmat_destroy(w->parts[i]);
    if (w->qs) cudaFree(w->qs);
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
// A second implementation of the same product, kept as a cross-check of the
// tensor-core path.
// ---------------------------------------------------------------------------
#define SIMT_MC 8

template <int QT>
__global__ void __launch_bounds__(128) k_qgemv_simt(const uint8_t *__restrict__ qs, int R, int nblk, float wscale,
                                                    const float *__restrict__ x, int M, float *__restrict__ out,
                                                    int bps) {
    constexpr int QB = QT == 2 ? 16 : 32;
    constexpr int REC = VXC_TILE_ROWS * QB + 256;
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
            const uint8_t *rec = qs + ((size_t)tile * nblk + b) * REC;
            float d = vxc_h2f(reinterpret_cast<const uint16_t *>(rec + VXC_TILE_ROWS * QB)[t]);
            float wv[32];
            if (QT == 2) {
                uint4 q = *reinterpret_cast<const uint4 *>(rec + t * 16);
                uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        wv[8 * j + 2 * i] = (float)((int)((wd[j] >> (4 * i)) & 0xF) - 8);
                        wv[8 * j + 2 * i + 1] = (float)((int)((wd[j] >> (16 + 4 * i)) & 0xF) - 8);
                    }
            } else {
                const int4 *p = reinterpret_cast<const int4 *>(rec + t * 32);
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
                if (m < mc) dst[(size_t)(m0 + m) * R + row] = acc[m] * wscale;
        }
    }
}

// Activation image of x[M][K] (one CTA per row): xs[m] and the hi/lo chunks.
__global__ void k_act_image(const float *__restrict__ x, int K, int N, uint8_t *__restrict__ img,
                            float *__restrict__ xs) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    const float *xr = x + (size_t)m * K;
    float mx = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(xr[k]));
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) mx = fmaxf(mx, red[i]);
    const float s = vxc_prescale(mx);
    if (threadIdx.x == 0) xs[m] = s;
    vxc_image_row(img, N, m, K, s, [&](int k) { return xr[k]; });
}

// Launch with programmatic dependent launch: the kernel may start while its
// predecessor drains; both kernels here call griddepcontrol.wait before
// touching memory.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*k)(KArgs...), unsigned grid, unsigned block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, ((KArgs)args)...);
    vxc_count_launches(1);
    return e;
}

int vxc_launch_act_image(const float *x, int M, int K, uint8_t *img, float *xs, cudaStream_t st) {
    return launch_pdl(k_act_image, (unsigned)M, 256, st, x, K, vxc_img_rows(M), img, xs) == cudaSuccess ? 0 : -3;
}

// Deterministic split-K reduction: y[m][r] = sum_{s<ks} ws[s][m][r] in order.
__global__ void k_splitk_reduce(const float *__restrict__ ws, int ks, int MR, float *__restrict__ y) {
    pdl_trigger();
    pdl_wait();
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= MR) return;
    float acc = ws[i];
    for (int s = 1; s < ks; s++) acc += ws[(size_t)s * MR + i];
    y[i] = acc;
}

int vxc_launch_splitk_reduce(const float *ws, int ks, int M, int R, float *y, cudaStream_t st) {
    int MR = M * R;
    return launch_pdl(k_splitk_reduce, (unsigned)((MR + 255) / 256), 256, st, ws, ks, MR, y) == cudaSuccess ? 0 : -3;
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
    if (vxc_is_kquant(w->type)) return 0;
    int ks, bps;
    simt_split(w, &ks, &bps);
    return ks > 1 ? (size_t)ks * M * w->rows * sizeof(float) : 0;
}

extern "C" int vxc_qgemv_simt(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
                              size_t workspace_bytes, void *stream) {
    if (!w || !x || !y || M <= 0) { vxc_set_error("vxc_qgemv_simt: bad arguments"); return -4; }
    if (vxc_is_kquant(w->type)) { vxc_set_error("vxc_qgemv_simt: Q4_0 / Q8_0 only"); return -7; }
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
        (k_qgemv_simt<2><<<grid, 128, smem, st>>>(w->qs, w->rows, w->nblk, w->wscale, x, M, dst, bps),
         vxc_count_launches(1));
    else
        (k_qgemv_simt<8><<<grid, 128, smem, st>>>(w->qs, w->rows, w->nblk, w->wscale, x, M, dst, bps),
         vxc_count_launches(1));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { vxc_set_error("vxc_qgemv_simt: %s", cudaGetErrorString(e)); return -3; }
    if (ks > 1) return vxc_launch_splitk_reduce(dst, ks, M, w->rows, y, st);
    return 0;
}
