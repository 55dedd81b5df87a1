/*
 * veltrix_cuda.h — the C-ABI between Veltrix's C host code and the B200
 * kernels (library libveltrix_b200.so).
 *
 * Plain C types only: device pointers are `void *` / `float *` obtained from
 * cudaMalloc (or any allocator of device memory), streams are cudaStream_t
 * passed as `void *` (NULL = the legacy default stream).  Every function
 * returns a vx_error code (0 = VX_OK); vxc_error_string() gives the text of
 * the last failure on the calling thread.  There is no CPU fallback: with no
 * usable CUDA device every call fails with VX_ERR_UNSUPPORTED.
 *
 * Each entry point names the reference interface it replaces
 * (spear34000/veltrix-engine, file:line).
 */
#ifndef VELTRIX_CUDA_H
#define VELTRIX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device & errors --------------------------------------------------- */

/* Select / initialise a CUDA device for the calling thread.  Fails with
 * VX_ERR_UNSUPPORTED when no CUDA device is present.  (No reference
 * counterpart: the reference is CPU-only, src/model.c:377-382 sets threads.) */
int vxc_device_init(int device);
int vxc_device_count(void);
const char *vxc_error_string(void);
/* Read and clear the device-side error word that kernels set instead of
 * trapping (timeouts, out-of-range token ids).  Synchronises the device. */
int vxc_check_device_error(unsigned int *code_out);

/* ---- quantised weight matrices ------------------------------------------ */

typedef struct vxc_qmat vxc_qmat;

/* Upload a GGUF-layout matrix of `rows` x `cols` (cols % 32 == 0) held in
 * host memory and repack it for the device (quant plane + scale plane, 128-row
 * tiles).  type: 2 = Q4_0 (18-byte blocks), 8 = Q8_0 (34-byte blocks).
 * Replaces the reference's tensor load + whole-matrix dequant buffer
 * (src/gguf.c:236-287, src/model.c:74-87). */
int vxc_qmat_create(int type, const void *host_blocks, int rows, int cols, vxc_qmat **out);
void vxc_qmat_destroy(vxc_qmat *w);
int vxc_qmat_shape(const vxc_qmat *w, int *type, int *rows, int *cols);

/* Bytes of scratch vxc_qgemv needs for M activation rows (0 when the chosen
 * split needs none). */
size_t vxc_qgemv_workspace_bytes(const vxc_qmat *w, int M);

/* y[m][r] = sum_k W[r][k] * x[m][k] for m < M (fp32 in, fp32 out, device
 * pointers, row-major with leading dimensions cols and rows).  Q4_0 follows
 * the reference's interleaved nibble order.  Replaces vx_gemv_q4_0
 * (src/quantize.c:728-750), vx_gemv_q4_0_avx2 (src/simd/avx2.c:311-370) and
 * apply_gemv's Q8_0 path (src/model.c:234-244), batched over M rows.
 * `workspace` must hold vxc_qgemv_workspace_bytes(w, M) bytes (may be NULL
 * when that is 0). */
int vxc_qgemv(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
              size_t workspace_bytes, void *stream);

/* Same product through the exact CUDA-core kernel (fp32 FMA, no tensor
 * cores); kept as an independent second implementation for tests. */
int vxc_qgemv_simt(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
                   size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif
