// vxc_internal.h — host-side declarations shared by the library's .cu files.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include "../../include/veltrix_cuda.h"

void vxc_set_error(const char *fmt, ...);
// 0 when a CUDA device is current; VX_ERR_UNSUPPORTED otherwise.
int vxc_require_device(void);
// Per-device error word (device memory), valid after vxc_require_device().
unsigned int *vxc_device_error_ptr(void);
int vxc_launch_splitk_reduce(const float *ws, int ks, int M, int R, float *y, cudaStream_t st);
// Activation image of x[M][K] (layout in vxc_qmat.cuh) and its prescales xs[M].
int vxc_launch_act_image(const float *x, int M, int K, uint8_t *img, float *xs, cudaStream_t st);

// A quantised matrix from GGUF blocks already in device memory (row-major,
// rows x cols/32 blocks); the blocks are only read.
int vxc_qmat_from_device(int type, const uint8_t *dev_blocks, int rows, int cols, vxc_qmat **out);

// Synthetic GGUF blocks of tensor ti (vxc_synth.cu): rows row0.. and column
// blocks blk0.. of a tensor whose rows hold nblk_full blocks, row-major into
// dev_out.  Enqueued on the legacy default stream.
int vxc_synth_blocks(int type, uint64_t seed, uint32_t ti, long long row0, int nrows, int nblk_full, int blk0,
                     int nblk, uint8_t *dev_out);

// K-quant matrices (vxc_kquant.cu): GGUF super-blocks kept as they are;
// nblk = super-blocks per row, rec = bytes per super-block.
bool vxc_is_kquant(int type);
int vxc_kquant_create(int type, const void *host_blocks, int rows, int cols, vxc_qmat **out);
int vxc_kquant_gemv(const vxc_qmat *w, const float *x, int M, float *y, cudaStream_t st);
// The forward's K-quant GEMV: activations from one chunk's GEMV image (N
// image rows, prescales xs), out[M][R]; programmatic dependent launch.
int vxc_kquant_gemv_image(const vxc_qmat *w, const uint8_t *img, int N, const float *xs, int M, float *out,
                          cudaStream_t st);
// A K-quant matrix from super-blocks already in device memory (copied).
int vxc_kquant_from_device(int type, const uint8_t *dev_blocks, int rows, int cols, vxc_qmat **out);
// K-quant matrices of different types stacked by rows (type VXC_QMAT_STACK;
// takes ownership of the parts).  The forward runs it like a K-quant matrix.
int vxc_kquant_stack(vxc_qmat **parts, int n, vxc_qmat **out);

// Tensor-core GEMV plan for M <= 64 activation rows (vxc_gemv_tc.cu).
struct VxcGemvPlan {
    int nt;       // N / 16 (N = padded rows of the image)
    int ks;       // K-slices; the output is ks partial sums [ks][M][R]
    int nbs;      // 32-column blocks per slice
    int grid;     // CTAs
    size_t smem;  // dynamic shared memory per CTA
};
bool vxc_gemv_plan(const vxc_qmat *w, int M, VxcGemvPlan *p);
// Launches the GEMV (programmatic dependent launch) reading an activation
// image + prescales, writing part[ks][M][R] (ks == 1: the output itself).
// With x != NULL the GEMV reads fp32 rows x[M][K] instead and builds each
// K-slice's operand itself (img and xs unused).
int vxc_gemv_run(const vxc_qmat *w, const uint8_t *img, const float *xs, int M, float *part,
                 const VxcGemvPlan &p, cudaStream_t st, const float *x = NULL);
size_t vxc_qgemv_simt_ws(const vxc_qmat *w, int M);

// Tensor-core GEMM for many activation rows (vxc_gemm_tc.cu), Q4_0 / Q8_0.
// The activation image is cut into slabs of VXC_GEMM_SLAB rows, slab s at
// img + s * slab_bytes in the vxc_qmat.cuh layout with N = padded rows of
// that slab (slab_bytes >= K/32 * 128 * VXC_GEMM_SLAB); prescales xs[M].
// K is cut into vxc_gemm_slices(w) slices (a function of K only); slice s of
// row m goes to out[(m >> 6) * slot + s * sst + (m & 63) * R + r] with
// sst = sstride, or (rows of m's 64-row chunk) * R when sstride == 0 (the
// forward's partial-sum slots).  The consumer adds the slices in order.  A
// row's result does not depend on the other rows of the call.  Programmatic
// dependent launch.
#define VXC_GEMM_SLAB 256
// Rows from which vxc_qgemv and vxc_forward use the GEMM.
#define VXC_GEMM_MIN_ROWS 64
int vxc_gemm_ok(const vxc_qmat *w);
int vxc_gemm_slices(const vxc_qmat *w);
size_t vxc_gemm_image_bytes(int K, int M);   // image of M rows in slabs of full size
int vxc_gemm_run(const vxc_qmat *w, const uint8_t *img, size_t slab_bytes, const float *xs, int M, float *out,
                 size_t slot, size_t sstride, cudaStream_t st);
// vxc_forward without logits for the speculative engine's prompt pass: every
// Q4_0 / Q8_0 matrix runs on the GEMM whatever the row count (vxc_model.cu).
int vxc_forward_prompt(vxc_seqs *s, const int *d_tokens, const int *d_slot, const int *d_pos, int n_groups,
                       int rows_per_group, void *stream);

// CUDA-core GEMV for few activation rows (vxc_gemv_skinny.cu): Q4_0 / Q8_0,
// 1 <= M <= VXC_SKINNY_MAX_M, x rows of ldx floats (16-byte aligned).
// Writes partials [ks][M][R] (the result itself when ks == 1), ks =
// vxc_skinny_slices(w), which depends on the shape only.  Up to 2 rows it is
// faster than the tensor-core kernel on every measured shape; from 5 rows on
// the tensor cores win (measured up to 2.2x: M FMAs per weight on the CUDA
// cores).
#ifndef VXC_SKINNY_MAX_M
#define VXC_SKINNY_MAX_M 2
#endif
int vxc_skinny_ok(const vxc_qmat *w, int M);
int vxc_skinny_slices(const vxc_qmat *w);
int vxc_skinny_run(const vxc_qmat *w, const float *x, int ldx, int M, float *out, cudaStream_t st);
// The calling thread's current CUDA context (driver handle), or NULL.
void *vxc_current_context(void);
// Library-wide count of kernel launches (a CUDA-graph replay adds its kernels).
void vxc_count_launches(long long n);

// Tensor parallelism (vxc_tp.cu).  rank/world of NULL are 0/1; the exchanges
// are enqueued on st (NCCL) and return 0 or -3 with the error set.
int vxc_tp_rank(const vxc_tp *t);
// GPUs a net is split over (1 without tensor parallelism).
int vxc_net_world(const vxc_net *n);
int vxc_tp_world(const vxc_tp *t);
int vxc_tp_allreduce_sum(const vxc_tp *t, float *buf, size_t n, cudaStream_t st);
int vxc_tp_allgather(const vxc_tp *t, const float *send, float *recv, size_t n, cudaStream_t st);
