/*
 * ref_shim.c — test-only glue linked into oracle/_ref/libvxref*.so, the
 * reference's own sources compiled in place by oracle/Makefile.
 *
 * 1. Patch P1 without editing the reference: tensor.c is compiled with
 *    -Dvx_gemv_f32=vxref_gemv_f32_impl, so model.c's calls to vx_gemv_f32
 *    land here.  The reference calls it in place for attn_o
 *    (src/model.c:543-544: y == x), a data race under OpenMP; this shim
 *    hands the kernel a private copy of x, i.e. the out-of-place GEMV.
 * 2. The same for the K-quant GEMVs that read x while writing y
 *    (src/quantize.c:486-505, the blockwise GEMV behind vx_gemv_q5_K,
 *    vx_gemv_q6_K and vx_gemv_q8_K): quantize.c is compiled with
 *    -Dvx_gemv_qN_K=vxref_gemv_qN_K_impl, and these wrappers copy x when the
 *    caller passes y == x.  (The Q2_K/Q3_K/Q4_K GEMVs copy x into int8
 *    blocks first and need no wrapper.)
 * The struct vx_model accessors live in ref_access.c, which both reference
 * builds link.
 */
#include <stdlib.h>
#include <string.h>
#include "veltrix.h"

void vxref_gemv_f32_impl(float *restrict y, const float *restrict A, const float *restrict x,
                         int rows, int cols);

void vx_gemv_f32(float *restrict y, const float *restrict A, const float *restrict x, int rows,
                 int cols) {
    if ((const float *)y == x) {
        float *cp = (float *)malloc((size_t)cols * sizeof(float));
        memcpy(cp, x, (size_t)cols * sizeof(float));
        vxref_gemv_f32_impl(y, A, cp, rows, cols);
        free(cp);
        return;
    }
    vxref_gemv_f32_impl(y, A, x, rows, cols);
}

#define KQ_OUT_OF_PLACE(name)                                                                       \
    void vxref_##name##_impl(const void *restrict A, const float *restrict x, float *restrict y,  \
                             int rows, int cols);                                                  \
    void vx_##name(const void *restrict A, const float *restrict x, float *restrict y, int rows,  \
                   int cols) {                                                                     \
        if ((const float *)y == x) {                                                               \
            float *cp = (float *)malloc((size_t)cols * sizeof(float));                             \
            memcpy(cp, x, (size_t)cols * sizeof(float));                                           \
            vxref_##name##_impl(A, cp, y, rows, cols);                                             \
            free(cp);                                                                              \
            return;                                                                                \
        }                                                                                          \
        vxref_##name##_impl(A, x, y, rows, cols);                                                  \
    }

KQ_OUT_OF_PLACE(gemv_q5_K)
KQ_OUT_OF_PLACE(gemv_q6_K)
KQ_OUT_OF_PLACE(gemv_q8_K)
