/*
 * ref_shim.c — test-only glue linked into oracle/_ref/libvxref*.so, the
 * reference's own sources compiled in place by oracle/Makefile.
 *
 * 1. Patch P1 without editing the reference: tensor.c is compiled with
 *    -Dvx_gemv_f32=vxref_gemv_f32_impl, so model.c's calls to vx_gemv_f32
 *    land here.  The reference calls it in place for attn_o
 *    (src/model.c:543-544: y == x), a data race under OpenMP; this shim
 *    hands the kernel a private copy of x, i.e. the out-of-place GEMV.
 * 2. Accessors for struct vx_model fields, so Python tests need no struct
 *    layout of their own.
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

int vxref_cache_len(const vx_model *m) { return m->cache_len; }
void vxref_set_cache_len(vx_model *m, int len) { m->cache_len = len; }
void vxref_config(const vx_model *m, int *out) {
    out[0] = m->config.n_layers; out[1] = m->config.n_heads; out[2] = m->config.n_kv_heads;
    out[3] = m->config.n_embd; out[4] = m->config.n_head_dim; out[5] = m->config.n_ff;
    out[6] = m->config.n_vocab; out[7] = m->config.n_ctx;
}
