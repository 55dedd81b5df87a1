/*
 * ref_access.c — test-only accessors for struct vx_model fields
 * (reference include/veltrix.h:80-102, :165-167), linked into both reference
 * builds under oracle/_ref/, so the Python tests and the CPU baseline need no
 * struct layout of their own.  Callers of the reference set cache_len
 * directly (src/speculative.c:101,153); vxref_set_cache_len does the same.
 */
#include "veltrix.h"

int vxref_cache_len(const vx_model *m) { return m->cache_len; }
void vxref_set_cache_len(vx_model *m, int len) { m->cache_len = len; }
void vxref_config(const vx_model *m, int *out) {
    out[0] = m->config.n_layers; out[1] = m->config.n_heads; out[2] = m->config.n_kv_heads;
    out[3] = m->config.n_embd; out[4] = m->config.n_head_dim; out[5] = m->config.n_ff;
    out[6] = m->config.n_vocab; out[7] = m->config.n_ctx;
}
