/*
 * vxo.h — CPU oracle for the Veltrix speculative-decoding hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (veltrix-engine_b200/)
 * includes, links or executes this code; only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference legs of bench.py use it,
 * and only as the checker or as the timed CPU baseline.
 *
 * It restates, in plain C, the reference's scalar (non-AVX2) arithmetic for
 * the path, with the one fix the reference needs to be deterministic
 * (out-of-place attn_o GEMV, reference src/model.c:543-544), plus the
 * corrected speculative-sampling procedure ("O-spec") whose uniforms come
 * from Philox4x32-10.  Each function cites the reference lines it follows.
 * Parity pin: tests/test_oracle_pin.py checks the forward restatement
 * bit-for-bit against the reference sources compiled by oracle/Makefile.
 */
#ifndef VXO_H
#define VXO_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 codec, quantised blocks (reference src/quantize.c) ---- */
float    vxo_fp16_to_fp32(uint16_t h);
uint16_t vxo_fp32_to_fp16_trunc(float f);
void     vxo_quantize_row_q4_0(const float *x, void *out, int n);
void     vxo_quantize_row_q8_0(const float *x, void *out, int n);
void     vxo_dequant_q4_0(const void *blocks, float *y, int n);
void     vxo_dequant_q8_0(const void *blocks, float *y, int n);
/* y[m][r] = sum_k W[r][k] x[m][k] with the reference's scalar order. */
void     vxo_qgemv(int type, const void *w, const float *x, float *y,
                   int M, int rows, int cols);

/* ---- K-quant weights (vxo_kquant.c; type ids 10..15 = Q2_K..Q8_K) ---- */
size_t vxo_kquant_block_bytes(int type);
/* The reference's vx_dequantize_row_* for the type; n % 256 == 0. */
int vxo_dequant_kquant(int type, const void *blocks, float *y, int n);
/* y[r] = dequant(W)[r] . x, one sequential fp32 sum per row (the
 * reference's blockwise GEMV); cols % 256 == 0. */
int vxo_gemv_kquant(int type, const void *w, const float *x, float *y, int rows, int cols);
/* The reference's GEMV as shipped: Q2_K/Q3_K/Q4_K through Q8_K-quantised
 * activations and integer dots, other types as vxo_gemv_kquant. */
int vxo_gemv_kquant_shipped(int type, const void *w, const float *x, float *y, int rows, int cols);

/* ---- elementwise ops (reference src/tensor.c scalar branches) ---- */
void vxo_rms_norm(float *o, const float *x, const float *w, int n);
void vxo_softmax(float *x, int n);
void vxo_rope(float *q, float *k, int pos, int n_heads, int n_kv_heads,
              int head_dim, float theta);
void vxo_silu(float *x, int n);

/* ---- model (reference src/model.c, src/gguf.c, src/format.c) ---- */
typedef struct vxo_model vxo_model;
vxo_model *vxo_model_load(const char *path, int n_ctx);
void vxo_model_free(vxo_model *m);
/* out[0..8) = layers, heads, kv_heads, embd, head_dim, ff, vocab, ctx */
void vxo_model_config(const vxo_model *m, int *out);
float vxo_model_rope_theta(const vxo_model *m);
int  vxo_model_cache_len(const vxo_model *m);
void vxo_model_set_cache_len(vxo_model *m, int len);
/* vx_model_forward semantics: logits of the last token. */
int  vxo_forward(vxo_model *m, const int *tokens, int n, float *logits);
/* Same, but logits of every token: logits[n][vocab]. */
int  vxo_forward_all(vxo_model *m, const int *tokens, int n, float *logits);

/* ---- sampling (O-spec; see vxo_spec.c) ---- */
uint32_t vxo_philox_u32(uint64_t seed, uint32_t pos, uint32_t seq,
                        uint32_t purpose);
float    vxo_expf(float x);
int      vxo_argmax(const float *l, int n);
int      vxo_sample(const float *l, int n, float temp, uint32_t word);
/* Fused acceptance for one sequence (config 3).  P: [k+1][V] target logits,
 * Q: [k][V] draft logits, d: k draft tokens at absolute positions
 * pos0..pos0+k-1.  Returns accepted count; *next = correction/bonus token. */
int      vxo_accept(const float *P, const float *Q, const int *d, int k, int V,
                    float temp, uint64_t seed, uint32_t seq, uint32_t pos0,
                    int *next);
int      vxo_greedy_generate(vxo_model *t, const int *prompt, int plen,
                             int *out, int n_new);
int      vxo_spec_generate(vxo_model *t, vxo_model *d, const int *prompt,
                           int plen, int k, float temp, uint64_t seed,
                           uint32_t seq, int *out, int n_new, int *n_rounds);

#define VXO_PURPOSE_DRAFT    1u
#define VXO_PURPOSE_ACCEPT   2u
#define VXO_PURPOSE_RESAMPLE 3u

#ifdef __cplusplus
}
#endif
#endif
