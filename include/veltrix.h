/*
 * veltrix.h — public types of the Veltrix C API, as seen by callers of the
 * B200 back end.
 *
 * Drop-in contract: a program compiled against the reference header
 * (include/veltrix.h of spear34000/veltrix-engine) must be able to link
 * against this library unchanged.  Callers read and write fields of
 * `struct vx_model` directly (the reference speculative loop sets
 * `model->cache_len`, src/speculative.c:101 and :153, and reads
 * `model->config.n_vocab`, :120-122), so the struct layouts below keep the
 * field order and types of the reference's include/veltrix.h:15-173.
 * Only pointers to the meta-predictor and tokenizer types appear in
 * `vx_model`; they stay opaque here because the B200 back end does not use
 * them.
 */
#ifndef VELTRIX_H
#define VELTRIX_H

#include <stdint.h>
#include <stddef.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VX_MAX_NAME 64
#define VX_MAX_LAYERS 256
#define VX_MAX_DIM 8192
#define VX_HEAD_DIM 128

/* Error codes: reference include/veltrix.h:15-24. */
typedef enum {
    VX_OK = 0,
    VX_ERR_FILE = -1,
    VX_ERR_FORMAT = -2,
    VX_ERR_MEMORY = -3,
    VX_ERR_PARAM = -4,
    VX_ERR_GGUF = -5,
    VX_ERR_NOMODEL = -6,
    VX_ERR_UNSUPPORTED = -7,
} vx_error;

/* Tensor element types (GGML numbering): reference include/veltrix.h:26-47. */
typedef enum {
    VX_TYPE_F32 = 0,
    VX_TYPE_F16 = 1,
    VX_TYPE_Q4_0 = 2,
    VX_TYPE_Q4_1 = 3,
    VX_TYPE_Q5_0 = 6,
    VX_TYPE_Q5_1 = 7,
    VX_TYPE_Q8_0 = 8,
    VX_TYPE_Q8_1 = 9,
    VX_TYPE_Q2_K = 10,
    VX_TYPE_Q3_K = 11,
    VX_TYPE_Q4_K = 12,
    VX_TYPE_Q5_K = 13,
    VX_TYPE_Q6_K = 14,
    VX_TYPE_Q8_K = 15,
    VX_TYPE_IQ1_S = 20,
    VX_TYPE_IQ2_XXS = 21,
    VX_TYPE_IQ2_XS = 22,
    VX_TYPE_IQ3_XXS = 26,
    VX_TYPE_IQ1_M = 31,
    VX_TYPE_BF16 = 32,
} vx_type;

/* Host tensor record: reference include/veltrix.h:49-56. */
typedef struct {
    int32_t ne[4];
    size_t nbytes;
    vx_type type;
    uint8_t *data;
    bool owned;
    char name[VX_MAX_NAME];
} vx_tensor;

typedef enum {
    VX_ARCH_QWEN2 = 0,
    VX_ARCH_LLAMA,
    VX_ARCH_MISTRAL,
    VX_ARCH_GEMMA,
    VX_ARCH_PHI,
    VX_ARCH_PHI3,
    VX_ARCH_STARCODER,
    VX_ARCH_COUNT,
} vx_arch;

typedef enum {
    VX_MLP_SWIGLU = 0,
    VX_MLP_GEGLU,
    VX_MLP_CLASSIC,
} vx_mlp_type;

typedef enum {
    VX_NORM_RMS = 0,
    VX_NORM_LAYER,
} vx_norm_type;

/* Model hyper-parameters: reference include/veltrix.h:80-102. */
typedef struct {
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int n_embd;
    int n_head_dim;
    int n_ff;
    int n_vocab;
    int n_ctx;
    float rope_theta;
    float rope_freq_base;
    int n_threads;
    vx_arch arch;
    vx_mlp_type mlp_type;
    vx_norm_type norm_type;
    int rope_partial_dims;
    bool has_q_bias;
    bool has_k_bias;
    bool has_v_bias;
    bool has_post_attn_norm;
    bool has_post_ffn_norm;
    bool has_ffn_bias;
} vx_model_config;

typedef enum {
    VX_COMPUTE_EXACT = 0,
    VX_COMPUTE_ATTN_ONLY,
    VX_COMPUTE_SKIP,
} vx_compute_level;

/* Opaque in this back end (pointers only inside vx_model). */
typedef struct vx_meta_predictor vx_meta_predictor;
struct vx_tokenizer;

/*
 * Model handle: reference include/veltrix.h:136-173, same field order.
 * In the B200 back end the weights live in device memory; the host tensor
 * arrays below stay NULL.  `config` and `cache_len` are authoritative and
 * are re-read at every API entry, so callers may keep setting them.
 */
typedef struct vx_model {
    vx_model_config config;
    vx_tensor **tensors;
    int n_tensors;
    void *tensor_data;
    vx_tensor *tok_embd;
    vx_tensor **attn_q;
    vx_tensor **attn_k;
    vx_tensor **attn_v;
    vx_tensor **attn_o;
    vx_tensor **attn_q_bias;
    vx_tensor **attn_k_bias;
    vx_tensor **attn_v_bias;
    vx_tensor **ffn_gate;
    vx_tensor **ffn_up;
    vx_tensor **ffn_down;
    vx_tensor **ffn_gate_bias;
    vx_tensor **ffn_up_bias;
    vx_tensor **ffn_down_bias;
    vx_tensor **attn_norm;
    vx_tensor **ffn_norm;
    vx_tensor **attn_norm_bias;
    vx_tensor **ffn_norm_bias;
    vx_tensor *norm_w;
    vx_tensor *norm_bias_w;
    vx_tensor *output_w;
    vx_meta_predictor **layer_predictors;
    vx_meta_predictor *attn_pattern_predictor;
    vx_meta_predictor *token_exit_predictor;
    float *k_cache;
    float *v_cache;
    int cache_len;
    float *scratch;
    size_t scratch_size;
    float *dequant_tmp;
    size_t dequant_tmp_size;
    struct vx_tokenizer *tokenizer;
} vx_model;

/* Core API: reference include/veltrix.h:175-183. */
vx_error vx_model_create(const char *path, vx_model **model);
void vx_model_destroy(vx_model *model);
vx_error vx_model_forward(vx_model *model, const int *tokens, int n_tokens, float *logits);
void vx_model_kv_truncate(vx_model *model, int length);
void vx_set_compute_level(vx_compute_level level);
void vx_enable_metalearn(bool enable);
void vx_set_n_threads(int n);
void vx_set_forward_timing_enabled(int enabled);
void vx_print_forward_timing(void);

#ifdef __cplusplus
}
#endif

#endif /* VELTRIX_H */
