/*
 * model.h — model lifecycle and forward pass (reference include/model.h:6-8).
 *
 * vx_model_create   loads a GGUF file (Q4_0 / Q8_0 / F32 tensors, llama
 *                   architecture) and uploads it to the current CUDA device.
 * vx_model_forward  appends n_tokens to the model's KV cache at
 *                   model->cache_len, advances cache_len by n_tokens and writes
 *                   the logits of the LAST token into the caller's host buffer
 *                   (n_vocab floats; entries the LM head does not cover hold
 *                   -1e30, reference src/model.c:604).
 * vx_model_generate_greedy (additive) the greedy loop of the reference's CLI
 *                   (src/main.c:283-324) on the device: appends the prompt at
 *                   cache_len, then emits the argmax token and forwards it,
 *                   up to max_tokens or until the argmax is eos_id (not
 *                   emitted; -1: none).  Returns the number of tokens written
 *                   to out, or a negative vx_error.  cache_len then counts
 *                   every forwarded token (the last emitted one is not yet
 *                   forwarded).  Unlike the CLI it does not forward the last
 *                   prompt token twice (src/main.c:283,300-304).
 * vx_model_create_tp (additive) loads this rank's shard of a model split over
 *                   `world` GPUs, one process each (tensor parallelism over
 *                   NCCL; nccl_id from vxc_tp_unique_id on rank 0).  Every
 *                   rank then makes the same calls in the same order and
 *                   gets the full logits.  Destroy speculative states that
 *                   use such a model before the model: their CUDA graphs
 *                   hold the model's NCCL operations.
 */
#ifndef VX_MODEL_H
#define VX_MODEL_H

#include "veltrix.h"

#ifdef __cplusplus
extern "C" {
#endif

vx_error vx_model_create(const char *path, vx_model **model);
void vx_model_destroy(vx_model *model);
vx_error vx_model_forward(vx_model *model, const int *tokens, int n_tokens, float *logits);
int vx_model_generate_greedy(vx_model *model, const int *prompt, int n_prompt, int *out, int max_tokens,
                             int eos_id);
vx_error vx_model_create_tp(const char *path, int rank, int world, const void *nccl_id, vx_model **model);

#ifdef __cplusplus
}
#endif

#endif
