/*
 * veltrix_synth.h — synthetic GGUF checkpoints for tests and benchmarks.
 *
 * No counterpart in the reference's library API; it follows the fixture
 * writer of the reference's tests/test_e2e.c:20-160 (llama architecture,
 * GGUF v3) but places tensor offsets relative to the data section, as the
 * loader expects (src/gguf.c:231-233).  Weights are N(0, 0.02) from
 * Philox4x32-10 keyed by (seed, tensor index, element index), quantised with
 * the reference's Q4_0 rule (src/quantize.c:88-114) or the GGML Q8_0 rule;
 * norm weights are 1.0.
 */
#ifndef VELTRIX_SYNTH_H
#define VELTRIX_SYNTH_H

#include <stdint.h>

#include "veltrix.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int n_embd, n_layers, n_heads, n_kv_heads, n_ff, n_vocab;
    float rope_theta;
    int wtype;   /* 2 = Q4_0, 8 = Q8_0 for every 2-D tensor; or a K-quant type
                  * 10..15 (Q2_K..Q8_K; n_embd, n_ff % 256 == 0), whose
                  * super-blocks hold Philox bytes with fixed scale fields
                  * (decoded weights of the order of 0.02), not quantised
                  * normals; or VX_SYNTH_KQ_MIX: Q4_K, with Q6_K for
                  * attn_v, ffn_down and the LM head */
} vx_synth_config;

#define VX_SYNTH_KQ_MIX 100

/* Writes `path`; returns 0 or a vx_error code. */
int vx_synth_write_gguf(const char *path, const vx_synth_config *cfg, uint64_t seed);

/* The same model created on the current device without a file: the weights
 * are generated in device memory (up to the device's rounding of
 * double-precision log/sqrt/cos/sin, the numbers the writer puts in the
 * file).  world == 1 and nccl_id == NULL load the whole model; otherwise
 * this rank's tensor-parallel shard, as vx_model_create_tp (model.h). */
vx_error vx_model_create_synth(const vx_synth_config *cfg, uint64_t seed, int rank, int world,
                               const void *nccl_id, vx_model **model);

#ifdef __cplusplus
}
#endif
#endif
