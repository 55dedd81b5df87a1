/*
 * speculative.h — speculative decoding (reference include/speculative.h:8-15,
 * same functions and argument meanings), plus a batched entry point, seed
 * control and statistics.
 *
 * Semantics of the B200 back end (the reference loop, src/speculative.c:148-294,
 * is not correct speculative sampling; this is the standard procedure):
 *   - temperature <= 0: greedy.  The output equals target-only greedy decoding.
 *   - temperature > 0: draft tokens ~ softmax(draft/T); accept with
 *     probability min(1, p/q); on rejection resample from max(0, p - q);
 *     a bonus token from the target when all drafts are accepted.  Uniforms
 *     come from Philox4x32-10 keyed by (seed, token position, sequence id).
 *     top_p is recorded but sampling always uses the full distribution
 *     (top_p = 1).  The reference applies top_p to the draft side only
 *     (src/speculative.c:164); with the standard procedure the output
 *     follows the target's tempered distribution for any draft
 *     distribution, so the cut would change acceptance rates, not the
 *     distribution of the output.
 *   - The state keeps its own device KV caches for both models; the models'
 *     own cache_len fields are not modified.
 * Functions return the number of generated tokens (0 on failure) like the
 * reference; create returns NULL on failure.
 */
#ifndef VX_SPECULATIVE_H
#define VX_SPECULATIVE_H

#include <stdint.h>

#include "veltrix.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct vx_speculative_state vx_speculative_state;

vx_speculative_state *vx_speculative_create(vx_model *draft, vx_model *target, int max_draft_tokens);
void vx_speculative_destroy(vx_speculative_state *state);
void vx_speculative_set_temp(vx_speculative_state *state, float temp, float top_p);

int vx_speculative_generate(vx_speculative_state *state, int *prompt, int prompt_len, int *output,
                            int max_tokens);
int vx_speculative_generate_stream(vx_speculative_state *state, int token, int *output, int max_tokens);

/* ---- additions (no reference counterpart: the reference drives one
 * sequence per model, include/speculative.h:12-15) ---- */

/* Philox seed of the sampler (default 1). */
void vx_speculative_set_seed(vx_speculative_state *state, uint64_t seed);
/* Sequence ids used as Philox counters start at `base` (default 0); a shard
 * of a larger batch passes its first global index so the uniforms, and thus
 * the tokens, do not depend on how the batch is split across GPUs. */
void vx_speculative_set_seq_id_base(vx_speculative_state *state, int base);

/* n_seq independent sequences decoded together on the device.  outputs[s]
 * receives up to max_tokens tokens and counts[s] their number.  Returns the
 * total number of generated tokens. */
int vx_speculative_generate_batch(vx_speculative_state *state, const int *const *prompts, const int *prompt_lens,
                                  int n_seq, int **outputs, int max_tokens, int *counts);

typedef struct {
    long long rounds, drafted, accepted, emitted;
    double prefill_ms, decode_ms;   /* device time of the last generate call */
} vx_speculative_stats;

int vx_speculative_get_stats(const vx_speculative_state *state, vx_speculative_stats *out);

/* Device time of one piece of the last generate call's final round, averaged
 * over `reps` re-runs: which = 0 target verify forward, 1 draft step, 2 fused
 * acceptance (vxc_spec_probe).  Returns VX_OK or a vx_error code. */
int vx_speculative_probe(vx_speculative_state *state, int which, int reps, double *ms, double *kv_bytes);

#ifdef __cplusplus
}
#endif

#endif
