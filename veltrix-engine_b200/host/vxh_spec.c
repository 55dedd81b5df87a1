/*
 * vxh_spec.c — the reference's speculative API (include/speculative.h) on
 * the device engine (vxc_spec_*).  The state borrows the two models
 * (src/speculative.c:109-139: destroy never frees them) and owns an engine
 * sized for the largest request seen so far.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "speculative.h"
#include "veltrix_cuda.h"
#include "vxh_model.h"

struct vx_speculative_state {
    vx_model *draft, *target;
    int k;
    float temperature, top_p;
    uint64_t seed;
    int seq_base;
    vxc_spec *eng;
    int eng_seqs, eng_ctx;
    vx_speculative_stats last;
};

vx_speculative_state *vx_speculative_create(vx_model *draft, vx_model *target, int max_draft_tokens) {
    if (!draft || !target || max_draft_tokens < 1) return NULL;
    if (draft->config.n_vocab != target->config.n_vocab) return NULL;
    vx_speculative_state *s = (vx_speculative_state *)calloc(1, sizeof *s);
    if (!s) return NULL;
    s->draft = draft;
    s->target = target;
    s->k = max_draft_tokens;
    s->temperature = 0.8f;   /* reference defaults, src/speculative.c:116-117 */
    s->top_p = 0.95f;
    s->seed = 1;
    return s;
}

void vx_speculative_destroy(vx_speculative_state *s) {
    if (!s) return;
    vxc_spec_destroy(s->eng);
    free(s);
}

void vx_speculative_set_temp(vx_speculative_state *s, float temp, float top_p) {
    if (s) {
        s->temperature = temp;
        s->top_p = top_p;
    }
}

void vx_speculative_set_seed(vx_speculative_state *s, uint64_t seed) {
    if (s) s->seed = seed;
}

void vx_speculative_set_seq_id_base(vx_speculative_state *s, int base) {
    if (s) s->seq_base = base;
}

int vx_speculative_get_stats(const vx_speculative_state *s, vx_speculative_stats *out) {
    if (!s || !out) return VX_ERR_PARAM;
    *out = s->last;
    return VX_OK;
}

int vx_speculative_probe(vx_speculative_state *s, int which, int reps, double *ms, double *kv_bytes) {
    if (!s || !s->eng || !ms) return VX_ERR_PARAM;
    int rc = vxc_spec_probe(s->eng, which, reps, ms, kv_bytes);
    if (rc) fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
    return rc ? VX_ERR_PARAM : VX_OK;
}

static int ensure_engine(vx_speculative_state *s, int n_seq, int ctx) {
    ctx = (ctx + 255) & ~255;
    if (s->eng && s->eng_seqs == n_seq && s->eng_ctx >= ctx) return 0;
    vxc_spec_destroy(s->eng);
    s->eng = NULL;
    int rc = vxc_spec_create(vxb_of(s->target)->net, vxb_of(s->draft)->net, n_seq, s->k, ctx, &s->eng);
    if (rc) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return rc;
    }
    s->eng_seqs = n_seq;
    s->eng_ctx = ctx;
    return 0;
}

int vx_speculative_generate_batch(vx_speculative_state *s, const int *const *prompts, const int *prompt_lens,
                                  int n_seq, int **outputs, int max_tokens, int *counts) {
    if (!s || !prompts || !prompt_lens || !outputs || n_seq < 1 || max_tokens < 1) return 0;
    for (int i = 0; i < n_seq; i++) {
        if (!prompts[i] || prompt_lens[i] < 1 || !outputs[i]) return 0;
        if (counts) counts[i] = 0;
    }
    /* The reference loop stops once prompt + generated tokens reach the
     * target's n_ctx (src/speculative.c:254, :258-262, :293), so a sequence
     * emits at most n_ctx - prompt_len tokens, and none when its prompt already
     * fills the context.  Sequences with room run together; each keeps its own
     * Philox sequence id (seq_id_base + its index in the call). */
    const int n_ctx = s->target->config.n_ctx;
    int *sel = (int *)malloc((size_t)n_seq * sizeof(int));
    if (!sel) return 0;
    int nsel = 0, maxp = 0, eff = 0;
    size_t total = 0;
    for (int i = 0; i < n_seq; i++) {
        const int cap = n_ctx > 0 ? n_ctx - prompt_lens[i] : max_tokens;
        if (cap <= 0) continue;
        sel[nsel++] = i;
        if (prompt_lens[i] > maxp) maxp = prompt_lens[i];
        const int want = cap < max_tokens ? cap : max_tokens;
        if (want > eff) eff = want;
        total += (size_t)prompt_lens[i];
    }
    if (nsel == 0 || ensure_engine(s, nsel, maxp + eff + s->k + 2)) {
        free(sel);
        return 0;
    }
    int *cat = (int *)malloc(total * sizeof(int));
    int *lens = (int *)malloc((size_t)nsel * sizeof(int));
    int *ids = (int *)malloc((size_t)nsel * sizeof(int));
    int *out = (int *)malloc((size_t)nsel * eff * sizeof(int));
    int *cnt = (int *)calloc((size_t)nsel, sizeof(int));
    if (!cat || !lens || !ids || !out || !cnt) {
        free(sel); free(cat); free(lens); free(ids); free(out); free(cnt);
        return 0;
    }
    size_t off = 0;
    for (int j = 0; j < nsel; j++) {
        const int i = sel[j];
        memcpy(cat + off, prompts[i], (size_t)prompt_lens[i] * sizeof(int));
        off += (size_t)prompt_lens[i];
        lens[j] = prompt_lens[i];
        ids[j] = s->seq_base + i;
    }
    vxc_spec_stats st;
    memset(&st, 0, sizeof st);
    int rc = vxc_spec_generate(s->eng, cat, lens, ids, nsel, eff, s->temperature, s->seed, out, cnt, &st);
    int total_gen = 0;
    if (rc == 0) {
        for (int j = 0; j < nsel; j++) {
            const int i = sel[j];
            int c = cnt[j];
            if (n_ctx > 0 && c > n_ctx - prompt_lens[i]) c = n_ctx - prompt_lens[i];
            if (c > max_tokens) c = max_tokens;
            memcpy(outputs[i], out + (size_t)j * eff, (size_t)c * sizeof(int));
            if (counts) counts[i] = c;
            total_gen += c;
        }
        s->last.rounds = st.rounds;
        s->last.drafted = st.drafted;
        s->last.accepted = st.accepted;
        s->last.emitted = st.emitted;
        s->last.prefill_ms = st.prefill_ms;
        s->last.decode_ms = st.decode_ms;
    } else {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
    }
    free(sel); free(cat); free(lens); free(ids); free(out); free(cnt);
    return total_gen;
}

int vx_speculative_generate(vx_speculative_state *s, int *prompt, int prompt_len, int *output, int max_tokens) {
    if (!s || !prompt || !output || prompt_len < 1 || max_tokens < 1) return 0;   /* src/speculative.c:240-241 */
    const int *pp[1] = {prompt};
    int *oo[1] = {output};
    int cnt = 0;
    return vx_speculative_generate_batch(s, pp, &prompt_len, 1, oo, max_tokens, &cnt);
}

int vx_speculative_generate_stream(vx_speculative_state *s, int token, int *output, int max_tokens) {
    int prompt[1] = {token};   /* src/speculative.c:296-300 */
    return vx_speculative_generate(s, prompt, 1, output, max_tokens);
}
