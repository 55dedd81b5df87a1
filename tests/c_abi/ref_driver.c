/*
 * A caller of the reference's public C API, compiled against the REFERENCE's
 * own headers (include/model.h, include/speculative.h, include/veltrix.h of
 * spear34000/veltrix-engine) and linked against libveltrix_b200.so, to show
 * that the library is a drop-in for that API: the same prototypes, and the
 * same layout of the struct vx_model fields a caller reads or pokes
 * (config.n_vocab, cache_len; src/speculative.c:101, :153 set cache_len).
 *
 *   ref_driver TARGET.gguf DRAFT.gguf N_NEW < prompt ids (whitespace separated)
 *
 * Prints three lines: the target-only greedy continuation (first-max argmax
 * over vx_model_forward logits, src/speculative.c:93-98), the greedy
 * speculative continuation (vx_speculative_generate at temperature 0, k = 4),
 * and "cache_len N" after rewinding cache_len by hand and re-running the last
 * prompt token.  Test infrastructure (tests/test_c_abi_gpu.py).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "model.h"
#include "speculative.h"

static int argmax_first(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

int main(int argc, char **argv) {
    if (argc != 4) {
        fprintf(stderr, "usage: %s TARGET.gguf DRAFT.gguf N_NEW < prompt\n", argv[0]);
        return 2;
    }
    const int n_new = atoi(argv[3]);
    int cap = 4096, n = 0;
    int *prompt = malloc(sizeof(int) * cap);
    while (n < cap && scanf("%d", &prompt[n]) == 1) n++;
    if (n < 1 || n_new < 1) return 2;

    vx_model *t = NULL, *d = NULL;
    if (vx_model_create(argv[1], &t) != VX_OK || vx_model_create(argv[2], &d) != VX_OK) {
        fprintf(stderr, "vx_model_create failed\n");
        return 1;
    }
    const int V = t->config.n_vocab;
    float *logits = malloc(sizeof(float) * V);
    if (vx_model_forward(t, prompt, n, logits) != VX_OK) return 1;
    printf("greedy");
    for (int i = 0; i < n_new; i++) {
        const int tok = argmax_first(logits, V);
        printf(" %d", tok);
        if (vx_model_forward(t, &tok, 1, logits) != VX_OK) return 1;
    }
    printf("\n");

    vx_speculative_state *s = vx_speculative_create(d, t, 4);
    if (!s) return 1;
    vx_speculative_set_temp(s, 0.0f, 1.0f);
    int *out = malloc(sizeof(int) * n_new);
    const int got = vx_speculative_generate(s, prompt, n, out, n_new);
    printf("spec");
    for (int i = 0; i < got; i++) printf(" %d", out[i]);
    printf("\n");
    vx_speculative_destroy(s);

    /* rewind by writing the field, as the reference's own loop does */
    t->cache_len = n - 1;
    if (vx_model_forward(t, &prompt[n - 1], 1, logits) != VX_OK) return 1;
    printf("cache_len %d\n", t->cache_len);

    vx_model_destroy(d);
    vx_model_destroy(t);
    free(out);
    free(logits);
    free(prompt);
    return 0;
}
