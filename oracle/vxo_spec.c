/*
 * vxo_spec.c — CPU oracle ("O-spec"): speculative decoding with standard
 * rejection sampling.  TEST INFRASTRUCTURE ONLY (see vxo.h).
 *
 * The reference loop (src/speculative.c:148-294) cannot be the oracle: it
 * stores raw logits as q (:167, :197), tests acceptance with rand() even at
 * temperature 0 (:200), emits no bonus token and re-prefills the draft every
 * round (:153-158).  This file keeps its structure (draft k tokens, verify,
 * accept/reject, residual resample from max(0, p - q), :199-231) with the
 * textbook procedure (Leviathan et al. 2023; Chen et al. 2023):
 *   - p = softmax(target/T), q = softmax(draft/T); T <= 0 means greedy with
 *     first-max argmax (src/speculative.c:93-98).
 *   - accept d_i iff u < p(d_i)/q(d_i) (the min(1, p/q) test of :199-202);
 *     on the first rejection sample from max(0, p - q) (:209-225), falling
 *     back to argmax(p) when that residual is empty; if all k are accepted,
 *     sample a bonus token from the last target row.
 *   - uniforms come from Philox4x32-10 keyed by (seed, absolute token
 *     position, sequence id, purpose), so the stream does not depend on the
 *     number of GPUs or on batch composition.
 *
 * Canonical sampling arithmetic (mirrored bit-for-bit by the CUDA kernels):
 *   e_v = vxo_expf((l_v - max_l) * (1/T))        fp32, no FMA contraction
 *   W_v = trunc(e_v * 2^32)                      integer weight, W_v <= 2^32
 *   draw: thr = floor(S * u24 / 2^24), S = sum W_v, u24 = philox >> 8;
 *         token = first v whose inclusive prefix sum of W exceeds thr.
 * Every decision is made in exact integer arithmetic, so any summation order
 * gives the same answer.
 */
#include "vxo.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), counter
 * (pos, seq, purpose, 0), key (seed lo, seed hi); returns output word 0. */
uint32_t vxo_philox_u32(uint64_t seed, uint32_t pos, uint32_t seq, uint32_t purpose) {
    uint32_t c0 = pos, c1 = seq, c2 = purpose, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

/* Full 4-word block, for known-answer tests of the generator itself. */
void vxo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* exp(x) for the sampler: Cody-Waite reduction x = k*ln2 + r with ln2 split
 * in two parts (W. J. Cody, W. Waite, "Software Manual for the Elementary
 * Functions", 1980), then the degree-7 Taylor polynomial of e^r evaluated by
 * Horner with fused multiply-adds, scaled by 2^k through the exponent bits.
 * Only IEEE-exact primitives (fmaf, *, rintf) are used so the CUDA kernels
 * reproduce it bit-for-bit.  Accurate to a few ulp on [-80, 0]; returns 0
 * below -80 (weights below 2^-32 truncate to zero anyway). */
float vxo_expf(float x) {
    if (!(x > -80.0f)) return 0.0f;
    if (x > 0.0f) x = 0.0f;
    float kf = rintf(x * 1.44269504088896341f);
    float r = fmaf(kf, -0.693145751953125f, x);
    r = fmaf(kf, -1.42860682030941723212e-6f, r);
    float p = 1.98412698412698413e-4f;      /* 1/7! */
    p = fmaf(p, r, 1.38888888888888889e-3f); /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333e-3f); /* 1/5! */
    p = fmaf(p, r, 4.16666666666666667e-2f); /* 1/4! */
    p = fmaf(p, r, 1.66666666666666667e-1f); /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int k = (int)kf;
    union { uint32_t u; float f; } s;
    s.u = (uint32_t)(k + 127) << 23;
    return p * s.f;
}

int vxo_argmax(const float *l, int n) {
    int b = 0;
    for (int i = 1; i < n; i++)
        if (l[i] > l[b]) b = i;
    return b;
}

static float vmax(const float *l, int n) {
    float m = l[0];
    for (int i = 1; i < n; i++) if (l[i] > m) m = l[i];
    return m;
}

/* W_v = trunc(exp((l_v - max) / T) * 2^32); returns S = sum W. */
static uint64_t weights(const float *l, int n, float temp, uint64_t *W) {
    float m = vmax(l, n);
    float invT = 1.0f / temp;
    uint64_t S = 0;
    for (int v = 0; v < n; v++) {
        float z = (l[v] - m) * invT;
        float e = vxo_expf(z);
        W[v] = (uint64_t)(e * 4294967296.0f);
        S += W[v];
    }
    return S;
}

static int draw(const uint64_t *W, int n, uint64_t S, uint32_t word) {
    uint64_t thr = (uint64_t)(((u128)S * (word >> 8)) >> 24);
    uint64_t acc = 0;
    for (int v = 0; v < n; v++) {
        acc += W[v];
        if (acc > thr) return v;
    }
    return n - 1;
}

int vxo_sample(const float *l, int n, float temp, uint32_t word) {
    if (!(temp > 0.0f)) return vxo_argmax(l, n);
    uint64_t *W = (uint64_t *)malloc((size_t)n * sizeof(uint64_t));
    uint64_t S = weights(l, n, temp, W);
    int t = draw(W, n, S, word);
    free(W);
    return t;
}

int vxo_accept(const float *P, const float *Q, const int *d, int k, int V, float temp, uint64_t seed,
               uint32_t seq, uint32_t pos0, int *next) {
    if (!(temp > 0.0f)) {
        for (int i = 0; i < k; i++) {
            int best = vxo_argmax(P + (size_t)i * V, V);
            if (d[i] != best) { *next = best; return i; }
        }
        *next = vxo_argmax(P + (size_t)k * V, V);
        return k;
    }
    uint64_t *Wp = (uint64_t *)malloc((size_t)V * sizeof(uint64_t));
    uint64_t *Wq = (uint64_t *)malloc((size_t)V * sizeof(uint64_t));
    int acc = k;
    for (int i = 0; i < k; i++) {
        const float *pl = P + (size_t)i * V, *ql = Q + (size_t)i * V;
        uint64_t Sp = weights(pl, V, temp, Wp);
        uint64_t Sq = weights(ql, V, temp, Wq);
        int t = d[i];
        uint32_t u = vxo_philox_u32(seed, pos0 + (uint32_t)i, seq, VXO_PURPOSE_ACCEPT) >> 8;
        /* u/2^24 < (Wp/Sp)/(Wq/Sq)  <=>  u*Wq*Sp < 2^24*Wp*Sq */
        int ok = (t >= 0 && t < V) && ((u128)u * Wq[t] * Sp < ((u128)Wp[t] * Sq << 24));
        if (ok) continue;
        /* residual max(0, p - q) scaled by Sp*Sq, shifted into 64 bits */
        uint64_t SR = 0;
        for (int v = 0; v < V; v++) {
            u128 a = (u128)Wp[v] * Sq, b = (u128)Wq[v] * Sp;
            Wq[v] = a > b ? (uint64_t)((a - b) >> 36) : 0;
            SR += Wq[v];
        }
        if (SR == 0) *next = vxo_argmax(pl, V);
        else *next = draw(Wq, V, SR, vxo_philox_u32(seed, pos0 + (uint32_t)i, seq, VXO_PURPOSE_RESAMPLE));
        acc = i;
        break;
    }
    if (acc == k) {
        const float *pl = P + (size_t)k * V;
        uint64_t Sp = weights(pl, V, temp, Wp);
        *next = draw(Wp, V, Sp, vxo_philox_u32(seed, pos0 + (uint32_t)k, seq, VXO_PURPOSE_RESAMPLE));
    }
    free(Wp);
    free(Wq);
    return acc;
}

/* Target-only greedy decoding: the semantics of the CLI loop
 * (src/main.c:299-324) without its duplicated last-prompt-token forward. */
int vxo_greedy_generate(vxo_model *t, const int *prompt, int plen, int *out, int n_new) {
    int cfg[8];
    vxo_model_config(t, cfg);
    int V = cfg[6];
    float *lg = (float *)malloc((size_t)V * sizeof(float));
    vxo_model_set_cache_len(t, 0);
    if (vxo_forward(t, prompt, plen, lg) != 0) { free(lg); return 0; }
    for (int i = 0; i < n_new; i++) {
        out[i] = vxo_argmax(lg, V);
        if (i + 1 < n_new && vxo_forward(t, &out[i], 1, lg) != 0) { free(lg); return i + 1; }
    }
    free(lg);
    return n_new;
}

int vxo_spec_generate(vxo_model *t, vxo_model *d, const int *prompt, int plen, int k, float temp,
                      uint64_t seed, uint32_t seq, int *out, int n_new, int *n_rounds) {
    int cfg[8];
    vxo_model_config(t, cfg);
    int V = cfg[6];
    int cap = plen + n_new + k + 2;
    int *c = (int *)malloc((size_t)cap * sizeof(int));
    memcpy(c, prompt, (size_t)plen * sizeof(int));
    int L = plen;
    float *P = (float *)malloc((size_t)(k + 1) * V * sizeof(float));
    float *Q = (float *)malloc((size_t)k * V * sizeof(float));
    int *vt = (int *)malloc((size_t)(k + 1) * sizeof(int));
    int *dt = (int *)malloc((size_t)k * sizeof(int));
    /* KV invariant: target holds positions 0..L-2; draft holds 0..dvalid-1 */
    vxo_model_set_cache_len(t, 0);
    vxo_model_set_cache_len(d, 0);
    if (L > 1) {
        vxo_forward(t, c, L - 1, P);
        vxo_forward(d, c, L - 1, Q);
    }
    int dvalid = L - 1;
    int gen = 0, rounds = 0;
    while (gen < n_new) {
        /* draft: bring draft KV to L-1 entries, then sample k tokens */
        vxo_model_set_cache_len(d, dvalid);
        vxo_forward(d, c + dvalid, L - dvalid, Q);
        for (int i = 0; i < k; i++) {
            dt[i] = vxo_sample(Q + (size_t)i * V, V, temp,
                               vxo_philox_u32(seed, (uint32_t)(L + i), seq, VXO_PURPOSE_DRAFT));
            if (i + 1 < k) vxo_forward(d, &dt[i], 1, Q + (size_t)(i + 1) * V);
        }
        /* verify k+1 rows at positions L-1 .. L+k-1 */
        vt[0] = c[L - 1];
        memcpy(vt + 1, dt, (size_t)k * sizeof(int));
        vxo_model_set_cache_len(t, L - 1);
        vxo_forward_all(t, vt, k + 1, P);
        int nxt;
        int a = vxo_accept(P, Q, dt, k, V, temp, seed, seq, (uint32_t)L, &nxt);
        for (int i = 0; i < a && gen < n_new; i++) { out[gen++] = dt[i]; c[L + i] = dt[i]; }
        if (gen < n_new) out[gen++] = nxt;
        c[L + a] = nxt;
        int dend = L + k - 1;       /* draft KV entries written this round */
        L += a + 1;
        dvalid = dend < L - 1 ? dend : L - 1;
        rounds++;
    }
    if (n_rounds) *n_rounds = rounds;
    free(c); free(P); free(Q); free(vt); free(dt);
    return gen;
}
