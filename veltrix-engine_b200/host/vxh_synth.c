/* vxh_synth.c — synthetic llama-architecture GGUF writer (see veltrix_synth.h). */
#define _GNU_SOURCE
#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "veltrix.h"
#include "veltrix_synth.h"

static void philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint64_t seed, uint32_t out[4]) {
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* 4 normals for elements 4q..4q+3 of tensor `ti` (Box-Muller in double). */
static void normals4(uint64_t seed, uint32_t ti, uint64_t q, float sd, float *z) {
    uint32_t w[4];
    philox((uint32_t)q, (uint32_t)(q >> 32), ti, 0x5EEDu, seed, w);
    for (int h = 0; h < 2; h++) {
        double u1 = ((double)w[2 * h] + 0.5) * (1.0 / 4294967296.0);
        double u2 = ((double)w[2 * h + 1] + 0.5) * (1.0 / 4294967296.0);
        double r = sqrt(-2.0 * log(u1));
        z[2 * h] = (float)(r * cos(6.283185307179586 * u2) * sd);
        z[2 * h + 1] = (float)(r * sin(6.283185307179586 * u2) * sd);
    }
}

/* Truncating fp32 -> fp16 encode (src/quantize.c:17-35). */
static uint16_t f2h_trunc(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t s = (x >> 31) & 1u, e = (x >> 23) & 0xFFu, m = x & 0x7FFFFFu;
    if (e == 0) return (uint16_t)(s << 15);
    if (e == 0xFF) return (uint16_t)((s << 15) | (0x1Fu << 10) | (m >> 13));
    int ne = (int)e - 127 + 15;
    if (ne <= 0) return (uint16_t)(s << 15);
    if (ne >= 31) return (uint16_t)((s << 15) | (0x1Fu << 10));
    return (uint16_t)((s << 15) | ((uint32_t)ne << 10) | (m >> 13));
}

static void quant_block(int type, const float *x, uint8_t *b) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
    if (type == 2) {   /* src/quantize.c:88-114 */
        float d = amax / 7.0f;
        if (d < 1e-10f) d = 1e-10f;
        uint16_t h = f2h_trunc(d);
        b[0] = (uint8_t)h; b[1] = (uint8_t)(h >> 8);
        float id = 1.0f / d;
        for (int j = 0; j < 32; j += 2) {
            int a = (int)(x[j] * id), c = (int)(x[j + 1] * id);
            a = a < -8 ? -8 : a > 7 ? 7 : a;
            c = c < -8 ? -8 : c > 7 ? 7 : c;
            b[2 + j / 2] = (uint8_t)((uint8_t)(a + 8) | ((uint8_t)(c + 8) << 4));
        }
    } else {           /* GGML Q8_0: d = amax/127, q = round(x/d) */
        float d = amax / 127.0f;
        uint16_t h = f2h_trunc(d);
        b[0] = (uint8_t)h; b[1] = (uint8_t)(h >> 8);
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        for (int j = 0; j < 32; j++) {
            float v = roundf(x[j] * id);
            v = v > 127.0f ? 127.0f : v < -127.0f ? -127.0f : v;
            b[2 + j] = (uint8_t)(int8_t)v;
        }
    }
}

/* K-quant super-blocks (256 weights; types 10..15 = Q2_K..Q8_K, layouts of
 * the reference's include/quantize.h:47-93).  Their quantised bytes are
 * Philox words keyed by (seed, tensor, super-block); the scale fields are
 * fixed per type so that the decoded weights are of the order of 0.02
 * (a valid block of any content decodes to finite weights). */
static int kq_bytes(int type) {
    return type == 10 ? 84 : type == 11 ? 110 : type == 12 ? 144 : type == 13 ? 176 : type == 14 ? 210
         : type == 15 ? 292 : 0;
}

static void put_h(uint8_t *b, float v) {
    uint16_t h = f2h_trunc(v);
    b[0] = (uint8_t)h;
    b[1] = (uint8_t)(h >> 8);
}

static void kq_block(int type, uint64_t seed, uint32_t ti, uint64_t blk, uint8_t *b) {
    const int n = kq_bytes(type);
    for (int w = 0; w * 16 < n; w++) {
        uint32_t r[4];
        philox((uint32_t)blk, (uint32_t)(blk >> 32), ti, 0xB10C0000u + (uint32_t)w, seed, r);
        for (int k = 0; k < 16 && w * 16 + k < n; k++) b[w * 16 + k] = (uint8_t)(r[k / 4] >> (8 * (k % 4)));
    }
    switch (type) {
    case 10: put_h(b + 80, 0.004f); put_h(b + 82, 0.004f); break;      /* d, dmin */
    case 11: put_h(b + 108, 0.0006f); break;                          /* d */
    case 12: put_h(b, 1.3e-4f); put_h(b + 2, 9.75e-4f); break;         /* d, dmin */
    case 13: put_h(b, 7e-5f); put_h(b + 2, 1.085e-3f); break;          /* d, dmin */
    case 14: put_h(b + 208, 6.2e-5f); break;                          /* d (smallest normal fp16 is 6.1e-5) */
    default: { const float d = 3e-4f; memcpy(b, &d, 4); } break;     /* Q8_K: float d */
    }
}

typedef struct { char name[64]; int nd; uint64_t ne0, ne1; int type; uint64_t off, bytes; } tinfo;

static void wr(FILE *f, const void *p, size_t n) { fwrite(p, 1, n, f); }
static void w32(FILE *f, uint32_t v) { wr(f, &v, 4); }
static void w64(FILE *f, uint64_t v) { wr(f, &v, 8); }
static void wstr(FILE *f, const char *s) { w64(f, strlen(s)); wr(f, s, strlen(s)); }
static void kv_u32(FILE *f, const char *k, uint32_t v) { wstr(f, k); w32(f, 4); w32(f, v); }
static void pad32(FILE *f) {
    long p = ftell(f);
    while (p % 32) { fputc(0, f); p++; }
}

int vx_synth_write_gguf(const char *path, const vx_synth_config *c, uint64_t seed) {
    /* wtype VX_SYNTH_KQ_MIX: Q4_K everywhere except Q6_K for attn_v, ffn_down
     * and the LM head, the split of common Q4_K_M GGUF files */
    const int mix = c && c->wtype == VX_SYNTH_KQ_MIX;
    const int wt = mix ? 12 : c ? c->wtype : 0, wt6 = mix ? 14 : wt;
    const int kq = kq_bytes(wt) > 0;
    if (!path || !c || c->n_embd % 32 || c->n_ff % 32 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
        (wt != 2 && wt != 8 && !kq) || (kq && (c->n_embd % 256 || c->n_ff % 256)))
        return VX_ERR_PARAM;
    const int hd = c->n_embd / c->n_heads, kvd = c->n_kv_heads * hd;
    const int nt = 9 * c->n_layers + 3;
    tinfo *t = (tinfo *)calloc((size_t)nt, sizeof(tinfo));
    int k = 0;
#define ADD(nm, d, a, b, ty) do { snprintf(t[k].name, 64, "%s", nm); t[k].nd = d; t[k].ne0 = a; t[k].ne1 = b; t[k].type = ty; k++; } while (0)
    char nm[64];
    for (int l = 0; l < c->n_layers; l++) {
        snprintf(nm, 64, "blk.%d.attn_norm.weight", l); ADD(nm, 1, c->n_embd, 1, 0);
        snprintf(nm, 64, "blk.%d.attn_q.weight", l); ADD(nm, 2, c->n_embd, c->n_embd, wt);
        snprintf(nm, 64, "blk.%d.attn_k.weight", l); ADD(nm, 2, c->n_embd, kvd, wt);
        snprintf(nm, 64, "blk.%d.attn_v.weight", l); ADD(nm, 2, c->n_embd, kvd, wt6);
        snprintf(nm, 64, "blk.%d.attn_output.weight", l); ADD(nm, 2, c->n_embd, c->n_embd, wt);
        snprintf(nm, 64, "blk.%d.ffn_norm.weight", l); ADD(nm, 1, c->n_embd, 1, 0);
        snprintf(nm, 64, "blk.%d.ffn_gate.weight", l); ADD(nm, 2, c->n_embd, c->n_ff, wt);
        snprintf(nm, 64, "blk.%d.ffn_up.weight", l); ADD(nm, 2, c->n_embd, c->n_ff, wt);
        snprintf(nm, 64, "blk.%d.ffn_down.weight", l); ADD(nm, 2, c->n_ff, c->n_embd, wt6);
    }
    ADD("token_embd.weight", 2, c->n_embd, c->n_vocab, wt);
    ADD("output_norm.weight", 1, c->n_embd, 1, 0);
    ADD("output.weight", 2, c->n_embd, c->n_vocab, wt6);
#undef ADD
    uint64_t off = 0;
    for (int i = 0; i < nt; i++) {
        uint64_t n = t[i].ne0 * t[i].ne1;
        t[i].bytes = t[i].type == 0 ? n * 4
                   : kq_bytes(t[i].type) ? (n / 256) * (uint64_t)kq_bytes(t[i].type)
                   : (n / 32) * (t[i].type == 8 ? 34 : 18);
        t[i].off = off;
        off += (t[i].bytes + 31) & ~31ull;
    }
    FILE *f = fopen(path, "wb");
    if (!f) { free(t); return VX_ERR_FILE; }
    w32(f, 0x46554747u);
    w32(f, 3);
    w64(f, (uint64_t)nt);
    w64(f, 8);
    /* key order matters to the reference's substring scan: head_count must
     * precede head_count_kv (src/gguf.c:526-527) */
    wstr(f, "general.architecture"); w32(f, 8); wstr(f, "llama");
    kv_u32(f, "llama.block_count", (uint32_t)c->n_layers);
    kv_u32(f, "llama.attention.head_count", (uint32_t)c->n_heads);
    kv_u32(f, "llama.attention.head_count_kv", (uint32_t)c->n_kv_heads);
    kv_u32(f, "llama.embedding_length", (uint32_t)c->n_embd);
    kv_u32(f, "llama.feedforward_length", (uint32_t)c->n_ff);
    wstr(f, "llama.rope.freq_base"); w32(f, 6); wr(f, &c->rope_theta, 4);
    kv_u32(f, "llama.vocab_size", (uint32_t)c->n_vocab);
    for (int i = 0; i < nt; i++) {
        wstr(f, t[i].name);
        w32(f, (uint32_t)t[i].nd);
        w64(f, t[i].ne0);
        if (t[i].nd == 2) w64(f, t[i].ne1);
        w32(f, (uint32_t)t[i].type);
        w64(f, t[i].off);
    }
    pad32(f);
    for (int i = 0; i < nt; i++) {
        uint8_t *buf = (uint8_t *)malloc(t[i].bytes ? t[i].bytes : 1);
        if (!buf) { fclose(f); free(t); return VX_ERR_MEMORY; }
        if (t[i].type == 0) {
            float *fb = (float *)buf;
            for (uint64_t j = 0; j < t[i].ne0 * t[i].ne1; j++) fb[j] = 1.0f;
        } else if (kq_bytes(t[i].type)) {
            const int64_t nsb = (int64_t)(t[i].ne0 * t[i].ne1 / 256);
            const int bb = kq_bytes(t[i].type);
#pragma omp parallel for schedule(static) num_threads(omp_get_num_procs())
            for (int64_t b = 0; b < nsb; b++) kq_block(t[i].type, seed, (uint32_t)i, (uint64_t)b, buf + (size_t)b * bb);
        } else {
            const int64_t nblk = (int64_t)(t[i].ne0 * t[i].ne1 / 32);
            const size_t bb = t[i].type == 8 ? 34 : 18;
            /* every core the process may run on, whatever OMP_NUM_THREADS says
             * (launchers such as torch.distributed.run set it to 1): a 70B-shape
             * checkpoint is ~70 G normals */
#pragma omp parallel for schedule(static) num_threads(omp_get_num_procs())
            for (int64_t b = 0; b < nblk; b++) {
                float x[32];
                for (int q = 0; q < 8; q++) normals4(seed, (uint32_t)i, (uint64_t)b * 8 + q, 0.02f, x + 4 * q);
                quant_block(t[i].type, x, buf + (size_t)b * bb);
            }
        }
        wr(f, buf, t[i].bytes);
        free(buf);
        pad32(f);
    }
    int bad = ferror(f);
    fclose(f);
    free(t);
    return bad ? VX_ERR_FILE : VX_OK;
}
