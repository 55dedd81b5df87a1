/*
 * vxo_fwd.c — CPU oracle ("O-fwd"): restatement of the reference's scalar
 * forward pass.  TEST INFRASTRUCTURE ONLY (see vxo.h).
 *
 * Arithmetic order follows the reference's non-AVX2 build exactly so that the
 * result is bit-identical to the reference compiled with -O2 -march=x86-64
 * (tests/test_oracle_pin.py).  The one semantic change is the reference's
 * in-place attn_o GEMV (src/model.c:543-544), which races under OpenMP; here
 * it is out of place, which is what the reference computes at one thread
 * with a private copy of its input.
 */
#include "vxo.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* fp16 codec: reference src/quantize.c:17-57                              */
/* ---------------------------------------------------------------------- */

/* src/quantize.c:37-57 (exact decode, subnormals normalised by shifting). */
float vxo_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t e = (uint32_t)(h >> 10) & 0x1Fu;
    uint32_t m = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign << 31;
        } else {
            while ((m & 0x400u) == 0) { m <<= 1; e--; }
            e++;
            m &= 0x3FFu;
            bits = (sign << 31) | ((e + 112u) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = (sign << 31) | (0xFFu << 23) | (m << 13);
    } else {
        bits = (sign << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* src/quantize.c:17-35: truncating encode, fp16 subnormals flushed to 0. */
uint16_t vxo_fp32_to_fp16_trunc(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 31) & 1u;
    uint32_t e = (x >> 23) & 0xFFu;
    uint32_t m = x & 0x7FFFFFu;
    if (e == 0) return (uint16_t)(sign << 15);
    if (e == 0xFF) return (uint16_t)((sign << 15) | (0x1Fu << 10) | (m >> 13));
    int32_t ne = (int32_t)e - 127 + 15;
    if (ne <= 0) return (uint16_t)(sign << 15);
    if (ne >= 31) return (uint16_t)((sign << 15) | (0x1Fu << 10));
    return (uint16_t)((sign << 15) | ((uint32_t)ne << 10) | (m >> 13));
}

/* ---------------------------------------------------------------------- */
/* Quantised blocks                                                        */
/* ---------------------------------------------------------------------- */
/* Q4_0: 2-byte fp16 scale + 16 bytes; element 2j is the LOW nibble of byte
 * j and element 2j+1 the HIGH nibble (interleaved, src/quantize.c:584-588).
 * Q8_0: 2-byte fp16 scale + 32 int8 (src/quantize.c:642-651). */
#define Q4_BYTES 18
#define Q8_BYTES 34

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* src/quantize.c:88-114 (d = amax/7, truncating int conversion, clamp). */
void vxo_quantize_row_q4_0(const float *x, void *vy, int n) {
    uint8_t *y = (uint8_t *)vy;
    for (int i = 0; i < n; i += 32) {
        uint8_t *blk = y + (size_t)(i / 32) * Q4_BYTES;
        int rem = (i + 32 <= n) ? 32 : (n - i);
        float amax = 0.0f;
        for (int j = 0; j < rem; j++) {
            float ax = fabsf(x[i + j]);
            if (ax > amax) amax = ax;
        }
        float d = amax / 7.0f;
        if (d < 1e-10f) d = 1e-10f;
        uint16_t h = vxo_fp32_to_fp16_trunc(d);
        blk[0] = (uint8_t)(h & 0xFF);
        blk[1] = (uint8_t)(h >> 8);
        float id = 1.0f / d;
        for (int j = 0; j < rem; j += 2) {
            int a = (int)(x[i + j] * id);
            int b = (int)(x[i + j + 1] * id);
            if (a < -8) a = -8;
            if (a > 7) a = 7;
            if (b < -8) b = -8;
            if (b > 7) b = 7;
            blk[2 + j / 2] = (uint8_t)((uint8_t)(a + 8) | ((uint8_t)(b + 8) << 4));
        }
        for (int j = rem; j < 32; j += 2) blk[2 + j / 2] = 0;
    }
}

/* Q8_0 quantiser.  The reference has none; this is the standard GGML rule
 * (d = amax/127, q = round-half-away(x/d)) used to write fixtures. */
void vxo_quantize_row_q8_0(const float *x, void *vy, int n) {
    uint8_t *y = (uint8_t *)vy;
    for (int i = 0; i < n; i += 32) {
        uint8_t *blk = y + (size_t)(i / 32) * Q8_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float ax = fabsf(x[i + j]);
            if (ax > amax) amax = ax;
        }
        float d = amax / 127.0f;
        uint16_t h = vxo_fp32_to_fp16_trunc(d);
        blk[0] = (uint8_t)(h & 0xFF);
        blk[1] = (uint8_t)(h >> 8);
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        for (int j = 0; j < 32; j++) {
            float v = roundf(x[i + j] * id);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            blk[2 + j] = (uint8_t)(int8_t)v;
        }
    }
}

/* src/quantize.c:578-591 (g_synthetic_weight_scale is 1.0 and multiplies
 * exactly, so it is omitted). */
void vxo_dequant_q4_0(const void *vx, float *y, int n) {
    const uint8_t *x = (const uint8_t *)vx;
    for (int i = 0; i < n; i += 32) {
        const uint8_t *blk = x + (size_t)(i / 32) * Q4_BYTES;
        float d = vxo_fp16_to_fp32(rd16(blk));
        for (int j = 0; j < 32 && (i + j) < n; j += 2) {
            uint8_t byte = blk[2 + j / 2];
            int8_t a = (int8_t)((int8_t)(byte & 0x0F) - 8);
            int8_t b = (int8_t)((int8_t)(byte >> 4) - 8);
            y[i + j] = a * d;
            y[i + j + 1] = b * d;
        }
    }
}

/* src/quantize.c:642-651. */
void vxo_dequant_q8_0(const void *vx, float *y, int n) {
    const uint8_t *x = (const uint8_t *)vx;
    for (int i = 0; i < n; i += 32) {
        const uint8_t *blk = x + (size_t)(i / 32) * Q8_BYTES;
        float d = vxo_fp16_to_fp32(rd16(blk));
        for (int j = 0; j < 32 && (i + j) < n; j++) y[i + j] = (int8_t)blk[2 + j] * d;
    }
}

#define T_F32 0
#define T_Q4_0 2
#define T_Q8_0 8

static size_t row_bytes(int type, int cols) {
    if (type == T_Q4_0) return (size_t)(cols / 32) * Q4_BYTES;
    if (type == T_Q8_0) return (size_t)(cols / 32) * Q8_BYTES;
    if (vxo_kquant_block_bytes(type)) return (size_t)(cols / 256) * vxo_kquant_block_bytes(type);
    return (size_t)cols * 4;
}

/* K-quant rows (types 10..15) decode as the reference's vx_dequantize does;
 * their GEMV is then the f32 GEMV of every other type.  The reference's own
 * apply_gemv runs Q2_K/Q3_K/Q4_K through int8-rounded activations
 * (src/quantize.c:439-561, with the Q4_K dot dropping half of every
 * super-block) and sums Q5_K/Q6_K/Q8_K in another order (:486-505); its
 * sparse-row up projection and its embedding lookup decode as here
 * (src/model.c:191-198, :462-496).  See oracle/vxo_kquant.c. */
static void dequant_row(int type, const uint8_t *src, float *dst, int cols) {
    if (type == T_Q4_0) vxo_dequant_q4_0(src, dst, cols);
    else if (type == T_Q8_0) vxo_dequant_q8_0(src, dst, cols);
    else if (vxo_kquant_block_bytes(type)) vxo_dequant_kquant(type, src, dst, cols);
    else memcpy(dst, src, (size_t)cols * 4);
}

/* One row of vx_gemv_f32 (src/tensor.c:103-120) applied to a dequantised
 * row; the reference dequantises the whole matrix first
 * (src/model.c:216-219, :235-241), which produces the same floats. */
static float dot_row(const float *A, const float *x, int cols) {
    float sum = 0.0f;
    int j = 0;
    for (; j + 4 <= cols; j += 4)
        sum += A[j] * x[j] + A[j + 1] * x[j + 1] + A[j + 2] * x[j + 2] + A[j + 3] * x[j + 3];
    for (; j < cols; j++) sum += A[j] * x[j];
    return sum;
}

/* apply_gemv / apply_gemv_sparse_rows (src/model.c:169-245) for F32, Q4_0
 * and Q8_0 in the scalar build; gate != NULL selects the sparse-row variant
 * (src/tensor.c:71-88): rows with |gate| < thr produce 0. */
static void gemv(int type, const uint8_t *w, const float *x, float *y, int rows, int cols,
                 const float *gate, float thr) {
    size_t rb = row_bytes(type, cols);
#pragma omp parallel
    {
        float *tmp = (float *)malloc((size_t)cols * sizeof(float));
#pragma omp for
        for (int i = 0; i < rows; i++) {
            if (gate && fabsf(gate[i]) < thr) { y[i] = 0.0f; continue; }
            dequant_row(type, w + (size_t)i * rb, tmp, cols);
            y[i] = dot_row(tmp, x, cols);
        }
        free(tmp);
    }
}

void vxo_qgemv(int type, const void *w, const float *x, float *y, int M, int rows, int cols) {
    for (int m = 0; m < M; m++)
        gemv(type, (const uint8_t *)w, x + (size_t)m * cols, y + (size_t)m * rows, rows, cols, NULL, 0.0f);
}

/* ---------------------------------------------------------------------- */
/* Elementwise ops: reference src/tensor.c scalar branches                 */
/* ---------------------------------------------------------------------- */

/* src/tensor.c:132-140 */
void vxo_rms_norm(float *o, const float *x, const float *w, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float rms = sqrtf(ss / n + 1e-5f);
    if (rms < 1e-10f) {
        for (int i = 0; i < n; i++) o[i] = 0.0f;
        return;
    }
    float inv = 1.0f / rms;
    for (int i = 0; i < n; i++) o[i] = w[i] * (x[i] * inv);
}

/* src/tensor.c:160-169 */
void vxo_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    if (sum < 1e-10f) {
        for (int i = 0; i < n; i++) x[i] = 1.0f / n;
        return;
    }
    float inv = 1.0f / (sum + 1e-10f);
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* src/tensor.c:173-187 and :249-270 (rope_dims = head_dim for llama). */
void vxo_rope(float *q, float *k, int pos, int n_heads, int n_kv_heads, int head_dim, float theta) {
    int npairs = head_dim / 2;
    float *fcr = (float *)malloc((size_t)npairs * sizeof(float));
    float *fci = (float *)malloc((size_t)npairs * sizeof(float));
    for (int i = 0; i < npairs; i++) {
        float freq = 1.0f / powf(theta, (float)(i * 2) / head_dim);
        float val = pos * freq;
        fcr[i] = cosf(val);
        fci[i] = sinf(val);
    }
    int nk = n_kv_heads > 0 ? n_kv_heads : n_heads;
    int mh = n_heads > nk ? n_heads : nk;
    for (int h = 0; h < mh; h++) {
        if (h < n_heads) {
            float *qh = q + (size_t)h * head_dim;
            for (int i = 0; i < head_dim; i += 2) {
                int p = i / 2;
                float a = qh[i], b = qh[i + 1];
                qh[i] = a * fcr[p] - b * fci[p];
                qh[i + 1] = a * fci[p] + b * fcr[p];
            }
        }
        if (h < nk) {
            float *kh = k + (size_t)h * head_dim;
            for (int i = 0; i < head_dim; i += 2) {
                int p = i / 2;
                float a = kh[i], b = kh[i + 1];
                kh[i] = a * fcr[p] - b * fci[p];
                kh[i + 1] = a * fci[p] + b * fcr[p];
            }
        }
    }
    free(fcr);
    free(fci);
}

/* src/tensor.c:277 */
void vxo_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* ---------------------------------------------------------------------- */
/* GGUF loading: reference src/gguf.c:31-44, :112-217, :293-489, :495-582   */
/* and weight resolution src/format.c:230-322 (GGUF tensor names only).     */
/* ---------------------------------------------------------------------- */

typedef struct {
    char name[96];
    int type;
    int ne0, ne1;
    const uint8_t *data;
} vxo_tensor;

struct vxo_model {
    int n_layers, n_heads, n_kv_heads, n_embd, n_head_dim, n_ff, n_vocab, n_ctx;
    float rope_theta;
    uint8_t *file;
    size_t file_size;
    vxo_tensor *t;
    int nt;
    vxo_tensor *tok_embd, *output, *output_norm;
    vxo_tensor **attn_norm, **wq, **wk, **wv, **wo, **ffn_norm, **wg, **wu, **wd;
    float *k_cache, *v_cache;
    int cache_len;
};

static int skip_value(const uint8_t *p, size_t size, uint64_t *o, uint32_t vt) {
    switch (vt) {
        case 0: case 1: case 7: *o += 1; return 0;
        case 2: case 3: *o += 2; return 0;
        case 4: case 5: case 6: *o += 4; return 0;
        case 10: case 11: case 12: *o += 8; return 0;
        case 8: {
            uint64_t sl;
            if (*o + 8 > size) return -1;
            memcpy(&sl, p + *o, 8);
            *o += 8 + sl;
            return 0;
        }
        case 9: {
            uint32_t at;
            uint64_t al;
            if (*o + 12 > size) return -1;
            memcpy(&at, p + *o, 4);
            memcpy(&al, p + *o + 4, 8);
            *o += 12;
            for (uint64_t j = 0; j < al; j++)
                if (skip_value(p, size, o, at) != 0) return -1;
            return 0;
        }
        default: return -1;
    }
}

/* gguf_scan_u32/_f32/_str (src/gguf.c:293-489): scan KV pairs from *off for
 * the first key CONTAINING `key` with a matching value type.  On a miss the
 * scan offset moves to the end of the KV section, as in the reference, so a
 * missing key makes every later scan fall back too. */
static int scan_kv(const uint8_t *p, size_t size, uint64_t *off, uint64_t nkv, const char *key,
                   int want, void *out, int out_len) {
    uint64_t o = *off;
    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        if (o + 8 > size) return -1;
        memcpy(&kl, p + o, 8);
        o += 8;
        if (o + kl > size) return -1;
        char k[128];
        int nc = kl > 127 ? 127 : (int)kl;
        memcpy(k, p + o, (size_t)nc);
        k[nc] = 0;
        o += kl;
        uint32_t vt;
        if (o + 4 > size) return -1;
        memcpy(&vt, p + o, 4);
        o += 4;
        int hit = strstr(k, key) != NULL;
        if (hit && want == 0 && (vt == 4 || vt == 5)) { memcpy(out, p + o, 4); return 0; }
        if (hit && want == 1 && vt == 6) { memcpy(out, p + o, 4); return 0; }
        if (hit && want == 2 && vt == 8) {
            uint64_t sl;
            memcpy(&sl, p + o, 8);
            int c = sl > (uint64_t)(out_len - 1) ? out_len - 1 : (int)sl;
            memcpy(out, p + o + 8, (size_t)c);
            ((char *)out)[c] = 0;
            return 0;
        }
        if (skip_value(p, size, &o, vt) != 0) return -1;
    }
    *off = o;
    return -1;
}

static uint32_t scan_u32(const uint8_t *p, size_t s, uint64_t *o, uint64_t n, const char *k, uint32_t fb) {
    uint32_t v;
    return scan_kv(p, s, o, n, k, 0, &v, 0) == 0 ? v : fb;
}

static vxo_tensor *find(vxo_model *m, const char *name) {
    for (int i = 0; i < m->nt; i++)
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}

static vxo_tensor *find_l(vxo_model *m, const char *fmt, int l) {
    char nm[96];
    snprintf(nm, sizeof nm, fmt, l);
    return find(m, nm);
}

vxo_model *vxo_model_load(const char *path, int n_ctx) {
    FILE *fp = fopen(path, "rb");
    if (!fp) return NULL;
    fseek(fp, 0, SEEK_END);
    size_t size = (size_t)ftell(fp);
    fseek(fp, 0, SEEK_SET);
    uint8_t *buf = (uint8_t *)malloc(size);
    if (!buf || fread(buf, 1, size, fp) != size) { fclose(fp); free(buf); return NULL; }
    fclose(fp);
    uint32_t magic;
    uint64_t nt, nkv;
    memcpy(&magic, buf, 4);
    if (magic != 0x46554747u) { free(buf); return NULL; }
    memcpy(&nt, buf + 8, 8);
    memcpy(&nkv, buf + 16, 8);
    uint64_t o = 24;
    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        memcpy(&kl, buf + o, 8);
        o += 8 + kl;
        uint32_t vt;
        memcpy(&vt, buf + o, 4);
        o += 4;
        if (skip_value(buf, size, &o, vt) != 0) { free(buf); return NULL; }
    }
    vxo_model *m = (vxo_model *)calloc(1, sizeof(vxo_model));
    m->file = buf;
    m->file_size = size;
    m->nt = (int)nt;
    m->t = (vxo_tensor *)calloc(nt, sizeof(vxo_tensor));
    uint64_t *offs = (uint64_t *)calloc(nt, sizeof(uint64_t));
    for (uint64_t i = 0; i < nt; i++) {
        uint64_t nl;
        memcpy(&nl, buf + o, 8);
        o += 8;
        int c = nl > 95 ? 95 : (int)nl;
        memcpy(m->t[i].name, buf + o, (size_t)c);
        o += nl;
        uint32_t nd;
        memcpy(&nd, buf + o, 4);
        o += 4;
        uint64_t dims[4] = {1, 1, 1, 1};
        for (uint32_t d = 0; d < nd; d++) { memcpy(&dims[d], buf + o, 8); o += 8; }
        uint32_t ty;
        memcpy(&ty, buf + o, 4);
        o += 4;
        memcpy(&offs[i], buf + o, 8);
        o += 8;
        m->t[i].type = (int)ty;
        m->t[i].ne0 = (int)dims[0];
        m->t[i].ne1 = (int)dims[1];
    }
    uint64_t data0 = o + (32 - o % 32) % 32; /* src/gguf.c:213-215 */
    for (uint64_t i = 0; i < nt; i++) m->t[i].data = buf + data0 + offs[i];
    free(offs);

    /* Scan order and fallbacks of src/gguf.c:524-533. */
    uint64_t ko = 24;
    m->n_layers = (int)scan_u32(buf, size, &ko, nkv, "block_count", 32);
    m->n_heads = (int)scan_u32(buf, size, &ko, nkv, "head_count", 32);
    m->n_kv_heads = (int)scan_u32(buf, size, &ko, nkv, "head_count_kv", (uint32_t)m->n_heads);
    m->n_embd = (int)scan_u32(buf, size, &ko, nkv, "embedding_length", 4096);
    m->n_ff = (int)scan_u32(buf, size, &ko, nkv, "feedforward_length", 0);
    m->n_vocab = (int)scan_u32(buf, size, &ko, nkv, "vocab_size", 0);
    if (m->n_vocab == 0) m->n_vocab = (int)scan_u32(buf, size, &ko, nkv, "vocabulary.vocab_size", 0);
    float th;
    m->rope_theta = scan_kv(buf, size, &ko, nkv, "rope.freq_base", 1, &th, 0) == 0 ? th : 10000.0f;
    if (m->n_kv_heads <= 0) m->n_kv_heads = m->n_heads;
    m->n_head_dim = m->n_embd / (m->n_heads > 0 ? m->n_heads : 1);
    m->n_ctx = n_ctx > 0 ? n_ctx : 4096; /* src/gguf.c:548 fixes 4096 */

    int L = m->n_layers;
    m->tok_embd = find(m, "token_embd.weight");
    m->output = find(m, "output.weight");
    if (!m->output) m->output = m->tok_embd; /* src/format.c:238 */
    m->output_norm = find(m, "output_norm.weight");
    vxo_tensor ***tabs[9] = {&m->attn_norm, &m->wq, &m->wk, &m->wv, &m->wo,
                             &m->ffn_norm, &m->wg, &m->wu, &m->wd};
    const char *fmts[9] = {"blk.%d.attn_norm.weight", "blk.%d.attn_q.weight", "blk.%d.attn_k.weight",
                           "blk.%d.attn_v.weight", "blk.%d.attn_output.weight", "blk.%d.ffn_norm.weight",
                           "blk.%d.ffn_gate.weight", "blk.%d.ffn_up.weight", "blk.%d.ffn_down.weight"};
    for (int j = 0; j < 9; j++) {
        *tabs[j] = (vxo_tensor **)calloc((size_t)L, sizeof(vxo_tensor *));
        for (int l = 0; l < L; l++) (*tabs[j])[l] = find_l(m, fmts[j], l);
    }
    /* vx_model_auto_detect_dims (src/format.c:287-322) */
    if (m->n_ff == 0 && L > 0 && m->wg[0]) m->n_ff = m->wg[0]->ne1;
    if (m->n_vocab <= 32000 && m->tok_embd && m->tok_embd->ne1 > m->n_vocab) m->n_vocab = m->tok_embd->ne1;

    size_t kvn = (size_t)L * m->n_ctx * m->n_kv_heads * m->n_head_dim;
    m->k_cache = (float *)calloc(kvn, sizeof(float));
    m->v_cache = (float *)calloc(kvn, sizeof(float));
    if (!m->k_cache || !m->v_cache) { vxo_model_free(m); return NULL; }
    return m;
}

void vxo_model_free(vxo_model *m) {
    if (!m) return;
    free(m->attn_norm); free(m->wq); free(m->wk); free(m->wv); free(m->wo);
    free(m->ffn_norm); free(m->wg); free(m->wu); free(m->wd);
    free(m->k_cache); free(m->v_cache);
    free(m->t);
    free(m->file);
    free(m);
}

void vxo_model_config(const vxo_model *m, int *out) {
    out[0] = m->n_layers; out[1] = m->n_heads; out[2] = m->n_kv_heads; out[3] = m->n_embd;
    out[4] = m->n_head_dim; out[5] = m->n_ff; out[6] = m->n_vocab; out[7] = m->n_ctx;
}
float vxo_model_rope_theta(const vxo_model *m) { return m->rope_theta; }
int vxo_model_cache_len(const vxo_model *m) { return m->cache_len; }
void vxo_model_set_cache_len(vxo_model *m, int len) {
    /* vx_model_kv_truncate semantics (src/model.c:384-389) plus direct set */
    if (len < 0) len = 0;
    m->cache_len = len;
}

/* ---------------------------------------------------------------------- */
/* Forward: reference src/model.c:391-628 (+ apply_norm :247-273 and        */
/* apply_attention :275-341), llama / SwiGLU / RMSNorm branch.              */
/* ---------------------------------------------------------------------- */

static void apply_norm(float *x, float *tmp, const vxo_tensor *w, int dim, float *ones) {
    const float *wt = (w && w->type == T_F32) ? (const float *)w->data : ones;
    vxo_rms_norm(tmp, x, wt, dim);
    memcpy(x, tmp, (size_t)dim * sizeof(float));
}

static void attention(vxo_model *m, float *out, const float *q, const float *k, const float *v, int layer,
                      float *scores) {
    int H = m->n_heads, KH = m->n_kv_heads, hd = m->n_head_dim;
    int kvd = KH * hd;
    int pos = m->cache_len;
    int max_ctx = m->n_ctx;
    if (pos >= max_ctx) { pos = max_ctx - 1; m->cache_len = pos; }
    int cs = pos + 1;
    size_t loff = (size_t)layer * max_ctx * kvd;
    memcpy(m->k_cache + loff + (size_t)pos * kvd, k, (size_t)kvd * sizeof(float));
    memcpy(m->v_cache + loff + (size_t)pos * kvd, v, (size_t)kvd * sizeof(float));
#pragma omp parallel for
    for (int h = 0; h < H; h++) {
        const float *qh = q + (size_t)h * hd;
        int kvh = KH == 1 ? 0 : (h * KH / H);
        float *ls = scores + (size_t)h * max_ctx;
        float scale = 1.0f / sqrtf((float)hd);
        for (int t = 0; t < cs; t++) {
            const float *kt = m->k_cache + loff + (size_t)t * kvd + (size_t)kvh * hd;
            float s = 0;
            for (int d = 0; d < hd; d++) s += qh[d] * kt[d];
            ls[t] = (t <= pos) ? s * scale : -1e9f;
        }
        vxo_softmax(ls, cs);
        for (int d = 0; d < hd; d++) {
            float sum = 0;
            for (int t = 0; t < cs; t++)
                sum += ls[t] * m->v_cache[loff + (size_t)t * kvd + (size_t)kvh * hd + d];
            out[(size_t)h * hd + d] = sum;
        }
    }
}

static int forward_impl(vxo_model *m, const int *tokens, int n, float *logits, int all) {
    int E = m->n_embd, L = m->n_layers, H = m->n_heads, KH = m->n_kv_heads, hd = m->n_head_dim;
    int F = m->n_ff, V = m->n_vocab;
    int kvd = KH * hd;
    if (E <= 0 || E > 8192) return -4;
    float *x = (float *)calloc((size_t)E, 4), *xo = (float *)calloc((size_t)E, 4);
    float *q = (float *)calloc((size_t)E, 4), *k = (float *)calloc((size_t)kvd, 4);
    float *v = (float *)calloc((size_t)kvd, 4), *ao = (float *)calloc((size_t)E, 4);
    float *ao2 = (float *)calloc((size_t)E, 4), *tmp = (float *)calloc((size_t)E, 4);
    float *fh = (float *)calloc((size_t)F, 4), *fh2 = (float *)calloc((size_t)F, 4);
    float *ones = (float *)malloc((size_t)E * 4);
    float *scores = (float *)malloc((size_t)H * m->n_ctx * 4);
    float *row = (float *)malloc((size_t)E * 4);
    for (int i = 0; i < E; i++) ones[i] = 1.0f;
    int rc = 0;
    for (int p = 0; p < n; p++) {
        int tok = tokens[p];
        int cache_pos = m->cache_len;
        memset(x, 0, (size_t)E * 4);
        if (tok < 0 || !m->tok_embd || tok >= m->tok_embd->ne1) { rc = -4; break; }
        {   /* embedding row (src/model.c:454-500): dequantise row `tok` */
            const vxo_tensor *te = m->tok_embd;
            dequant_row(te->type, te->data + (size_t)tok * row_bytes(te->type, te->ne0), row, te->ne0);
            memcpy(x, row, (size_t)E * 4);
        }
        for (int l = 0; l < L; l++) {
            memcpy(xo, x, (size_t)E * 4);
            apply_norm(x, tmp, m->attn_norm[l], E, ones);
            gemv(m->wq[l]->type, m->wq[l]->data, x, q, E, E, NULL, 0);
            gemv(m->wk[l]->type, m->wk[l]->data, x, k, kvd, E, NULL, 0);
            gemv(m->wv[l]->type, m->wv[l]->data, x, v, kvd, E, NULL, 0);
            vxo_rope(q, k, cache_pos, H, KH, hd, m->rope_theta);
            attention(m, ao, q, k, v, l, scores);
            /* out-of-place attn_o (fix of src/model.c:543-544) */
            gemv(m->wo[l]->type, m->wo[l]->data, ao, ao2, E, E, NULL, 0);
            for (int i = 0; i < E; i++) x[i] = xo[i] + ao2[i];
            memcpy(xo, x, (size_t)E * 4);
            apply_norm(x, tmp, m->ffn_norm[l], E, ones);
            memset(fh, 0, (size_t)F * 4);
            memset(fh2, 0, (size_t)F * 4);
            gemv(m->wg[l]->type, m->wg[l]->data, x, fh, F, E, NULL, 0);
            vxo_silu(fh, F);
            gemv(m->wu[l]->type, m->wu[l]->data, x, fh2, F, E, fh, 0.01f);
            for (int i = 0; i < F; i++) fh[i] = fh[i] * fh2[i];
            memset(ao, 0, (size_t)E * 4);
            gemv(m->wd[l]->type, m->wd[l]->data, fh, ao, E, F, NULL, 0);
            for (int i = 0; i < E; i++) x[i] = xo[i] + ao[i];
        }
        m->cache_len++;
        if (p == n - 1 || all) {
            float *lg = all ? logits + (size_t)p * V : logits;
            float *xf = tmp;   /* final norm must not disturb x for later tokens */
            memcpy(row, x, (size_t)E * 4);
            if (m->output_norm) apply_norm(row, xf, m->output_norm, E, ones);
            for (int i = 0; i < V; i++) lg[i] = -1e30f;
            const vxo_tensor *ow = m->output;
            if (ow) {
                int orows = ow->ne1, ocols = ow->ne0 > 0 ? ow->ne0 : E;
                if (orows > 0 && orows <= V * 2) gemv(ow->type, ow->data, row, lg, orows, ocols, NULL, 0);
            }
        }
    }
    free(x); free(xo); free(q); free(k); free(v); free(ao); free(ao2); free(tmp);
    free(fh); free(fh2); free(ones); free(scores); free(row);
    return rc;
}

int vxo_forward(vxo_model *m, const int *tokens, int n, float *logits) {
    return forward_impl(m, tokens, n, logits, 0);
}

int vxo_forward_all(vxo_model *m, const int *tokens, int n, float *logits) {
    return forward_impl(m, tokens, n, logits, 1);
}
