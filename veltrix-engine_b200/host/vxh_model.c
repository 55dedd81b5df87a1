/*
 * vxh_model.c — the reference's model API (include/model.h:6-8,
 * include/veltrix.h:175-183) on the B200 back end.
 *
 * vx_model_create  maps the GGUF file, reads the hyper-parameters the way the
 *                  reference does (src/gguf.c:524-551, src/format.c:185-203,
 *                  :287-322), resolves the GGUF tensor names
 *                  (src/format.c:84-150, :230-281) and uploads every weight
 *                  to the current CUDA device (vxc_net_create).  The host
 *                  mapping is released afterwards; vx_model.tensors stays NULL.
 * vx_model_forward keeps the reference's contract (src/model.c:391-628):
 *                  appends n_tokens at cache_len, advances cache_len, writes
 *                  the last token's logits.  cache_len is re-read on every
 *                  call, so callers that set it directly (the reference's
 *                  speculative loop does) keep working.  The KV cache is
 *                  created at the first forward with config.n_ctx positions
 *                  (4096 unless the caller changed it, src/gguf.c:548).
 * Deviations: positions past n_ctx are an error (VX_ERR_PARAM) instead of
 * being clamped onto position n_ctx-1 (src/model.c:282-285); compute levels
 * other than VX_COMPUTE_EXACT are refused (VX_ERR_UNSUPPORTED) because they
 * change the model (src/model.c:503-511).
 */
#define _GNU_SOURCE
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "model.h"
#include "veltrix.h"
#include "veltrix_cuda.h"
#include "vxh_gguf.h"
#include "vxh_model.h"
#include "veltrix_synth.h"

static vx_compute_level g_level = VX_COMPUTE_EXACT;
static int g_threads = 1;
static int g_timing = 0;
static double g_fwd_us = 0.0;
static long g_fwd_calls = 0, g_fwd_tokens = 0;

static double now_us(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e6 + (double)ts.tv_nsec / 1e3;
}

static vxc_tensor_view view_of(const vxh_tensor *t) {
    vxc_tensor_view v = {0, 0, 0, NULL};
    if (!t) return v;
    v.type = t->type;
    v.cols = (int)t->ne[0];
    v.rows = (int)(t->ne[1] * t->ne[2] * t->ne[3]);
    v.data = t->data;
    return v;
}

static const vxh_tensor *find_l(const vxh_gguf *g, const char *fmt, int l) {
    char nm[128];
    snprintf(nm, sizeof nm, fmt, l);
    return vxh_gguf_find(g, nm);
}

/* arch table entries with SwiGLU + RMSNorm and no biases
 * (src/format.c:164-183); anything else is not on the device path. */
static int arch_supported(const char *a) {
    static const char *ok[] = {"llama", "mistral", "mistralnemo", "qwen2", "qwen2.5", "qwen3", "qwen3.5",
                               "qwen3.6", "qwen3moe", ""};
    for (size_t i = 0; i < sizeof ok / sizeof ok[0]; i++)
        if (strcmp(a, ok[i]) == 0) return 1;
    /* unknown names default to llama in the reference (src/format.c:199-202) */
    static const char *bad[] = {"gemma", "gemma2", "gemma3", "gemma-3", "gemma4", "gemma-4", "phi2", "phi3",
                                "starcoder2"};
    for (size_t i = 0; i < sizeof bad / sizeof bad[0]; i++)
        if (strcmp(a, bad[i]) == 0) return 0;
    return 1;
}

/* A model handle around a device net (the handle owns net and tp). */
static vx_error wrap_net(vxc_net *net, vxc_tp *tp, int dev, const vxc_net_config *nc, vx_model **out) {
    vxb_model *m = (vxb_model *)calloc(1, sizeof(vxb_model));
    if (!m) { vxc_net_destroy(net); return VX_ERR_MEMORY; }
    m->net = net;
    m->tp = tp;
    m->device = dev;
    vx_model_config *c = &m->pub.config;
    c->n_layers = nc->n_layers;
    c->n_heads = nc->n_heads;
    c->n_kv_heads = nc->n_kv_heads;
    c->n_embd = nc->n_embd;
    c->n_head_dim = nc->n_head_dim;
    c->n_ff = nc->n_ff;
    c->n_vocab = nc->n_vocab;
    c->n_ctx = 4096;
    c->rope_theta = nc->rope_theta;
    c->n_threads = g_threads;
    c->arch = VX_ARCH_LLAMA;
    c->mlp_type = VX_MLP_SWIGLU;
    c->norm_type = VX_NORM_RMS;
    m->pub.cache_len = 0;
    *out = &m->pub;
    return VX_OK;
}

/* Load `path` onto the current device; with tp != NULL only this rank's
 * shard of the weights (the handle then owns tp). */
static vx_error model_create(const char *path, vxc_tp *tp, vx_model **out) {
    int dev = vxc_device_current();
    vxh_gguf g;
    int rc = vxh_gguf_open(path, &g);
    if (rc) return (vx_error)rc;
    if (!arch_supported(g.arch)) {
        fprintf(stderr, "veltrix-b200: architecture '%s' is not supported on the device path\n", g.arch);
        vxh_gguf_close(&g);
        return VX_ERR_UNSUPPORTED;
    }
    int L = g.n_layers, H = g.n_heads, KH = g.n_kv_heads > 0 ? g.n_kv_heads : g.n_heads, E = g.n_embd;
    const vxh_tensor *te = vxh_gguf_find(&g, "token_embd.weight");
    const vxh_tensor *to = vxh_gguf_find(&g, "output.weight");
    const vxh_tensor *tn = vxh_gguf_find(&g, "output_norm.weight");
    int F = g.n_ff, V = g.n_vocab;
    if (F == 0) {   /* src/format.c:291-306 */
        const vxh_tensor *tg = find_l(&g, "blk.%d.ffn_gate.weight", 0);
        if (tg) F = (int)tg->ne[1];
    }
    if (V <= 32000 && te && (int)te->ne[1] > V) V = (int)te->ne[1];   /* src/format.c:309-321 */
    if (!te || L <= 0 || H <= 0 || E <= 0 || E > 8192 || F <= 0) {
        vxh_gguf_close(&g);
        return VX_ERR_FORMAT;
    }
    if (find_l(&g, "blk.%d.attn_q.bias", 0) || find_l(&g, "blk.%d.ffn_up.bias", 0)) {
        fprintf(stderr, "veltrix-b200: models with projection biases are not supported\n");
        vxh_gguf_close(&g);
        return VX_ERR_UNSUPPORTED;
    }
    vxc_layer_views *lv = (vxc_layer_views *)calloc((size_t)L, sizeof *lv);
    for (int l = 0; l < L; l++) {
        lv[l].attn_norm = view_of(find_l(&g, "blk.%d.attn_norm.weight", l));
        lv[l].wq = view_of(find_l(&g, "blk.%d.attn_q.weight", l));
        lv[l].wk = view_of(find_l(&g, "blk.%d.attn_k.weight", l));
        lv[l].wv = view_of(find_l(&g, "blk.%d.attn_v.weight", l));
        lv[l].wo = view_of(find_l(&g, "blk.%d.attn_output.weight", l));
        lv[l].ffn_norm = view_of(find_l(&g, "blk.%d.ffn_norm.weight", l));
        lv[l].wg = view_of(find_l(&g, "blk.%d.ffn_gate.weight", l));
        lv[l].wu = view_of(find_l(&g, "blk.%d.ffn_up.weight", l));
        lv[l].wd = view_of(find_l(&g, "blk.%d.ffn_down.weight", l));
    }
    vxc_net_config nc;
    memset(&nc, 0, sizeof nc);
    nc.n_layers = L;
    nc.n_heads = H;
    nc.n_kv_heads = KH;
    nc.n_embd = E;
    nc.n_head_dim = E / H;
    nc.n_ff = F;
    nc.n_vocab = V;
    nc.rope_theta = g.rope_theta;
    nc.max_pos = 16384;
    vxc_tensor_view ve = view_of(te), vo = view_of(to), vn = view_of(tn);
    vxc_net *net = NULL;
    rc = vxc_net_create_tp(&nc, &ve, tn ? &vn : NULL, to ? &vo : NULL, lv, tp, &net);
    free(lv);
    vxh_gguf_close(&g);
    if (rc) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return rc == -3 ? VX_ERR_MEMORY : (vx_error)rc;
    }
    return wrap_net(net, tp, dev, &nc, out);
}

vx_error vx_model_create(const char *path, vx_model **out) {
    if (!path || !out) return VX_ERR_PARAM;
    int dev = vxc_device_current();
    if (dev < 0 || vxc_device_init(dev) != 0) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return VX_ERR_UNSUPPORTED;
    }
    return model_create(path, NULL, out);
}

vx_error vx_model_create_tp(const char *path, int rank, int world, const void *nccl_id, vx_model **out) {
    if (!path || !out || !nccl_id || world < 1 || rank < 0 || rank >= world) return VX_ERR_PARAM;
    int dev = vxc_device_current();
    if (dev < 0 || vxc_device_init(dev) != 0) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return VX_ERR_UNSUPPORTED;
    }
    vxc_tp *tp = NULL;
    int rc = vxc_tp_create(nccl_id, rank, world, &tp);
    if (rc) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return rc == -4 ? VX_ERR_PARAM : VX_ERR_UNSUPPORTED;
    }
    vx_error e = model_create(path, tp, out);
    if (e != VX_OK) vxc_tp_destroy(tp);
    return e;
}

vx_error vx_model_create_synth(const vx_synth_config *cfg, uint64_t seed, int rank, int world,
                               const void *nccl_id, vx_model **out) {
    if (!cfg || !out || world < 1 || rank < 0 || rank >= world || (world > 1 && !nccl_id) || cfg->n_heads <= 0 ||
        cfg->n_embd % cfg->n_heads)
        return VX_ERR_PARAM;
    int dev = vxc_device_current();
    if (dev < 0 || vxc_device_init(dev) != 0) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return VX_ERR_UNSUPPORTED;
    }
    vxc_tp *tp = NULL;
    if (nccl_id) {
        int rc = vxc_tp_create(nccl_id, rank, world, &tp);
        if (rc) {
            fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
            return rc == -4 ? VX_ERR_PARAM : VX_ERR_UNSUPPORTED;
        }
    }
    vxc_net_config nc;
    memset(&nc, 0, sizeof nc);
    nc.n_layers = cfg->n_layers;
    nc.n_heads = cfg->n_heads;
    nc.n_kv_heads = cfg->n_kv_heads;
    nc.n_embd = cfg->n_embd;
    nc.n_head_dim = cfg->n_embd / cfg->n_heads;
    nc.n_ff = cfg->n_ff;
    nc.n_vocab = cfg->n_vocab;
    nc.rope_theta = cfg->rope_theta;
    nc.max_pos = 16384;
    vxc_net *net = NULL;
    int rc = vxc_net_create_synth(&nc, cfg->wtype, seed, tp, &net);
    if (rc) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        vxc_tp_destroy(tp);
        return rc == -3 ? VX_ERR_MEMORY : (vx_error)rc;
    }
    vx_error e = wrap_net(net, tp, dev, &nc, out);
    if (e != VX_OK) vxc_tp_destroy(tp);
    return e;
}

void vx_model_destroy(vx_model *model) {
    if (!model) return;
    vxb_model *m = vxb_of(model);
    vxc_seqs_destroy(m->seqs);
    vxc_net_destroy(m->net);
    vxc_tp_destroy(m->tp);
    free(m);
}

/* Create (or re-create after an n_ctx change) the one-sequence cache. */
static vx_error ensure_seqs(vxb_model *m) {
    int ctx = m->pub.config.n_ctx > 0 ? m->pub.config.n_ctx : 4096;
    if (m->seqs && m->seqs_ctx == ctx) return VX_OK;
    vxc_seqs_destroy(m->seqs);
    m->seqs = NULL;
    vxc_net_config nc;
    vxc_net_config_get(m->net, &nc);
    if (ctx > nc.max_pos) return VX_ERR_PARAM;
    if (vxc_seqs_create(m->net, 1, ctx, VXB_CHUNK_ROWS, &m->seqs) != 0) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return VX_ERR_MEMORY;
    }
    m->seqs_ctx = ctx;
    m->pub.cache_len = 0;
    return VX_OK;
}

vx_error vx_model_forward(vx_model *model, const int *tokens, int n_tokens, float *logits) {
    if (!model || !tokens || !logits) return VX_ERR_PARAM;
    if (model->config.n_embd <= 0 || model->config.n_embd > 8192 || n_tokens <= 0) return VX_ERR_PARAM;
    if (g_level != VX_COMPUTE_EXACT) return VX_ERR_UNSUPPORTED;
    vxb_model *m = vxb_of(model);
    int keep = model->cache_len;
    vx_error e = ensure_seqs(m);
    if (e) return e;
    model->cache_len = keep;
    if (model->cache_len < 0) model->cache_len = 0;
    if ((long long)model->cache_len + n_tokens > m->seqs_ctx) return VX_ERR_PARAM;
    if (vxc_device_current() != m->device) vxc_device_init(m->device);
    double t0 = g_timing ? now_us() : 0.0;
    int rc = vxc_forward_host(m->seqs, 0, model->cache_len, tokens, n_tokens, logits);
    if (g_timing) { g_fwd_us += now_us() - t0; g_fwd_calls++; g_fwd_tokens += n_tokens; }
    if (rc) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return rc == -4 ? VX_ERR_PARAM : VX_ERR_MEMORY;
    }
    model->cache_len += n_tokens;
    return VX_OK;
}

int vx_model_generate_greedy(vx_model *model, const int *prompt, int n_prompt, int *out, int max_tokens,
                             int eos_id) {
    if (!model || !prompt || n_prompt <= 0 || !out || max_tokens <= 0) return VX_ERR_PARAM;
    if (g_level != VX_COMPUTE_EXACT) return VX_ERR_UNSUPPORTED;
    vxb_model *m = vxb_of(model);
    int keep = model->cache_len;
    vx_error e = ensure_seqs(m);
    if (e) return e;
    model->cache_len = keep < 0 ? 0 : keep;
    if ((long long)model->cache_len + n_prompt + max_tokens > m->seqs_ctx) return VX_ERR_PARAM;
    if (vxc_device_current() != m->device) vxc_device_init(m->device);
    int n = 0, pos = 0;
    double t0 = g_timing ? now_us() : 0.0;
    int rc = vxc_greedy_generate(m->seqs, 0, model->cache_len, prompt, n_prompt, out, max_tokens, eos_id, &n, &pos);
    if (g_timing) { g_fwd_us += now_us() - t0; g_fwd_calls++; g_fwd_tokens += n_prompt + n; }
    if (rc) {
        fprintf(stderr, "veltrix-b200: %s\n", vxc_error_string());
        return rc == -4 ? VX_ERR_PARAM : VX_ERR_MEMORY;
    }
    model->cache_len = pos;
    return n;
}

void vx_model_kv_truncate(vx_model *model, int length) {   /* src/model.c:384-389 */
    if (!model) return;
    if (length < 0) length = 0;
    if (length <= model->cache_len) model->cache_len = length;
}

void vx_set_compute_level(vx_compute_level level) { g_level = level; }
void vx_enable_metalearn(bool enable) { (void)enable; }   /* never used by the forward pass */
void vx_set_n_threads(int n) {                              /* host threads: unused by the device path */
    if (n < 1) n = 1;
    if (n > 128) n = 128;
    g_threads = n;
}

void vx_set_forward_timing_enabled(int enabled) {
    g_timing = enabled ? 1 : 0;
    g_fwd_us = 0.0;
    g_fwd_calls = g_fwd_tokens = 0;
}

void vx_print_forward_timing(void) {
    if (!g_timing) return;
    fprintf(stderr, "[timing] device forward=%.1fms calls=%ld tokens=%ld\n", g_fwd_us / 1000.0, g_fwd_calls,
            g_fwd_tokens);
}
