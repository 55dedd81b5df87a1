/*
 * vxh_gguf.c — GGUF v3 reader: maps the file read-only and records tensor
 * pointers into the mapping, so a 39 GB checkpoint is never copied on the
 * host (the reference reads the whole file, copies every tensor and then
 * consolidates them again: src/gguf.c:495-503, src/model.c:54-72).
 *
 * Format rules followed (reference src/gguf.c): header magic/version/counts
 * (:31-44); KV value encoding (:46-100); tensor infos (:112-211); the data
 * section starts at the next 32-byte boundary after the infos (:213-215) and
 * tensor offsets are relative to it (:231-233).  Hyper-parameters are found
 * by the reference's key-substring scan with its quirk that a missing key
 * moves the scan cursor to the end of the KV section (:293-356, :524-533).
 */
#define _GNU_SOURCE
#include "vxh_gguf.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "veltrix.h"

static int skip_val(const uint8_t *p, size_t n, uint64_t *o, uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: *o += 1; break;
        case 2: case 3: *o += 2; break;
        case 4: case 5: case 6: *o += 4; break;
        case 10: case 11: case 12: *o += 8; break;
        case 8: {
            uint64_t l;
            if (*o + 8 > n) return -1;
            memcpy(&l, p + *o, 8);
            *o += 8 + l;
            break;
        }
        case 9: {
            uint32_t at;
            uint64_t al;
            if (*o + 12 > n) return -1;
            memcpy(&at, p + *o, 4);
            memcpy(&al, p + *o + 4, 8);
            *o += 12;
            for (uint64_t i = 0; i < al; i++)
                if (skip_val(p, n, o, at)) return -1;
            break;
        }
        default: return -1;
    }
    return *o <= n ? 0 : -1;
}

/* want: 0 = u32/i32, 1 = f32, 2 = string */
static int scan(const vxh_gguf *g, uint64_t *cur, uint64_t nkv, const char *key, int want, void *out, int olen) {
    const uint8_t *p = (const uint8_t *)g->map;
    uint64_t o = *cur;
    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        if (o + 8 > g->size) return -1;
        memcpy(&kl, p + o, 8);
        o += 8;
        if (o + kl + 4 > g->size) return -1;
        char k[160];
        size_t c = kl < sizeof k - 1 ? kl : sizeof k - 1;
        memcpy(k, p + o, c);
        k[c] = 0;
        o += kl;
        uint32_t vt;
        memcpy(&vt, p + o, 4);
        o += 4;
        if (strstr(k, key)) {
            if (want == 0 && (vt == 4 || vt == 5)) { memcpy(out, p + o, 4); return 0; }
            if (want == 1 && vt == 6) { memcpy(out, p + o, 4); return 0; }
            if (want == 2 && vt == 8) {
                uint64_t sl;
                memcpy(&sl, p + o, 8);
                size_t cc = sl < (uint64_t)olen - 1 ? sl : (uint64_t)olen - 1;
                memcpy(out, p + o + 8, cc);
                ((char *)out)[cc] = 0;
                return 0;
            }
        }
        if (skip_val(p, g->size, &o, vt)) return -1;
    }
    *cur = o;
    return -1;
}

static int scan_u32(const vxh_gguf *g, uint64_t *cur, uint64_t nkv, const char *k, int fb) {
    uint32_t v;
    return scan(g, cur, nkv, k, 0, &v, 0) == 0 ? (int)v : fb;
}

int vxh_gguf_open(const char *path, vxh_gguf *g) {
    memset(g, 0, sizeof *g);
    int fd = open(path, O_RDONLY);
    if (fd < 0) return VX_ERR_FILE;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) { close(fd); return VX_ERR_FORMAT; }
    g->size = (size_t)st.st_size;
    g->map = mmap(NULL, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (g->map == MAP_FAILED) { g->map = NULL; return VX_ERR_MEMORY; }
    const uint8_t *p = (const uint8_t *)g->map;
    uint32_t magic;
    uint64_t nt, nkv;
    memcpy(&magic, p, 4);
    if (magic != 0x46554747u) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
    memcpy(&nt, p + 8, 8);
    memcpy(&nkv, p + 16, 8);
    uint64_t o = 24;
    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        uint32_t vt;
        if (o + 8 > g->size) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
        memcpy(&kl, p + o, 8);
        o += 8 + kl;
        if (o + 4 > g->size) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
        memcpy(&vt, p + o, 4);
        o += 4;
        if (skip_val(p, g->size, &o, vt)) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
    }
    if (nt > 1000000) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
    g->n_tensors = (int)nt;
    g->t = (vxh_tensor *)calloc(nt ? nt : 1, sizeof(vxh_tensor));
    uint64_t *offs = (uint64_t *)calloc(nt ? nt : 1, sizeof(uint64_t));
    for (uint64_t i = 0; i < nt; i++) {
        uint64_t nl;
        uint32_t nd, ty;
        if (o + 8 > g->size) goto bad;
        memcpy(&nl, p + o, 8);
        o += 8;
        if (o + nl + 4 > g->size) goto bad;
        size_t c = nl < sizeof g->t[i].name - 1 ? nl : sizeof g->t[i].name - 1;
        memcpy(g->t[i].name, p + o, c);
        o += nl;
        memcpy(&nd, p + o, 4);
        o += 4;
        if (nd > 4 || o + 8ull * nd + 12 > g->size) goto bad;
        g->t[i].n_dims = (int)nd;
        for (int d = 0; d < 4; d++) g->t[i].ne[d] = 1;
        for (uint32_t d = 0; d < nd; d++) { memcpy(&g->t[i].ne[d], p + o, 8); o += 8; }
        memcpy(&ty, p + o, 4);
        o += 4;
        memcpy(&offs[i], p + o, 8);
        o += 8;
        g->t[i].type = (int)ty;
    }
    {
        uint64_t data0 = o + (32 - o % 32) % 32;
        for (uint64_t i = 0; i < nt; i++) {
            if (data0 + offs[i] > g->size) goto bad;
            g->t[i].data = p + data0 + offs[i];
        }
    }
    free(offs);
    {
        uint64_t cur = 24;
        g->n_layers = scan_u32(g, &cur, nkv, "block_count", 32);
        g->n_heads = scan_u32(g, &cur, nkv, "head_count", 32);
        g->n_kv_heads = scan_u32(g, &cur, nkv, "head_count_kv", g->n_heads);
        g->n_embd = scan_u32(g, &cur, nkv, "embedding_length", 4096);
        g->n_ff = scan_u32(g, &cur, nkv, "feedforward_length", 0);
        g->n_vocab = scan_u32(g, &cur, nkv, "vocab_size", 0);
        if (g->n_vocab == 0) g->n_vocab = scan_u32(g, &cur, nkv, "vocabulary.vocab_size", 0);
        float th;
        g->rope_theta = scan(g, &cur, nkv, "rope.freq_base", 1, &th, 0) == 0 ? th : 10000.0f;
        if (scan(g, &cur, nkv, "general.architecture", 2, g->arch, sizeof g->arch) != 0) g->arch[0] = 0;
    }
    madvise(g->map, g->size, MADV_SEQUENTIAL);
    return VX_OK;
bad:
    free(offs);
    vxh_gguf_close(g);
    return VX_ERR_FORMAT;
}

void vxh_gguf_close(vxh_gguf *g) {
    if (g->map) munmap(g->map, g->size);
    free(g->t);
    memset(g, 0, sizeof *g);
}

const vxh_tensor *vxh_gguf_find(const vxh_gguf *g, const char *name) {
    for (int i = 0; i < g->n_tensors; i++)
        if (strcmp(g->t[i].name, name) == 0) return &g->t[i];
    return NULL;
}
