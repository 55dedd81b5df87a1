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
 *
 * A file that is truncated or whose lengths and offsets point outside it is
 * rejected with VX_ERR_FORMAT before any byte past its end is touched, as the
 * reference rejects a tensor whose bytes run past the end of the file
 * (:257-275; tensor sizes as src/quantize.c:59-85 computes them).  Every
 * length is compared against the bytes left rather than added to an offset
 * first, so no crafted length can wrap the arithmetic, and array values may
 * nest at most VXH_GGUF_MAX_NEST deep.
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

#define VXH_GGUF_MAX_NEST 8

/* Skip one value of GGUF type t at *o; -1 if it does not fit in n bytes. */
static int skip_val(const uint8_t *p, size_t n, uint64_t *o, uint32_t t, int depth) {
    uint64_t w = 0;
    switch (t) {
        case 0: case 1: case 7: w = 1; break;
        case 2: case 3: w = 2; break;
        case 4: case 5: case 6: w = 4; break;
        case 10: case 11: case 12: w = 8; break;
        case 8: {
            uint64_t l;
            if (*o > n || n - *o < 8) return -1;
            memcpy(&l, p + *o, 8);
            *o += 8;
            w = l;
            break;
        }
        case 9: {
            uint32_t at;
            uint64_t al;
            if (depth >= VXH_GGUF_MAX_NEST || *o > n || n - *o < 12) return -1;
            memcpy(&at, p + *o, 4);
            memcpy(&al, p + *o + 4, 8);
            *o += 12;
            for (uint64_t i = 0; i < al; i++)
                if (skip_val(p, n, o, at, depth + 1)) return -1;
            return 0;
        }
        default: return -1;
    }
    if (*o > n || w > n - *o) return -1;
    *o += w;
    return 0;
}

/* want: 0 = u32/i32, 1 = f32, 2 = string */
static int scan(const vxh_gguf *g, uint64_t *cur, uint64_t nkv, const char *key, int want, void *out, int olen) {
    const uint8_t *p = (const uint8_t *)g->map;
    const uint64_t n = g->size;
    uint64_t o = *cur;
    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        if (o > n || n - o < 8) return -1;
        memcpy(&kl, p + o, 8);
        o += 8;
        if (kl > n - o || n - o - kl < 4) return -1;
        char k[160];
        size_t c = kl < sizeof k - 1 ? kl : sizeof k - 1;
        memcpy(k, p + o, c);
        k[c] = 0;
        o += kl;
        uint32_t vt;
        memcpy(&vt, p + o, 4);
        o += 4;
        if (strstr(k, key)) {
            if (want == 0 && (vt == 4 || vt == 5) && n - o >= 4) { memcpy(out, p + o, 4); return 0; }
            if (want == 1 && vt == 6 && n - o >= 4) { memcpy(out, p + o, 4); return 0; }
            if (want == 2 && vt == 8 && n - o >= 8) {
                uint64_t sl;
                memcpy(&sl, p + o, 8);
                if (sl <= n - o - 8) {
                    size_t cc = sl < (uint64_t)olen - 1 ? sl : (uint64_t)olen - 1;
                    memcpy(out, p + o + 8, cc);
                    ((char *)out)[cc] = 0;
                    return 0;
                }
            }
        }
        if (skip_val(p, n, &o, vt, 0)) return -1;
    }
    *cur = o;
    return -1;
}

static int scan_u32(const vxh_gguf *g, uint64_t *cur, uint64_t nkv, const char *k, int fb) {
    uint32_t v;
    return scan(g, cur, nkv, k, 0, &v, 0) == 0 ? (int)v : fb;
}

/* Largest dimension accepted in a tensor info. */
#define VXH_GGUF_MAX_DIM (1ll << 32)

/* Bytes of `elems` elements of GGML type `ty` stored as whole blocks, as the
 * reference computes a tensor's size (src/quantize.c:59-85: blocks rounded
 * up; block bytes of include/quantize.h).  0 for a type whose block size is
 * not known here: such a tensor is refused later by the device upload, so
 * only its start offset is checked. */
static uint64_t tensor_bytes(uint32_t ty, uint64_t elems) {
    uint64_t per = 0, blk = 1;
    switch (ty) {
        case 0: per = 4; break;                  /* F32 */
        case 1: case 30: per = 2; break;         /* F16, BF16 */
        case 2: per = 18; blk = 32; break;       /* Q4_0 */
        case 3: per = 20; blk = 32; break;       /* Q4_1 */
        case 6: per = 22; blk = 32; break;       /* Q5_0 */
        case 7: per = 24; blk = 32; break;       /* Q5_1 */
        case 8: per = 34; blk = 32; break;       /* Q8_0 */
        case 10: per = 84; blk = 256; break;     /* Q2_K */
        case 11: per = 110; blk = 256; break;    /* Q3_K */
        case 12: per = 144; blk = 256; break;    /* Q4_K */
        case 13: per = 176; blk = 256; break;    /* Q5_K */
        case 14: per = 210; blk = 256; break;    /* Q6_K */
        case 15: per = 292; blk = 256; break;    /* Q8_K */
        default: return 0;
    }
    const uint64_t nb = elems / blk + (elems % blk != 0);
    return nb > UINT64_MAX / per ? UINT64_MAX : nb * per;
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
    const uint64_t n = g->size;
    for (uint64_t i = 0; i < nkv; i++) {
        uint64_t kl;
        uint32_t vt;
        if (n - o < 8) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
        memcpy(&kl, p + o, 8);
        o += 8;
        if (kl > n - o || n - o - kl < 4) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
        o += kl;
        memcpy(&vt, p + o, 4);
        o += 4;
        if (skip_val(p, n, &o, vt, 0)) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
    }
    if (nt > 1000000) { vxh_gguf_close(g); return VX_ERR_FORMAT; }
    g->n_tensors = (int)nt;
    g->t = (vxh_tensor *)calloc(nt ? nt : 1, sizeof(vxh_tensor));
    uint64_t *offs = (uint64_t *)calloc(nt ? nt : 1, sizeof(uint64_t));
    if (!g->t || !offs) {
        free(offs);
        vxh_gguf_close(g);
        return VX_ERR_MEMORY;
    }
    for (uint64_t i = 0; i < nt; i++) {
        uint64_t nl;
        uint32_t nd, ty;
        if (n - o < 8) goto bad;
        memcpy(&nl, p + o, 8);
        o += 8;
        if (nl > n - o || n - o - nl < 4) goto bad;
        size_t c = nl < sizeof g->t[i].name - 1 ? nl : sizeof g->t[i].name - 1;
        memcpy(g->t[i].name, p + o, c);
        o += nl;
        memcpy(&nd, p + o, 4);
        o += 4;
        if (nd > 4 || n - o < 8ull * nd + 12) goto bad;
        g->t[i].n_dims = (int)nd;
        for (int d = 0; d < 4; d++) g->t[i].ne[d] = 1;
        for (uint32_t d = 0; d < nd; d++) {
            memcpy(&g->t[i].ne[d], p + o, 8);
            o += 8;
            if (g->t[i].ne[d] < 0 || g->t[i].ne[d] > VXH_GGUF_MAX_DIM) goto bad;
        }
        memcpy(&ty, p + o, 4);
        o += 4;
        memcpy(&offs[i], p + o, 8);
        o += 8;
        g->t[i].type = (int)ty;
    }
    {
        const uint64_t data0 = o + (32 - o % 32) % 32;
        if (nt && data0 > n) goto bad;   /* only a file without tensors may end before it */
        for (uint64_t i = 0; i < nt; i++) {
            const vxh_tensor *t = &g->t[i];
            if (offs[i] > n - data0) goto bad;
            /* the tensor's own bytes must lie inside the file too
             * (src/gguf.c:257-275); an element count that overflows 64 bits
             * cannot fit in any file */
            uint64_t elems = 1;
            int over = 0;
            for (int d = 0; d < 4; d++) {
                const uint64_t e = (uint64_t)t->ne[d];
                if (e && elems > UINT64_MAX / e) over = 1;
                elems *= e;
            }
            const uint64_t bytes = over ? UINT64_MAX : tensor_bytes((uint32_t)t->type, elems);
            if (bytes > n - data0 - offs[i]) {
                fprintf(stderr, "veltrix-b200: GGUF tensor %s (%llu bytes at offset %llu) runs past the end of the "
                        "file (%zu bytes)\n", t->name, (unsigned long long)bytes,
                        (unsigned long long)(data0 + offs[i]), g->size);
                goto bad;
            }
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
