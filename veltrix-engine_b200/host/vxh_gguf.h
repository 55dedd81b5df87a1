/* vxh_gguf.h — GGUF reader of the host library (mmap, no copies). */
#ifndef VXH_GGUF_H
#define VXH_GGUF_H

#include <stddef.h>
#include <stdint.h>

typedef struct {
    char name[128];
    int type;            /* GGML type: 0 F32, 2 Q4_0, 8 Q8_0, ... */
    int n_dims;
    int64_t ne[4];
    const uint8_t *data; /* into the mapping */
} vxh_tensor;

typedef struct {
    void *map;
    size_t size;
    int n_tensors;
    vxh_tensor *t;
    /* hyper-parameters, scanned as the reference does (src/gguf.c:524-533) */
    int n_layers, n_heads, n_kv_heads, n_embd, n_ff, n_vocab;
    float rope_theta;
    char arch[64];
} vxh_gguf;

/* 0 on success, vx_error code otherwise. */
int vxh_gguf_open(const char *path, vxh_gguf *g);
void vxh_gguf_close(vxh_gguf *g);
const vxh_tensor *vxh_gguf_find(const vxh_gguf *g, const char *name);

#endif
