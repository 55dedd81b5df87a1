/* vxh_model.h — private layout of a model handle of the B200 back end. */
#ifndef VXH_MODEL_H
#define VXH_MODEL_H

#include "veltrix.h"
#include "veltrix_cuda.h"

/* The public struct comes first so a vx_model* is also a vxb_model*. */
typedef struct {
    vx_model pub;
    vxc_net *net;
    vxc_tp *tp;       /* communicator of a tensor-parallel model (owned), else NULL */
    vxc_seqs *seqs;   /* one-sequence KV cache of the drop-in API, created at the first forward */
    int seqs_ctx;     /* n_ctx the cache was created with */
    int device;
} vxb_model;

static inline vxb_model *vxb_of(vx_model *m) { return (vxb_model *)m; }

/* Rows processed per device forward call by the one-sequence API. */
#define VXB_CHUNK_ROWS 64

#endif
