// vxc_tp.cu — tensor parallelism for the 70B-shaped target (one process per
// GPU, NCCL over NVLink): the communicator and the two exchanges a forward
// needs (sum of the row-split projections' outputs, gather of the
// vocabulary-split logits).  The kernels around them stay per GPU.
#include "vxc_common.cuh"
#include "vxc_internal.h"

#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

static_assert(sizeof(ncclUniqueId) == VXC_TP_ID_BYTES, "NCCL unique id size");

// NCCL is opened at run time, so the library loads (and serves one GPU)
// without it; a process that already holds libnccl (torch) shares that copy.
namespace {
struct Nccl {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

Nccl load_nccl() {
    Nccl n;
    // connect every channel at communicator creation, not lazily at a first
    // collective that may sit inside a CUDA-graph capture (kept if the caller set it)
    setenv("NCCL_RUNTIME_CONNECT", "0", 0);
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return n;
    n.get_unique_id = (decltype(n.get_unique_id))dlsym(h, "ncclGetUniqueId");
    n.comm_init_rank = (decltype(n.comm_init_rank))dlsym(h, "ncclCommInitRank");
    n.comm_destroy = (decltype(n.comm_destroy))dlsym(h, "ncclCommDestroy");
    n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
    n.all_gather = (decltype(n.all_gather))dlsym(h, "ncclAllGather");
    n.error_string = (decltype(n.error_string))dlsym(h, "ncclGetErrorString");
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.all_gather && n.error_string;
    return n;
}

// The library, opened once (thread-safe static initialisation); NULL with the
// error set when it is missing or incomplete.
const Nccl *nccl() {
    static const Nccl n = load_nccl();
    if (!n.ok) vxc_set_error("tensor parallelism needs libnccl.so.2 with the collectives it uses");
    return n.ok ? &n : NULL;
}
}  // namespace

struct vxc_tp {
    ncclComm_t comm;
    int rank, world;
};

extern "C" int vxc_tp_unique_id(void *id_out) {
    if (!id_out) { vxc_set_error("vxc_tp_unique_id: NULL buffer"); return -4; }
    const Nccl *N = nccl();
    if (!N) return -7;
    ncclUniqueId id;
    ncclResult_t r = N->get_unique_id(&id);
    if (r != ncclSuccess) { vxc_set_error("ncclGetUniqueId: %s", N->error_string(r)); return -3; }
    memcpy(id_out, &id, sizeof id);
    return 0;
}

extern "C" int vxc_tp_create(const void *id, int rank, int world, vxc_tp **out) {
    if (!id || !out || world < 1 || rank < 0 || rank >= world) {
        vxc_set_error("vxc_tp_create: bad arguments");
        return -4;
    }
    int rc = vxc_require_device();
    if (rc) return rc;
    const Nccl *N = nccl();
    if (!N) return -7;
    vxc_tp *t = (vxc_tp *)calloc(1, sizeof(vxc_tp));
    if (!t) { vxc_set_error("vxc_tp_create: out of host memory"); return -3; }
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclResult_t r = N->comm_init_rank(&t->comm, world, uid, rank);
    if (r != ncclSuccess) {
        vxc_set_error("ncclCommInitRank: %s", N->error_string(r));
        free(t);
        return -3;
    }
    // one all-reduce and one all-gather now, outside any stream capture, so
    // that the connections they use exist before a forward is captured
    float *buf = NULL;
    cudaError_t ce = cudaMalloc((void **)&buf, 2 * 1024 * sizeof(float) * (size_t)world);
    if (ce == cudaSuccess) ce = cudaMemset(buf, 0, 2 * 1024 * sizeof(float) * (size_t)world);
    if (ce == cudaSuccess) {
        r = N->all_reduce(buf, buf, 1024, ncclFloat32, ncclSum, t->comm, 0);
        if (r == ncclSuccess) r = N->all_gather(buf, buf + 1024, 1024, ncclFloat32, t->comm, 0);
        ce = cudaStreamSynchronize(0);
    }
    if (buf) cudaFree(buf);
    if (ce != cudaSuccess || r != ncclSuccess) {
        vxc_set_error("vxc_tp_create: warm-up exchange failed: %s",
                      ce != cudaSuccess ? cudaGetErrorString(ce) : N->error_string(r));
        N->comm_destroy(t->comm);
        free(t);
        return -3;
    }
    t->rank = rank;
    t->world = world;
    *out = t;
    return 0;
}

extern "C" void vxc_tp_destroy(vxc_tp *t) {
    if (!t) return;
    const Nccl *N = nccl();
    if (N) N->comm_destroy(t->comm);
    free(t);
}

int vxc_tp_rank(const vxc_tp *t) { return t ? t->rank : 0; }
int vxc_tp_world(const vxc_tp *t) { return t ? t->world : 1; }

int vxc_tp_allreduce_sum(const vxc_tp *t, float *buf, size_t n, cudaStream_t st) {
    const Nccl *N = nccl();
    ncclResult_t r = N->all_reduce(buf, buf, n, ncclFloat32, ncclSum, t->comm, st);
    if (r != ncclSuccess) { vxc_set_error("ncclAllReduce: %s", N->error_string(r)); return -3; }
    return 0;
}

int vxc_tp_allgather(const vxc_tp *t, const float *send, float *recv, size_t n, cudaStream_t st) {
    const Nccl *N = nccl();
    ncclResult_t r = N->all_gather(send, recv, n, ncclFloat32, t->comm, st);
    if (r != ncclSuccess) { vxc_set_error("ncclAllGather: %s", N->error_string(r)); return -3; }
    return 0;
}
