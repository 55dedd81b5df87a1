// vxc_spec.cu — sampling, fused acceptance and the device-resident
// speculative-decoding round loop.
//
// Semantics (the corrected form of reference src/speculative.c:148-294; the
// CPU oracle oracle/vxo_spec.c restates the same procedure):
//   round, for every active sequence with committed tokens c[0..L):
//     draft step 0   rows (c[L-2], c[L-1]) at positions L-2, L-1 -> q_0
//     draft step i   row d_i at position L+i-1 -> q_i            (i = 1..k-1)
//     d_{i+1}        sampled from q_i with Philox (pos L+i, DRAFT)
//     verify         rows (c[L-1], d_1..d_k) at positions L-1..L+k-1 -> p_0..p_k
//     accept         first rejection i: sample max(0, p_i - q_i); all accepted:
//                    bonus from p_k                (fused kernel k_accept)
//     commit         c += d_1..d_a, next ; L += a + 1
// KV invariants: target holds 0..L-2 at round start (the verify rewrites
// L-1..); draft holds 0..L-3 (step 0 rewrites L-2, L-1).  Positions past a
// rejection hold stale K/V that the next round overwrites before reading.
// All sampling decisions use exact integer weights (vxc_weight), so they match
// the oracle bit-for-bit given the same logits.
#include "vxc_common.cuh"
#include "vxc_internal.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

typedef unsigned long long u64;
typedef unsigned __int128 u128;

#define SMP_THREADS 1024

// ---------------------------------------------------------------------------
// block-wide helpers (blockDim.x a multiple of 32, at most 1024)
// ---------------------------------------------------------------------------
struct MaxIdx {
    float v;
    int i;
};

__device__ __forceinline__ MaxIdx better(MaxIdx a, MaxIdx b) {
    // larger value wins; on ties the lower index (first maximum)
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

// f(v, x) for every element v of a row, x = row[v].  Rows of 16-byte aligned
// start and V % 4 == 0 are read as float4 with RP_UNROLL loads in flight per
// thread (one memory latency per RP_UNROLL * 4 * blockDim.x elements, not one
// per element); other rows element by element.  Visiting order differs per
// thread, so f must be order-independent (integer sums, first-max argmax).
#define RP_UNROLL 8
template <class F>
__device__ __forceinline__ void row_pass(const float *__restrict__ row, int V, F f) {
    const int nt = blockDim.x;
    if ((((uintptr_t)row) & 15) == 0 && (V & 3) == 0) {
        const int V4 = V >> 2;
        const float4 *r4 = reinterpret_cast<const float4 *>(row);
        for (int base = 0; base < V4; base += nt * RP_UNROLL) {
            float4 x[RP_UNROLL];
#pragma unroll
            for (int u = 0; u < RP_UNROLL; u++) {
                const int j = base + u * nt + (int)threadIdx.x;
                x[u] = j < V4 ? __ldg(r4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < RP_UNROLL; u++) {
                const int j = base + u * nt + (int)threadIdx.x;
                if (j < V4) {
                    f(4 * j, x[u].x);
                    f(4 * j + 1, x[u].y);
                    f(4 * j + 2, x[u].z);
                    f(4 * j + 3, x[u].w);
                }
            }
        }
    } else {
        for (int v = threadIdx.x; v < V; v += nt) f(v, row[v]);
    }
}

__device__ MaxIdx block_argmax(const float *__restrict__ row, int V, MaxIdx *red) {
    MaxIdx m = {-INFINITY, 0x7fffffff};
    row_pass(row, V, [&](int v, float x) { m = better(m, MaxIdx{x, v}); });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        MaxIdx t;
        t.v = __shfl_xor_sync(0xffffffffu, m.v, o);
        t.i = __shfl_xor_sync(0xffffffffu, m.i, o);
        m = better(m, t);
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = m;
    __syncthreads();
    MaxIdx r = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) r = better(r, red[i]);
    __syncthreads();
    return r;
}

__device__ u64 block_sum_u64(u64 v, u64 *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    u64 r = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) r += red[i];
    __syncthreads();
    return r;
}

// Exclusive prefix of per-thread values in thread order.
__device__ u64 block_excl_scan_u64(u64 v, u64 *red) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    u64 inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        u64 t = __shfl_up_sync(0xffffffffu, inc, o);
        if (l >= o) inc += t;
    }
    __syncthreads();
    if (l == 31) red[w] = inc;
    __syncthreads();
    u64 base = 0;
    for (int i = 0; i < w; i++) base += red[i];
    __syncthreads();
    return base + inc - v;
}

// Chunked search: thread t owns elements [t*C, (t+1)*C).  Returns the first
// v with inclusive prefix sum of wt(v) > thr (or V-1 if none).
template <class WF>
__device__ int block_draw(int V, u64 thr, WF wt, u64 *red, int *res) {
    const int C = (V + blockDim.x - 1) / blockDim.x;
    const int a = threadIdx.x * C, b = min(V, a + C);
    u64 s = 0;
    for (int v = a; v < b; v++) s += wt(v);
    u64 ex = block_excl_scan_u64(s, red);
    if (threadIdx.x == 0) *res = V - 1;
    __syncthreads();
    if (a < b && ex <= thr && thr < ex + s) {
        u64 acc = ex;
        for (int v = a; v < b; v++) {
            acc += wt(v);
            if (acc > thr) { *res = v; break; }
        }
    }
    __syncthreads();
    int r = *res;
    __syncthreads();
    return r;
}

__device__ __forceinline__ u64 draw_threshold(u64 S, uint32_t word) {
    return (u64)(((u128)S * (word >> 8)) >> 24);
}

// ---------------------------------------------------------------------------
// per-row sampler
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(SMP_THREADS) k_sample_rows(const float *__restrict__ logits, int V, float temp,
                                                             u64 seed, const int *__restrict__ pos,
                                                             const int *__restrict__ seq, unsigned purpose,
                                                             int *__restrict__ out) {
    __shared__ MaxIdx red_m[32];
    __shared__ u64 red_u[32];
    __shared__ int res;
    const int r = blockIdx.x;
    const float *row = logits + (size_t)r * V;
    MaxIdx mx = block_argmax(row, V, red_m);
    if (!(temp > 0.0f)) {
        if (threadIdx.x == 0) out[r] = mx.i;
        return;
    }
    const float invT = 1.0f / temp;
    auto wt = [&](int v) -> u64 { return vxc_weight(row[v], mx.v, invT); };
    u64 s = 0;
    row_pass(row, V, [&](int, float x) { s += vxc_weight(x, mx.v, invT); });
    u64 S = block_sum_u64(s, red_u);
    uint32_t word = vxc_philox_u32(seed, (uint32_t)pos[r], (uint32_t)seq[r], purpose);
    int t = block_draw(V, draw_threshold(S, word), wt, red_u, &res);
    if (threadIdx.x == 0) out[r] = t;
}

extern "C" int vxc_sample_rows(const float *logits, int n_rows, int V, float temp, uint64_t seed, const int *d_pos,
                               const int *d_seq, unsigned int purpose, int *d_tokens, void *stream) {
    if (!logits || n_rows <= 0 || V <= 0 || !d_pos || !d_seq || !d_tokens) {
        vxc_set_error("vxc_sample_rows: bad arguments");
        return -4;
    }
    (k_sample_rows<<<n_rows, SMP_THREADS, 0, (cudaStream_t)stream>>>(logits, V, temp, seed, d_pos, d_seq, purpose,
                                                                    d_tokens), vxc_count_launches(1));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { vxc_set_error("vxc_sample_rows: %s", cudaGetErrorString(e)); return -3; }
    return 0;
}

// ---------------------------------------------------------------------------
// fused acceptance
// ---------------------------------------------------------------------------
struct AccStat {
    float maxp, maxq;
    int argp, pad;
    u64 Sp, Sq, Wpd, Wqd;
};

#define ACC_THREADS 256   // 64 x 6 CTAs of 256 threads (<= 64 registers): one wave at 4 CTAs per SM

__global__ void __launch_bounds__(ACC_THREADS, 4) k_accept(const float *__restrict__ P, long long p_seq, long long p_pos,
                                                        const float *__restrict__ Q, long long q_seq, long long q_pos,
                                                        const int *__restrict__ d, int k, int V, float temp, u64 seed,
                                                        const int *__restrict__ seq_id, const int *__restrict__ pos0,
                                                        int *__restrict__ n_acc, int *__restrict__ next,
                                                        AccStat *st, unsigned int *__restrict__ cnt) {
    __shared__ MaxIdx red_m[32];
    __shared__ u64 red_u[32];
    __shared__ int res;
    __shared__ int is_last;
    const int s = blockIdx.x, i = blockIdx.y;
    const bool greedy = !(temp > 0.0f);
    const float invT = greedy ? 0.0f : 1.0f / temp;
    // ---- phase 1: statistics of row i ----
    {
        const float *pr = P + s * p_seq + i * p_pos;
        MaxIdx mp = block_argmax(pr, V, red_m);
        AccStat a;
        a.maxp = mp.v;
        a.argp = mp.i;
        a.maxq = 0.0f;
        a.Sp = a.Sq = a.Wpd = a.Wqd = 0;
        if (!greedy) {
            u64 sp = 0;
            row_pass(pr, V, [&](int, float x) { sp += vxc_weight(x, mp.v, invT); });
            a.Sp = block_sum_u64(sp, red_u);
            if (i < k) {
                const float *qr = Q + s * q_seq + i * q_pos;
                MaxIdx mq = block_argmax(qr, V, red_m);
                a.maxq = mq.v;
                u64 sq = 0;
                row_pass(qr, V, [&](int, float x) { sq += vxc_weight(x, mq.v, invT); });
                a.Sq = block_sum_u64(sq, red_u);
                int t = d[s * k + i];
                if (t >= 0 && t < V) {
                    a.Wpd = vxc_weight(pr[t], mp.v, invT);
                    a.Wqd = vxc_weight(qr[t], mq.v, invT);
                }
            }
        }
        if (threadIdx.x == 0) {
            st[s * (k + 1) + i] = a;
            __threadfence();
            unsigned prev = atomicAdd(&cnt[s], 1u);
            is_last = (prev == (unsigned)k);
        }
        __syncthreads();
        if (!is_last) return;
    }
    // ---- phase 2 (last CTA of sequence s): decision and resample ----
    __threadfence();
    if (threadIdx.x == 0) cnt[s] = 0;   // re-arm for the next launch
    // other CTAs wrote these; read them through L2, not a stale L1 line
    const AccStat *S_ = st + s * (k + 1);
    __syncthreads();
    const int p0 = pos0[s], sid = seq_id[s];
    int acc = k, nxt = -1, rej = -1;
    for (int j = 0; j < k; j++) {
        AccStat a = S_[j];
        int t = d[s * k + j];
        bool ok;
        if (greedy) {
            ok = (t == a.argp);
        } else {
            u64 u = vxc_philox_u32(seed, (uint32_t)(p0 + j), (uint32_t)sid, VXC_PURPOSE_ACCEPT) >> 8;
            ok = (t >= 0 && t < V) && ((u128)u * a.Wqd * a.Sp < (((u128)a.Wpd * a.Sq) << 24));
        }
        if (!ok) { acc = j; rej = j; break; }
    }
    if (greedy) {
        nxt = S_[acc].argp;
    } else if (rej >= 0) {
        const AccStat a = S_[rej];
        const float *pr = P + s * p_seq + rej * p_pos;
        const float *qr = Q + s * q_seq + rej * q_pos;
        auto rw = [&](int v) -> u64 {
            u128 x = (u128)vxc_weight(pr[v], a.maxp, invT) * a.Sq;
            u128 y = (u128)vxc_weight(qr[v], a.maxq, invT) * a.Sp;
            return x > y ? (u64)((x - y) >> 36) : 0ull;
        };
        u64 sr = 0;
        for (int v = threadIdx.x; v < V; v += blockDim.x) sr += rw(v);
        u64 SR = block_sum_u64(sr, red_u);
        if (SR == 0) {
            nxt = a.argp;
        } else {
            uint32_t w = vxc_philox_u32(seed, (uint32_t)(p0 + rej), (uint32_t)sid, VXC_PURPOSE_RESAMPLE);
            nxt = block_draw(V, draw_threshold(SR, w), rw, red_u, &res);
        }
    } else {
        const AccStat a = S_[k];
        const float *pr = P + s * p_seq + k * p_pos;
        auto pw = [&](int v) -> u64 { return vxc_weight(pr[v], a.maxp, invT); };
        uint32_t w = vxc_philox_u32(seed, (uint32_t)(p0 + k), (uint32_t)sid, VXC_PURPOSE_RESAMPLE);
        nxt = block_draw(V, draw_threshold(a.Sp, w), pw, red_u, &res);
    }
    if (threadIdx.x == 0) {
        n_acc[s] = acc;
        next[s] = nxt;
    }
}

static size_t accept_ws(int n_seq, int k) {
    size_t a = (size_t)n_seq * (k + 1) * sizeof(AccStat);
    a = (a + 255) & ~(size_t)255;
    return a + (size_t)n_seq * sizeof(unsigned int);
}

extern "C" size_t vxc_accept_workspace_bytes(int n_seq, int k) { return accept_ws(n_seq, k); }

// The counters at the end of the workspace must be zero on the first launch;
// the kernel re-arms them itself.
static int launch_accept(const float *P, long long p_seq, long long p_pos, const float *Q, long long q_seq,
                         long long q_pos, const int *d, int n_seq, int k, int V, float temp, uint64_t seed,
                         const int *seq_id, const int *pos0, int *n_acc, int *next, void *ws, cudaStream_t st) {
    size_t a = ((size_t)n_seq * (k + 1) * sizeof(AccStat) + 255) & ~(size_t)255;
    (k_accept<<<dim3(n_seq, k + 1), ACC_THREADS, 0, st>>>(P, p_seq, p_pos, Q, q_seq, q_pos, d, k, V, temp, seed,
                                                         seq_id, pos0, n_acc, next, (AccStat *)ws,
                                                         (unsigned int *)((char *)ws + a)), vxc_count_launches(1));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { vxc_set_error("vxc_accept: %s", cudaGetErrorString(e)); return -3; }
    return 0;
}

extern "C" int vxc_accept(const float *P, long long p_seq, long long p_pos, const float *Q, long long q_seq,
                          long long q_pos, const int *d, int n_seq, int k, int V, float temp, uint64_t seed,
                          const int *seq_id, const int *pos0, int *n_acc, int *next, void *workspace,
                          size_t workspace_bytes, void *stream) {
    if (!P || !Q || !d || n_seq <= 0 || k <= 0 || V <= 0 || !seq_id || !pos0 || !n_acc || !next) {
        vxc_set_error("vxc_accept: bad arguments");
        return -4;
    }
    if (!workspace || workspace_bytes < accept_ws(n_seq, k)) {
        vxc_set_error("vxc_accept: workspace of %zu bytes needed", accept_ws(n_seq, k));
        return -4;
    }
    return launch_accept(P, p_seq, p_pos, Q, q_seq, q_pos, d, n_seq, k, V, temp, seed, seq_id, pos0, n_acc, next,
                         workspace, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// round-loop kernels
// ---------------------------------------------------------------------------
struct SpecDev {
    int S, k, cap, max_new, max_ctx;
    int *c;          // [S][cap] committed tokens (prompt + generated)
    int *L;          // [S]
    int *gen;        // [S]
    int *done;       // [S]
    int *seq_id;     // [S]
    int *slot;       // [S] = 0..S-1
    int *out;        // [S][max_new]
    int *tok0, *pos0, *lrow0;   // draft step 0: [2S], [S], [S]
    int *dpos;       // [k][S] positions of draft step i rows (i>=1) / sampling positions
    int *dtok;       // [k][S] sampled draft tokens
    int *vtok, *vpos, *vrows;   // verify: [S(k+1)], [S], [S(k+1)]
    int *dseq;       // [S][k] draft tokens seq-major
    int *apos;       // [S] = L (position of d_1)
    int *n_acc, *next;
    long long *ctr;  // [3] drafted, accepted, emitted
    int *n_done;     // [1]
};

__global__ void k_round_prep(SpecDev D) {
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= D.S) return;
    const int L = D.L[s];
    const int *c = D.c + (size_t)s * D.cap;
    if (L >= 2) {
        D.tok0[2 * s] = c[L - 2];
        D.tok0[2 * s + 1] = c[L - 1];
        D.pos0[s] = L - 2;
        D.lrow0[s] = 2 * s + 1;
    } else {
        D.tok0[2 * s] = c[0];
        D.tok0[2 * s + 1] = c[0];
        D.pos0[s] = 0;
        D.lrow0[s] = 2 * s;
    }
    for (int i = 0; i < D.k; i++) D.dpos[i * D.S + s] = L + i;   // sampling position of d_{i+1}
    D.vpos[s] = L - 1;
    D.apos[s] = L;
    D.vtok[s * (D.k + 1)] = c[L - 1];
    for (int j = 0; j <= D.k; j++) D.vrows[s * (D.k + 1) + j] = s * (D.k + 1) + j;
}

// draft step i >= 1 processes d_i at position L+i-1 = dpos[(i-1)][s]
__global__ void k_gather_verify(SpecDev D) {
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= D.S) return;
    for (int i = 0; i < D.k; i++) {
        int t = D.dtok[i * D.S + s];
        D.vtok[s * (D.k + 1) + 1 + i] = t;
        D.dseq[s * D.k + i] = t;
    }
}

__global__ void k_commit(SpecDev D) {
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= D.S) return;
    if (D.done[s]) return;
    const int a = D.n_acc[s], nx = D.next[s];
    const int L = D.L[s];
    int *c = D.c + (size_t)s * D.cap;
    int g = D.gen[s];
    int emitted = 0;
    for (int i = 0; i <= a; i++) {
        int t = i < a ? D.dseq[s * D.k + i] : nx;
        c[L + i] = t;
        if (g < D.max_new) {
            D.out[(size_t)s * D.max_new + g] = t;
            g++;
            emitted++;
        }
    }
    D.L[s] = L + a + 1;
    D.gen[s] = g;
    atomicAdd((unsigned long long *)&D.ctr[0], (unsigned long long)D.k);
    atomicAdd((unsigned long long *)&D.ctr[1], (unsigned long long)a);
    atomicAdd((unsigned long long *)&D.ctr[2], (unsigned long long)emitted);
    if (g >= D.max_new || L + a + 1 + D.k + 1 > D.max_ctx) {
        D.done[s] = 1;
        atomicAdd(D.n_done, 1);
    }
}

// ---------------------------------------------------------------------------
// engine
// ---------------------------------------------------------------------------
struct vxc_spec {
    const vxc_net *tnet, *dnet;
    vxc_seqs *ts, *ds;
    int S, k, max_ctx, V, cap_alloc;
    SpecDev D;
    float *dlog;       // [k][S][V]
    float *vlog;       // [S][k+1][V]
    void *acc_ws;
    int *prefill_meta; // per prompt chunk: sequence slot, first position
    int prefill_cap;   // ints in prefill_meta
    cudaStream_t st;
    cudaStream_t st2;  // the draft's prompt pass runs here, beside the target's
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    int *h_ndone;      // pinned
};

extern "C" int vxc_spec_create(const vxc_net *target, const vxc_net *draft, int n_seq, int k, int max_ctx,
                               vxc_spec **out) {
    int rc = vxc_require_device();
    if (rc) return rc;
    vxc_net_config tc, dc;
    if (!target || !draft || !out || n_seq <= 0 || k <= 0 || max_ctx <= 2 || vxc_net_config_get(target, &tc) ||
        vxc_net_config_get(draft, &dc)) {
        vxc_set_error("vxc_spec_create: bad arguments");
        return -4;
    }
    if (tc.n_vocab != dc.n_vocab) {
        vxc_set_error("vxc_spec_create: draft vocab %d != target vocab %d", dc.n_vocab, tc.n_vocab);
        return -4;
    }
    vxc_spec *e = (vxc_spec *)calloc(1, sizeof(vxc_spec));
    e->tnet = target;
    e->dnet = draft;
    e->S = n_seq;
    e->k = k;
    e->max_ctx = max_ctx;
    e->V = tc.n_vocab;
    int trows = n_seq * (k + 1) > 64 ? n_seq * (k + 1) : 64;
    int drows = 2 * n_seq > 64 ? 2 * n_seq : 64;
    e->prefill_cap = 2 * 2 * n_seq * ((max_ctx + 63) / 64);
    if ((rc = vxc_seqs_create(target, n_seq, max_ctx, trows, &e->ts)) ||
        (rc = vxc_seqs_create(draft, n_seq, max_ctx, drows, &e->ds))) {
        vxc_spec_destroy(e);
        return rc;
    }
    const int S = n_seq;
    SpecDev &D = e->D;
    D.S = S;
    D.k = k;
    D.cap = max_ctx + k + 2;
    D.max_ctx = max_ctx;
    cudaError_t err = cudaSuccess;
#define DALLOC(p, n) if (err == cudaSuccess) err = cudaMalloc((void **)&(p), (n))
    DALLOC(D.c, (size_t)S * D.cap * sizeof(int));
    DALLOC(D.L, S * sizeof(int));
    DALLOC(D.gen, S * sizeof(int));
    DALLOC(D.done, S * sizeof(int));
    DALLOC(D.seq_id, S * sizeof(int));
    DALLOC(D.slot, S * sizeof(int));
    DALLOC(D.tok0, 2 * S * sizeof(int));
    DALLOC(D.pos0, S * sizeof(int));
    DALLOC(D.lrow0, S * sizeof(int));
    DALLOC(D.dpos, (size_t)k * S * sizeof(int));
    DALLOC(D.dtok, (size_t)k * S * sizeof(int));
    DALLOC(D.vtok, (size_t)S * (k + 1) * sizeof(int));
    DALLOC(D.vpos, S * sizeof(int));
    DALLOC(D.vrows, (size_t)S * (k + 1) * sizeof(int));
    DALLOC(D.dseq, (size_t)S * k * sizeof(int));
    DALLOC(D.apos, S * sizeof(int));
    DALLOC(D.n_acc, S * sizeof(int));
    DALLOC(D.next, S * sizeof(int));
    DALLOC(D.ctr, 3 * sizeof(long long));
    DALLOC(D.n_done, sizeof(int));
    DALLOC(e->dlog, (size_t)k * S * e->V * sizeof(float));
    DALLOC(e->vlog, (size_t)S * (k + 1) * e->V * sizeof(float));
    DALLOC(e->acc_ws, accept_ws(S, k));
    DALLOC(e->prefill_meta, (size_t)e->prefill_cap * sizeof(int));
#undef DALLOC
    if (err == cudaSuccess) err = cudaMemset(e->acc_ws, 0, accept_ws(S, k));
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&e->st2, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaMallocHost((void **)&e->h_ndone, 4 * sizeof(int));
    if (err == cudaSuccess) {
        std::vector<int> sl(S);
        for (int i = 0; i < S; i++) sl[i] = i;
        err = cudaMemcpy(D.slot, sl.data(), S * sizeof(int), cudaMemcpyHostToDevice);
    }
    if (err != cudaSuccess) {
        vxc_set_error("vxc_spec_create: %s", cudaGetErrorString(err));
        vxc_spec_destroy(e);
        return -3;
    }
    *out = e;
    return 0;
}

extern "C" void vxc_spec_destroy(vxc_spec *e) {
    if (!e) return;
    if (e->exec) cudaGraphExecDestroy(e->exec);
    if (e->graph) cudaGraphDestroy(e->graph);
    vxc_seqs_destroy(e->ts);
    vxc_seqs_destroy(e->ds);
    SpecDev &D = e->D;
    void *ptrs[] = {D.c, D.L, D.gen, D.done, D.seq_id, D.slot, D.out, D.tok0, D.pos0, D.lrow0, D.dpos, D.dtok,
                    D.vtok, D.vpos, D.vrows, D.dseq, D.apos, D.n_acc, D.next, D.ctr, D.n_done, e->dlog, e->vlog,
                    e->acc_ws, e->prefill_meta};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    if (e->h_ndone) cudaFreeHost(e->h_ndone);
    if (e->st) cudaStreamDestroy(e->st);
    if (e->st2) cudaStreamDestroy(e->st2);
    free(e);
}

// Enqueue one round on e->st (capturable).
static int enqueue_round(vxc_spec *e, float temp, uint64_t seed) {
    SpecDev &D = e->D;
    const int S = D.S, k = D.k, V = e->V;
    cudaStream_t st = e->st;
    const int tb = 128, gb = (S + tb - 1) / tb;
    int rc;
    (k_round_prep<<<gb, tb, 0, st>>>(D), vxc_count_launches(1));
    // draft step 0: 2 rows per sequence
    if ((rc = vxc_forward(e->ds, D.tok0, D.slot, D.pos0, S, 2, D.lrow0, S, e->dlog, st))) return rc;
    (k_sample_rows<<<S, SMP_THREADS, 0, st>>>(e->dlog, V, temp, seed, D.dpos, D.seq_id, VXC_PURPOSE_DRAFT, D.dtok), vxc_count_launches(1));
    for (int i = 1; i < k; i++) {
        float *q = e->dlog + (size_t)i * S * V;
        // rows: d_i at position L+i-1 == dpos[i-1]; logits of all S rows
        if ((rc = vxc_forward(e->ds, D.dtok + (size_t)(i - 1) * S, D.slot, D.dpos + (size_t)(i - 1) * S, S, 1,
                              D.slot, S, q, st)))
            return rc;
        (k_sample_rows<<<S, SMP_THREADS, 0, st>>>(q, V, temp, seed, D.dpos + (size_t)i * S, D.seq_id,
                                                 VXC_PURPOSE_DRAFT, D.dtok + (size_t)i * S), vxc_count_launches(1));
    }
    (k_gather_verify<<<gb, tb, 0, st>>>(D), vxc_count_launches(1));
    if ((rc = vxc_forward(e->ts, D.vtok, D.slot, D.vpos, S, k + 1, D.vrows, S * (k + 1), e->vlog, st))) return rc;
    if ((rc = launch_accept(e->vlog, (long long)(k + 1) * V, V, e->dlog, V, (long long)S * V, D.dseq, S, k, V, temp,
                            seed, D.seq_id, D.apos, D.n_acc, D.next, e->acc_ws, st)))
        return rc;
    (k_commit<<<gb, tb, 0, st>>>(D), vxc_count_launches(1));
    cudaError_t er = cudaGetLastError();
    if (er != cudaSuccess) { vxc_set_error("round: %s", cudaGetErrorString(er)); return -3; }
    return 0;
}

// Tail of a generate call: wait for the rounds, copy the outputs and the
// counters, fill *stats (events ev[0..2]: start, end of prompt pass, end).
static int finish_generate(vxc_spec *e, int *out, int *counts, vxc_spec_stats *stats, cudaEvent_t *ev,
                           int launched) {
    SpecDev &D = e->D;
    const int S = e->S, max_new = D.max_new;
    cudaStream_t st = e->st;
    cudaEventRecord(ev[2], st);
    cudaError_t err = cudaStreamSynchronize(st);
    if (err == cudaSuccess) {
        std::vector<int> gen(S);
        err = cudaMemcpy(out, D.out, (size_t)S * max_new * sizeof(int), cudaMemcpyDeviceToHost);
        if (err == cudaSuccess) err = cudaMemcpy(gen.data(), D.gen, S * sizeof(int), cudaMemcpyDeviceToHost);
        if (err == cudaSuccess && counts) memcpy(counts, gen.data(), S * sizeof(int));
        if (err == cudaSuccess && stats) {
            long long ctr[3];
            cudaMemcpy(ctr, D.ctr, sizeof ctr, cudaMemcpyDeviceToHost);
            float a = 0, b = 0;
            cudaEventElapsedTime(&a, ev[0], ev[1]);
            cudaEventElapsedTime(&b, ev[1], ev[2]);
            stats->rounds = launched;
            stats->drafted = ctr[0];
            stats->accepted = ctr[1];
            stats->emitted = ctr[2];
            stats->prefill_ms = a;
            stats->decode_ms = b;
        }
    }
    for (int i = 0; i < 4; i++) cudaEventDestroy(ev[i]);
    if (err != cudaSuccess) { vxc_set_error("vxc_spec_generate: %s", cudaGetErrorString(err)); return -3; }
    return vxc_check_device_error(NULL);
}

extern "C" int vxc_spec_generate(vxc_spec *e, const int *prompts, const int *prompt_len, const int *seq_id,
                                 int n_seq, int max_new, float temp, uint64_t seed, int *out, int *counts,
                                 vxc_spec_stats *stats) {
    if (!e || !prompts || !prompt_len || n_seq != e->S || max_new <= 0 || !out) {
        vxc_set_error("vxc_spec_generate: bad arguments (engine holds %d sequences)", e ? e->S : 0);
        return -4;
    }
    SpecDev &D = e->D;
    const int S = e->S, k = e->k;
    int maxp = 0;
    for (int s = 0; s < S; s++) {
        if (prompt_len[s] < 1) { vxc_set_error("vxc_spec_generate: empty prompt"); return -4; }
        if (prompt_len[s] > maxp) maxp = prompt_len[s];
    }
    if (maxp + k + 2 > e->max_ctx) { vxc_set_error("vxc_spec_generate: prompt longer than the context"); return -4; }
    cudaStream_t st = e->st;
    cudaError_t err = cudaSuccess;
    // output buffer sized for this call
    if (D.out == NULL || D.max_new < max_new) {
        if (D.out) cudaFree(D.out);
        D.out = NULL;
        err = cudaMalloc((void **)&D.out, (size_t)S * max_new * sizeof(int));
        if (err != cudaSuccess) { vxc_set_error("vxc_spec_generate: %s", cudaGetErrorString(err)); return -3; }
        if (e->exec) { cudaGraphExecDestroy(e->exec); e->exec = NULL; }
        if (e->graph) { cudaGraphDestroy(e->graph); e->graph = NULL; }
    }
    D.max_new = max_new;
    // committed tokens, lengths, ids
    {
        std::vector<int> c((size_t)S * D.cap, 0), L(S), ids(S);
        size_t off = 0;
        for (int s = 0; s < S; s++) {
            memcpy(&c[(size_t)s * D.cap], prompts + off, (size_t)prompt_len[s] * sizeof(int));
            off += prompt_len[s];
            L[s] = prompt_len[s];
            ids[s] = seq_id ? seq_id[s] : s;
        }
        err = cudaMemcpyAsync(D.c, c.data(), c.size() * sizeof(int), cudaMemcpyHostToDevice, st);
        if (err == cudaSuccess) err = cudaMemcpyAsync(D.L, L.data(), S * sizeof(int), cudaMemcpyHostToDevice, st);
        if (err == cudaSuccess) err = cudaMemcpyAsync(D.seq_id, ids.data(), S * sizeof(int), cudaMemcpyHostToDevice, st);
        if (err == cudaSuccess) err = cudaMemsetAsync(D.gen, 0, S * sizeof(int), st);
        if (err == cudaSuccess) err = cudaMemsetAsync(D.done, 0, S * sizeof(int), st);
        if (err == cudaSuccess) err = cudaMemsetAsync(D.ctr, 0, 3 * sizeof(long long), st);
        if (err == cudaSuccess) err = cudaMemsetAsync(D.n_done, 0, sizeof(int), st);
        if (err == cudaSuccess) err = cudaStreamSynchronize(st);
        if (err != cudaSuccess) { vxc_set_error("vxc_spec_generate: %s", cudaGetErrorString(err)); return -3; }
    }
    cudaEvent_t ev[4];
    for (int i = 0; i < 4; i++) cudaEventCreate(&ev[i]);
    // ---- prompt pass: target rows 0..L-2, draft rows 0..L-3, in chunks of 64 rows
    // read straight from the committed tokens; the draft's chunks run on st2
    // beside the target's, with no host round trip between chunks ----
    cudaEventRecord(ev[0], st);
    {
        std::vector<int> meta;
        std::vector<int> which_of, len_of;
        for (int which = 0; which < 2; which++)
            for (int sq = 0; sq < S; sq++) {
                const int n = prompt_len[sq] - (which == 0 ? 1 : 2);
                for (int done = 0; done < n; done += 64) {
                    meta.push_back(sq);
                    meta.push_back(done);
                    which_of.push_back(which);
                    len_of.push_back(n - done < 64 ? n - done : 64);
                }
            }
        if ((int)meta.size() > e->prefill_cap) {
            vxc_set_error("vxc_spec_generate: prompt chunks exceed the engine's context");
            return -4;
        }
        cudaEvent_t up, join;
        cudaEventCreateWithFlags(&up, cudaEventDisableTiming);
        cudaEventCreateWithFlags(&join, cudaEventDisableTiming);
        if (!meta.empty())
            err = cudaMemcpyAsync(e->prefill_meta, meta.data(), meta.size() * sizeof(int), cudaMemcpyHostToDevice, st);
        cudaEventRecord(up, st);
        cudaStreamWaitEvent(e->st2, up, 0);
        int rc = 0;
        for (size_t i = 0; i < which_of.size() && rc == 0 && err == cudaSuccess; i++) {
            const int sq = meta[2 * i], done = meta[2 * i + 1];
            const bool tgt = which_of[i] == 0;
            rc = vxc_forward(tgt ? e->ts : e->ds, D.c + (size_t)sq * D.cap + done, e->prefill_meta + 2 * i,
                             e->prefill_meta + 2 * i + 1, 1, len_of[i], NULL, 0, NULL, tgt ? st : e->st2);
        }
        cudaEventRecord(join, e->st2);
        cudaStreamWaitEvent(st, join, 0);
        cudaEventDestroy(up);
        cudaEventDestroy(join);
        if (rc) return rc;
        if (err != cudaSuccess) { vxc_set_error("vxc_spec_generate: %s", cudaGetErrorString(err)); return -3; }
    }
    cudaEventRecord(ev[1], st);
    // ---- round loop: first round eager, then a captured graph ----
    int rc = enqueue_round(e, temp, seed);
    if (rc) return rc;
    int launched = 1;
    // VX_SPEC_EAGER=1 runs every round as plain launches (for kernel profilers,
    // which cannot attribute work inside graph replays); results are identical.
    static const bool eager = getenv("VX_SPEC_EAGER") != NULL && getenv("VX_SPEC_EAGER")[0] == '1';
    if (eager) {
        while (launched < max_new + 1 && rc == 0) {
            err = cudaMemcpyAsync(e->h_ndone, D.n_done, sizeof(int), cudaMemcpyDeviceToHost, st);
            if (err == cudaSuccess) err = cudaStreamSynchronize(st);
            if (err != cudaSuccess || *(volatile int *)e->h_ndone >= S) break;
            rc = enqueue_round(e, temp, seed);
            launched++;
        }
        if (rc) return rc;
        return finish_generate(e, out, counts, stats, ev, launched);
    }
    // temp/seed are baked into the graph: rebuild it each call
    if (e->exec) { cudaGraphExecDestroy(e->exec); e->exec = NULL; }
    if (e->graph) { cudaGraphDestroy(e->graph); e->graph = NULL; }
    const long long n_before = vxc_launch_count();
    err = cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed);
    if (err == cudaSuccess) {
        rc = enqueue_round(e, temp, seed);
        if (rc == 0) err = cudaMemcpyAsync(e->h_ndone, D.n_done, sizeof(int), cudaMemcpyDeviceToHost, st);
        cudaError_t e2 = cudaStreamEndCapture(st, &e->graph);
        if (err == cudaSuccess) err = e2;
        if (rc) return rc;
    }
    // captured launches are not executed; each replay below counts them
    const long long per_round = vxc_launch_count() - n_before;
    vxc_count_launches(-per_round);
    if (err == cudaSuccess) err = cudaGraphInstantiate(&e->exec, e->graph, 0);
    if (err != cudaSuccess) { vxc_set_error("vxc_spec_generate: graph: %s", cudaGetErrorString(err)); return -3; }
    // each round emits >= 1 token per active sequence: max_new rounds suffice
    int checked = 0;
    cudaEvent_t rev[2];
    cudaEventCreateWithFlags(&rev[0], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&rev[1], cudaEventDisableTiming);
    // Two rounds stay in flight, and the older one's count decides whether to
    // stop; the newer round may already have written that count, so the number
    // of rounds run can vary by one with timing.  A tensor-parallel target runs
    // collectives in every round, which all GPUs must run equally often: there
    // each round's own count decides, one round in flight.
    const int depth = vxc_net_world(e->tnet) > 1 ? 1 : 2;
    int pending = 0;
    while (launched < max_new + 1) {
        err = cudaGraphLaunch(e->exec, st);
        if (err != cudaSuccess) break;
        vxc_count_launches(per_round);
        cudaEventRecord(rev[launched & 1], st);
        launched++;
        pending++;
        if (pending == depth) {
            // wait for the oldest round in flight and read its count
            cudaEventSynchronize(rev[(launched - depth) & 1]);
            pending = depth - 1;
            checked++;
            if (*(volatile int *)e->h_ndone >= S) break;
        }
    }
    cudaEventDestroy(rev[0]);
    cudaEventDestroy(rev[1]);
    (void)checked;
    if (err != cudaSuccess) { vxc_set_error("vxc_spec_generate: %s", cudaGetErrorString(err)); return -3; }
    return finish_generate(e, out, counts, stats, ev, launched);
}

// Re-runs one piece of the last round `reps` times on the engine's stream and
// reports its average device time: which = 0 the (k+1)-row target verify
// forward, 1 one draft step (one row per sequence), 2 the fused acceptance.
// Positions and tokens are those of the last round, so the KV rows written
// lie past every committed position and the committed state is unchanged.
// *kv_bytes receives the K/V bytes that one such forward reads and writes.
extern "C" int vxc_spec_probe(vxc_spec *e, int which, int reps, double *ms, double *kv_bytes) {
    if (!e || reps < 1 || which < 0 || which > 2 || !ms) {
        vxc_set_error("vxc_spec_probe: bad arguments");
        return -4;
    }
    SpecDev &D = e->D;
    const int S = D.S, k = D.k, V = e->V;
    cudaStream_t st = e->st;
    std::vector<int> vpos(S);
    cudaError_t err = cudaMemcpy(vpos.data(), D.vpos, S * sizeof(int), cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) { vxc_set_error("vxc_spec_probe: %s", cudaGetErrorString(err)); return -3; }
    vxc_net_config c;
    vxc_net_config_get(which == 1 ? e->dnet : e->tnet, &c);
    const double kvd = (double)c.n_kv_heads * c.n_head_dim;
    double kvb = 0.0;
    for (int s = 0; s < S; s++) {
        // verify: reads positions 0..vpos+k, writes k+1; draft step: reads 0..vpos+1, writes 1
        double rd = which == 0 ? vpos[s] + k + 1 : which == 1 ? vpos[s] + 2 : 0;
        double wr = which == 0 ? k + 1 : which == 1 ? 1 : 0;
        kvb += (rd + wr) * kvd * 2.0 * 4.0 * c.n_layers;
    }
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    int rc = 0;
    for (int it = -1; it < reps && rc == 0; it++) {   // it == -1: untimed warm-up
        if (it == 0) cudaEventRecord(a, st);
        if (which == 0)
            rc = vxc_forward(e->ts, D.vtok, D.slot, D.vpos, S, k + 1, D.vrows, S * (k + 1), e->vlog, st);
        else if (which == 1)
            rc = vxc_forward(e->ds, D.dtok, D.slot, D.dpos, S, 1, D.slot, S, e->dlog, st);
        else
            rc = launch_accept(e->vlog, (long long)(k + 1) * V, V, e->dlog, V, (long long)S * V, D.dseq, S, k, V,
                               0.8f, 1, D.seq_id, D.apos, D.n_acc, D.next, e->acc_ws, st);
    }
    cudaEventRecord(b, st);
    err = cudaStreamSynchronize(st);
    float t = 0.0f;
    if (rc == 0 && err == cudaSuccess) cudaEventElapsedTime(&t, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (rc) return rc;
    if (err != cudaSuccess) { vxc_set_error("vxc_spec_probe: %s", cudaGetErrorString(err)); return -3; }
    *ms = t / reps;
    if (kv_bytes) *kv_bytes = kvb;
    return vxc_check_device_error(NULL);
}
