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
//                    bonus from p_k         (fused kernel k_accept, one cluster)
//     commit         c += d_1..d_a, next ; L += a + 1
// KV invariants: target holds 0..L-2 at round start (the verify rewrites
// L-1..); draft holds 0..L-3 (step 0 rewrites L-2, L-1).  Positions past a
// rejection hold stale K/V that the next round overwrites before reading.
// All sampling decisions use exact integer weights (vxc_weight), so they match
// the oracle bit-for-bit given the same logits.
#include "vxc_common.cuh"
#include "vxc_internal.h"

#include <cooperative_groups.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <algorithm>
#include <utility>
#include <vector>

namespace cg = cooperative_groups;

typedef unsigned long long u64;
typedef unsigned __int128 u128;

// ---------------------------------------------------------------------------
// cluster row helpers
//
// A row of V logits is handled by one thread-block cluster of CL CTAs.  CTA c
// owns the slice [c*sw, (c+1)*sw) of the row (sw a multiple of 128 elements,
// so slices of a 16-byte aligned row start 16-byte aligned) and cuts it into
// at most CL_SPB draw sub-blocks (CL_SPW per warp), so that the row's
// sub-block table has one entry per thread of a CTA.  Partial results (maxima,
// weight sums, sub-block sums) are exchanged through distributed shared
// memory between cluster barriers; every CTA of a cluster passes the same
// sequence of barriers.
// ---------------------------------------------------------------------------
#define CL 8
#define CL_THREADS 256
#define CL_WARPS (CL_THREADS / 32)
#define CL_SPW 4                   // draw sub-blocks per warp
#define CL_SPB (CL_WARPS * CL_SPW)  // draw sub-blocks per CTA
#define CL_SUBS (CL * CL_SPB)       // draw sub-blocks of a row, in element order
static_assert(CL_SUBS <= CL_THREADS, "one sub-block entry per thread of the leader");

struct MaxIdx {
    float v;
    int i;
};

__device__ __forceinline__ MaxIdx better(MaxIdx a, MaxIdx b) {
    // larger value wins; on ties the lower index (first maximum)
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

struct Slice {
    int a, b;   // elements [a, b) of the row
    int sb;     // draw sub-block length, a multiple of 128
    int nsb;    // sub-blocks in [a, b), at most CL_SPB
};

__device__ __forceinline__ Slice cl_slice(int V, int c) {
    const int sw = ((V + CL - 1) / CL + 127) & ~127;
    Slice s;
    s.a = min(V, c * sw);
    s.b = min(V, s.a + sw);
    s.sb = ((sw / 128 + CL_SPB - 1) / CL_SPB) * 128;
    s.nsb = (s.b - s.a + s.sb - 1) / s.sb;
    return s;
}

// Elements v..v+3 of a row (v % 4 == 0); positions at or past `end` read as
// -inf (sampling weight 0).  One 16-byte load when the row is 16-byte aligned.
__device__ __forceinline__ float4 ld_quad(const float *__restrict__ row, int v, int end, bool vec) {
    if (vec && v + 4 <= end) return __ldg(reinterpret_cast<const float4 *>(row + v));
    float4 r;
    r.x = v < end ? __ldg(row + v) : -INFINITY;
    r.y = v + 1 < end ? __ldg(row + v + 1) : -INFINITY;
    r.z = v + 2 < end ? __ldg(row + v + 2) : -INFINITY;
    r.w = v + 3 < end ? __ldg(row + v + 3) : -INFINITY;
    return r;
}

// f(v, x) for every element v of [a, b) (a % 4 == 0), a quad per thread per
// step with up to four quads in flight.  The visiting order differs per
// thread, so f must be order-independent (integer sums, first-max argmax).
template <class F>
__device__ __forceinline__ void slice_pass(const float *__restrict__ row, int a, int b, bool vec, F f) {
#pragma unroll 4
    for (int v = a + 4 * (int)threadIdx.x; v < b; v += 4 * CL_THREADS) {
        const float4 x = ld_quad(row, v, b, vec);
        f(v, x.x);
        if (v + 1 < b) f(v + 1, x.y);
        if (v + 2 < b) f(v + 2, x.z);
        if (v + 3 < b) f(v + 3, x.w);
    }
}

// The same over two rows at once (twice the loads in flight; a 32000-wide
// row's slice is four steps, all unrolled): fa(v, ra[v]) and fb(v, rb[v]).
template <class F, class G>
__device__ __forceinline__ void slice_pass2(const float *__restrict__ ra, const float *__restrict__ rb, int a, int b,
                                            bool vec, F fa, G fb) {
#pragma unroll 4
    for (int v = a + 4 * (int)threadIdx.x; v < b; v += 4 * CL_THREADS) {
        const float4 x = ld_quad(ra, v, b, vec), y = ld_quad(rb, v, b, vec);
        fa(v, x.x);
        fb(v, y.x);
        if (v + 1 < b) {
            fa(v + 1, x.y);
            fb(v + 1, y.y);
        }
        if (v + 2 < b) {
            fa(v + 2, x.z);
            fb(v + 2, y.z);
        }
        if (v + 3 < b) {
            fa(v + 3, x.w);
            fb(v + 3, y.w);
        }
    }
}

__device__ __forceinline__ MaxIdx warp_best(MaxIdx m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        MaxIdx t;
        t.v = __shfl_xor_sync(0xffffffffu, m.v, o);
        t.i = __shfl_xor_sync(0xffffffffu, m.i, o);
        m = better(m, t);
    }
    return m;
}

__device__ __forceinline__ u64 warp_sum_u64(u64 v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ u64 warp_incl_scan_u64(u64 v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const u64 t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

__device__ u64 block_sum_u64(u64 v, u64 *red) {
    v = warp_sum_u64(v);
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
    const u64 inc = warp_incl_scan_u64(v, l);
    __syncthreads();
    if (l == 31) red[w] = inc;
    __syncthreads();
    u64 base = 0;
    for (int i = 0; i < w; i++) base += red[i];
    __syncthreads();
    return base + inc - v;
}

// Sum of w4's weights over each draw sub-block of this CTA's slice: warp w
// takes sub-blocks w, w + CL_WARPS, ... (CL_SPW of them, summed side by side
// for loads in flight), lane l the quads at s0 + 128 q + 4 l.  w4(v, end, w)
// writes the weights of elements v..v+3 (0 at or past end).
template <class W4>
__device__ __forceinline__ void slice_sub_sums(const Slice &sl, W4 w4, u64 *sub) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    u64 acc[CL_SPW];
#pragma unroll
    for (int t = 0; t < CL_SPW; t++) {
        const int j = w + t * CL_WARPS;
        acc[t] = 0;
        if (j < sl.nsb) {
            const int s0 = sl.a + j * sl.sb, s1 = min(sl.b, s0 + sl.sb);
            for (int q = s0 + 4 * lane; q < s1; q += 128) {
                u64 x[4];
                w4(q, s1, x);
                acc[t] += x[0] + x[1] + x[2] + x[3];
            }
        }
    }
#pragma unroll
    for (int t = 0; t < CL_SPW; t++) {
        const int j = w + t * CL_WARPS;
        const u64 a = warp_sum_u64(acc[t]);
        if (lane == 0 && j < sl.nsb) sub[j] = a;
    }
}

// The cluster leader's entry of the row's sub-block table: thread t <
// CL_SUBS reads sub-block t % CL_SPB of CTA t / CL_SPB (0 where that slice
// has fewer sub-blocks), so threads 0..CL_SUBS-1 hold the table in element
// order.  Call between two cluster barriers.
__device__ __forceinline__ u64 cl_table_entry(cg::cluster_group &cl, int V, u64 *sub) {
    u64 e = 0;
    if (threadIdx.x < CL_SUBS) {
        const int c = threadIdx.x / CL_SPB, j = threadIdx.x % CL_SPB;
        if (j < cl_slice(V, c).nsb) e = *cl.map_shared_rank(sub + j, c);
    }
    return e;
}

// First element whose inclusive prefix weight exceeds thr (V - 1 if none, as
// the oracle's draw), given each thread's table entry e: a block scan finds
// the sub-block holding thr, then warp 0 rescans it quad by quad with w4.
// The result is valid in warp 0.
template <class W4>
__device__ int cl_draw(int V, u64 e, u64 thr, W4 w4, u64 *red, int *s_sub, u64 *s_base) {
    const u64 ex = block_excl_scan_u64(e, red);
    if (threadIdx.x == 0) *s_sub = -1;
    __syncthreads();
    if (e != 0 && ex <= thr && thr < ex + e) {
        *s_sub = threadIdx.x;
        *s_base = ex;
    }
    __syncthreads();
    const int f = *s_sub;
    int res = V - 1;
    if (f >= 0 && threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const Slice sl = cl_slice(V, f / CL_SPB);
        const int s0 = sl.a + (f % CL_SPB) * sl.sb, s1 = min(sl.b, s0 + sl.sb);
        u64 base = *s_base;
        for (int q = s0; q < s1; q += 128) {
            const int v = q + 4 * lane;
            u64 w[4];
            w4(v, s1, w);
            const u64 lt = w[0] + w[1] + w[2] + w[3];
            const u64 inc = warp_incl_scan_u64(lt, lane);
            const u64 lex = base + inc - lt;
            const unsigned hit = __ballot_sync(0xffffffffu, lt != 0 && lex <= thr && thr < lex + lt);
            if (hit) {
                const int hl = __ffs(hit) - 1;
                int t = V - 1;
                if (lane == hl) {
                    u64 a = lex;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        a += w[i];
                        if (a > thr) {
                            t = v + i;
                            break;
                        }
                    }
                }
                res = __shfl_sync(0xffffffffu, t, hl);
                break;
            }
            base += __shfl_sync(0xffffffffu, inc, 31);
        }
    }
    __syncthreads();
    return res;
}

__device__ __forceinline__ u64 draw_threshold(u64 S, uint32_t word) {
    return (u64)(((u128)S * (word >> 8)) >> 24);
}

// ---------------------------------------------------------------------------
// per-row sampler: one cluster per row (grid CL x n_rows)
// ---------------------------------------------------------------------------
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(CL_THREADS)
    k_sample_rows(const float *__restrict__ logits, int V, float temp, u64 seed, const int *__restrict__ pos,
                  const int *__restrict__ seq, unsigned purpose, int *__restrict__ out, int vec) {
    cg::cluster_group cl = cg::this_cluster();
    __shared__ MaxIdx red_m[CL_WARPS];
    __shared__ MaxIdx part_m, g_m;
    __shared__ u64 red_u[32];
    __shared__ u64 sub[CL_SPB];
    __shared__ int s_sub;
    __shared__ u64 s_base;
    const int c = blockIdx.x, r = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *row = logits + (size_t)r * V;
    const Slice sl = cl_slice(V, c);
    // first maximum of the row
    MaxIdx m = {-INFINITY, 0x7fffffff};
    slice_pass(row, sl.a, sl.b, vec, [&](int v, float x) { m = better(m, MaxIdx{x, v}); });
    m = warp_best(m);
    if (lane == 0) red_m[w] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        MaxIdx b = red_m[0];
        for (int i = 1; i < CL_WARPS; i++) b = better(b, red_m[i]);
        part_m = b;
    }
    cl.sync();
    if (threadIdx.x == 0) {
        MaxIdx b = *cl.map_shared_rank(&part_m, 0);
        for (int i = 1; i < CL; i++) b = better(b, *cl.map_shared_rank(&part_m, i));
        g_m = b;
    }
    __syncthreads();
    const MaxIdx g = g_m;
    if (!(temp > 0.0f)) {
        cl.sync();   // every remote read is done before any CTA of the cluster exits
        if (c == 0 && threadIdx.x == 0) out[r] = g.i;
        return;
    }
    // integer weights W_v = vxc_weight(l_v, max, 1/T): sub-block sums, then the draw
    const float invT = 1.0f / temp;
    auto w4 = [&](int v, int end, u64 *wt) {
        const float4 x = ld_quad(row, v, end, vec);
        wt[0] = vxc_weight(x.x, g.v, invT);
        wt[1] = vxc_weight(x.y, g.v, invT);
        wt[2] = vxc_weight(x.z, g.v, invT);
        wt[3] = vxc_weight(x.w, g.v, invT);
    };
    slice_sub_sums(sl, w4, sub);
    cl.sync();
    const u64 e = c == 0 ? cl_table_entry(cl, V, sub) : 0;
    cl.sync();
    if (c != 0) return;
    const u64 S = block_sum_u64(e, red_u);
    const uint32_t word = vxc_philox_u32(seed, (uint32_t)pos[r], (uint32_t)seq[r], purpose);
    const int t = cl_draw(V, e, draw_threshold(S, word), w4, red_u, &s_sub, &s_base);
    if (threadIdx.x == 0) out[r] = t;
}

static int launch_sample_rows(const float *logits, int n_rows, int V, float temp, uint64_t seed, const int *pos,
                              const int *seq, unsigned purpose, int *out, cudaStream_t st) {
    if (n_rows > 65535) {
        vxc_set_error("vxc_sample_rows: %d rows, at most 65535 per launch", n_rows);
        return -4;
    }
    const int vec = (((uintptr_t)logits) & 15) == 0 && (V & 3) == 0;
    (k_sample_rows<<<dim3(CL, n_rows), CL_THREADS, 0, st>>>(logits, V, temp, seed, pos, seq, purpose, out, vec),
     vxc_count_launches(1));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        vxc_set_error("vxc_sample_rows: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}

extern "C" int vxc_sample_rows(const float *logits, int n_rows, int V, float temp, uint64_t seed, const int *d_pos,
                               const int *d_seq, unsigned int purpose, int *d_tokens, void *stream) {
    if (!logits || n_rows <= 0 || V <= 0 || !d_pos || !d_seq || !d_tokens) {
        vxc_set_error("vxc_sample_rows: bad arguments");
        return -4;
    }
    return launch_sample_rows(logits, n_rows, V, temp, seed, d_pos, d_seq, purpose, d_tokens, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// fused acceptance: one cluster per sequence (grid CL x n_seq)
//
// Rows r = 0..k are the target rows P_0..P_k, rows k+1..2k the draft rows
// Q_0..Q_{k-1}; every CTA covers its slice of all of them.
//   1. max and first argmax of every row                      (exchange)
//   2. integer weight sums S_r of P_j and Q_j, j < k           (exchange)
//   3. first rejection j: u24 * Wq(d_j) * Sp_j >= 2^24 * Wp(d_j) * Sq_j
//   4. sub-block sums of the residual (Wp Sq - Wq Sp)^+ >> 36 of row j, or
//      of the bonus row P_k's weights when all k are accepted (exchange)
//   5. the cluster leader draws from the sub-block table.
// Greedy (temp <= 0) stops after 1: the first j with d_j != argmax P_j.
// ---------------------------------------------------------------------------
#define ACC_MAX_K 64
// Prompt pass: rows of one sequence per forward group, and rows per forward call.
#define PREFILL_PIECE 512
#define PREFILL_ROWS 4096
#define ACC_MAX_ROWS (2 * ACC_MAX_K + 1)

__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(CL_THREADS, 4)
    k_accept(const float *__restrict__ P, long long p_seq, long long p_pos, const float *__restrict__ Q,
             long long q_seq, long long q_pos, const int *__restrict__ d, int k, int V, float temp, u64 seed,
             const int *__restrict__ seq_id, const int *__restrict__ pos0, int *__restrict__ n_acc,
             int *__restrict__ next, int vec) {
    cg::cluster_group cl = cg::this_cluster();
    __shared__ MaxIdx red_m[ACC_MAX_ROWS][CL_WARPS];
    __shared__ u64 red_s[ACC_MAX_ROWS][CL_WARPS];
    __shared__ MaxIdx part_m[ACC_MAX_ROWS], g_m[ACC_MAX_ROWS];
    __shared__ u64 part_s[ACC_MAX_ROWS], g_s[ACC_MAX_ROWS];
    __shared__ u64 sub[CL_SPB];
    __shared__ u64 red_u[32];
    __shared__ int first_rej, s_sub;
    __shared__ u64 s_base;
    const int c = blockIdx.x, s = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool greedy = !(temp > 0.0f);
    const int R = greedy ? k + 1 : 2 * k + 1;
    const Slice sl = cl_slice(V, c);
    auto rowp = [&](int r) -> const float * {
        return r <= k ? P + s * p_seq + r * p_pos : Q + s * q_seq + (r - k - 1) * q_pos;
    };
    if (threadIdx.x == 0) first_rej = k;
    // 1. maxima: P_j with Q_j (sampled), then the rest of the P rows alone
    const int npair = greedy ? 0 : k;
    for (int j = 0; j < npair; j++) {
        MaxIdx mp = {-INFINITY, 0x7fffffff}, mq = mp;
        slice_pass2(rowp(j), rowp(k + 1 + j), sl.a, sl.b, vec, [&](int v, float x) { mp = better(mp, MaxIdx{x, v}); },
                    [&](int v, float x) { mq = better(mq, MaxIdx{x, v}); });
        mp = warp_best(mp);
        mq = warp_best(mq);
        if (lane == 0) {
            red_m[j][w] = mp;
            red_m[k + 1 + j][w] = mq;
        }
    }
    for (int r = npair; r <= k; r++) {
        MaxIdx m = {-INFINITY, 0x7fffffff};
        slice_pass(rowp(r), sl.a, sl.b, vec, [&](int v, float x) { m = better(m, MaxIdx{x, v}); });
        m = warp_best(m);
        if (lane == 0) red_m[r][w] = m;
    }
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += CL_THREADS) {
        MaxIdx b = red_m[r][0];
        for (int i = 1; i < CL_WARPS; i++) b = better(b, red_m[r][i]);
        part_m[r] = b;
    }
    cl.sync();
    for (int r = threadIdx.x; r < R; r += CL_THREADS) {
        MaxIdx b = cl.map_shared_rank(part_m, 0)[r];
        for (int i = 1; i < CL; i++) b = better(b, cl.map_shared_rank(part_m, i)[r]);
        g_m[r] = b;
    }
    __syncthreads();
    if (greedy) {
        cl.sync();   // every remote read is done before any CTA of the cluster exits
        if (c == 0 && threadIdx.x == 0) {
            int acc = k;
            for (int j = 0; j < k; j++)
                if (d[s * k + j] != g_m[j].i) {
                    acc = j;
                    break;
                }
            n_acc[s] = acc;
            next[s] = g_m[acc].i;
        }
        return;
    }
    const float invT = 1.0f / temp;
    // 2. weight sums of P_j and Q_j, j < k (the bonus row's total comes out
    //    of its sub-block table in 4)
    for (int j = 0; j < k; j++) {
        const float mp = g_m[j].v, mq = g_m[k + 1 + j].v;
        u64 ap = 0, aq = 0;
        slice_pass2(rowp(j), rowp(k + 1 + j), sl.a, sl.b, vec, [&](int, float x) { ap += vxc_weight(x, mp, invT); },
                    [&](int, float x) { aq += vxc_weight(x, mq, invT); });
        ap = warp_sum_u64(ap);
        aq = warp_sum_u64(aq);
        if (lane == 0) {
            red_s[j][w] = ap;
            red_s[k + 1 + j][w] = aq;
        }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += CL_THREADS) {
        if (r == k) continue;
        u64 a = 0;
        for (int i = 0; i < CL_WARPS; i++) a += red_s[r][i];
        part_s[r] = a;
    }
    cl.sync();
    for (int r = threadIdx.x; r < R; r += CL_THREADS) {
        if (r == k) continue;
        u64 a = 0;
        for (int i = 0; i < CL; i++) a += cl.map_shared_rank(part_s, i)[r];
        g_s[r] = a;
    }
    __syncthreads();
    // 3. acceptance tests; the first failing draft position wins
    const int p0 = pos0[s], sid = seq_id[s];
    for (int j = threadIdx.x; j < k; j += CL_THREADS) {
        const int t = d[s * k + j];
        bool ok = false;
        if (t >= 0 && t < V) {
            const u64 wp = vxc_weight(rowp(j)[t], g_m[j].v, invT);
            const u64 wq = vxc_weight(rowp(k + 1 + j)[t], g_m[k + 1 + j].v, invT);
            const u64 u = vxc_philox_u32(seed, (uint32_t)(p0 + j), (uint32_t)sid, VXC_PURPOSE_ACCEPT) >> 8;
            ok = (u128)u * wq * g_s[j] < (((u128)wp * g_s[k + 1 + j]) << 24);
        }
        if (!ok) atomicMin(&first_rej, j);
    }
    __syncthreads();
    const int acc = first_rej;
    const bool resid = acc < k;
    // 4. the distribution to draw from: residual of row acc, or the bonus row
    const float *pr = rowp(acc);
    const float *qr = resid ? rowp(k + 1 + acc) : pr;
    const float mp = g_m[acc].v, mq = resid ? g_m[k + 1 + acc].v : 0.0f;
    const u64 Sp = resid ? g_s[acc] : 0, Sq = resid ? g_s[k + 1 + acc] : 0;
    auto w4 = [&](int v, int end, u64 *wt) {
        const float4 x = ld_quad(pr, v, end, vec);
        if (resid) {
            const float4 y = ld_quad(qr, v, end, vec);
            const float xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const u128 a = (u128)vxc_weight(xs[i], mp, invT) * Sq;
                const u128 b = (u128)vxc_weight(ys[i], mq, invT) * Sp;
                wt[i] = a > b ? (u64)((a - b) >> 36) : 0ull;
            }
        } else {
            wt[0] = vxc_weight(x.x, mp, invT);
            wt[1] = vxc_weight(x.y, mp, invT);
            wt[2] = vxc_weight(x.z, mp, invT);
            wt[3] = vxc_weight(x.w, mp, invT);
        }
    };
    slice_sub_sums(sl, w4, sub);
    cl.sync();
    const u64 e = c == 0 ? cl_table_entry(cl, V, sub) : 0;
    cl.sync();
    if (c != 0) return;
    // 5. draw
    const u64 SR = block_sum_u64(e, red_u);
    int nxt;
    if (resid && SR == 0) {
        nxt = g_m[acc].i;   // p <= q everywhere after rounding: the target's first maximum
    } else {
        const uint32_t word = vxc_philox_u32(seed, (uint32_t)(p0 + acc), (uint32_t)sid, VXC_PURPOSE_RESAMPLE);
        nxt = cl_draw(V, e, draw_threshold(SR, word), w4, red_u, &s_sub, &s_base);
    }
    if (threadIdx.x == 0) {
        n_acc[s] = acc;
        next[s] = nxt;
    }
}

// The kernel keeps all of its state in shared memory; no scratch is needed.
static size_t accept_ws(int, int) { return 0; }

extern "C" size_t vxc_accept_workspace_bytes(int n_seq, int k) { return accept_ws(n_seq, k); }

static int launch_accept(const float *P, long long p_seq, long long p_pos, const float *Q, long long q_seq,
                         long long q_pos, const int *d, int n_seq, int k, int V, float temp, uint64_t seed,
                         const int *seq_id, const int *pos0, int *n_acc, int *next, cudaStream_t st) {
    if (k > ACC_MAX_K || n_seq > 65535) {
        vxc_set_error("vxc_accept: k = %d, n_seq = %d (at most %d and 65535)", k, n_seq, ACC_MAX_K);
        return -4;
    }
    const int vec = (((uintptr_t)P) & 15) == 0 && (((uintptr_t)Q) & 15) == 0 && (p_seq & 3) == 0 &&
                    (p_pos & 3) == 0 && (q_seq & 3) == 0 && (q_pos & 3) == 0;
    (k_accept<<<dim3(CL, n_seq), CL_THREADS, 0, st>>>(P, p_seq, p_pos, Q, q_seq, q_pos, d, k, V, temp, seed, seq_id,
                                                     pos0, n_acc, next, vec),
     vxc_count_launches(1));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        vxc_set_error("vxc_accept: %s", cudaGetErrorString(e));
        return -3;
    }
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
    if (workspace_bytes < accept_ws(n_seq, k) || (accept_ws(n_seq, k) && !workspace)) {
        vxc_set_error("vxc_accept: workspace of %zu bytes needed", accept_ws(n_seq, k));
        return -4;
    }
    return launch_accept(P, p_seq, p_pos, Q, q_seq, q_pos, d, n_seq, k, V, temp, seed, seq_id, pos0, n_acc, next,
                         (cudaStream_t)stream);
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
    int *prefill_meta; // per prompt-pass call: the groups' sequence slots, then their first positions
    int prefill_cap;   // ints in prefill_meta
    int *prefill_tok;  // the prompt-pass calls' token rows, one call after another
    size_t prefill_tok_cap;
    int prefill_rows;  // rows per prompt-pass call (pieces of up to PREFILL_PIECE rows of several sequences)
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
    if (k > ACC_MAX_K || n_seq > 65535) {
        vxc_set_error("vxc_spec_create: k = %d, n_seq = %d (at most %d and 65535)", k, n_seq, ACC_MAX_K);
        return -4;
    }
    vxc_spec *e = (vxc_spec *)calloc(1, sizeof(vxc_spec));
    e->tnet = target;
    e->dnet = draft;
    e->S = n_seq;
    e->k = k;
    e->max_ctx = max_ctx;
    e->V = tc.n_vocab;
    // the prompt pass runs pieces of up to PREFILL_PIECE rows of many sequences per call, up to
    // PREFILL_ROWS rows per call, so the GEMM reads the weights once per VXC_GEMM_SLAB rows
    {
        const long piece = max_ctx < PREFILL_PIECE ? max_ctx : PREFILL_PIECE;
        const long want = (long)n_seq * piece;
        e->prefill_rows = (int)(want < PREFILL_ROWS ? want : PREFILL_ROWS);
    }
    int trows = n_seq * (k + 1) > e->prefill_rows ? n_seq * (k + 1) : e->prefill_rows;
    int drows = 2 * n_seq > e->prefill_rows ? 2 * n_seq : e->prefill_rows;
    e->prefill_cap = 2 * 2 * n_seq * ((max_ctx + 63) / 64);
    e->prefill_tok_cap = (size_t)2 * n_seq * max_ctx;
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
    DALLOC(e->prefill_meta, (size_t)e->prefill_cap * sizeof(int));
    DALLOC(e->prefill_tok, e->prefill_tok_cap * sizeof(int));
#undef DALLOC
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
                    e->prefill_meta, e->prefill_tok};
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
    if ((rc = launch_sample_rows(e->dlog, S, V, temp, seed, D.dpos, D.seq_id, VXC_PURPOSE_DRAFT, D.dtok, st)))
        return rc;
    for (int i = 1; i < k; i++) {
        float *q = e->dlog + (size_t)i * S * V;
        // rows: d_i at position L+i-1 == dpos[i-1]; logits of all S rows
        if ((rc = vxc_forward(e->ds, D.dtok + (size_t)(i - 1) * S, D.slot, D.dpos + (size_t)(i - 1) * S, S, 1,
                              D.slot, S, q, st)))
            return rc;
        if ((rc = launch_sample_rows(q, S, V, temp, seed, D.dpos + (size_t)i * S, D.seq_id, VXC_PURPOSE_DRAFT,
                                     D.dtok + (size_t)i * S, st)))
            return rc;
    }
    (k_gather_verify<<<gb, tb, 0, st>>>(D), vxc_count_launches(1));
    if ((rc = vxc_forward(e->ts, D.vtok, D.slot, D.vpos, S, k + 1, D.vrows, S * (k + 1), e->vlog, st))) return rc;
    if ((rc = launch_accept(e->vlog, (long long)(k + 1) * V, V, e->dlog, V, (long long)S * V, D.dseq, S, k, V, temp,
                            seed, D.seq_id, D.apos, D.n_acc, D.next, st)))
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
    // ---- prompt pass: target rows 0..L-2, draft rows 0..L-3.  Each sequence's
    // rows are cut into pieces of PREFILL_PIECE; piece i of every sequence
    // comes after piece i-1 of all of them, and pieces of equal length go
    // through one forward call, one group per sequence, up to prefill_rows
    // rows.  Every matrix runs on the GEMM (vxc_forward_prompt), whose result
    // for a row depends on that row only, so batching changes no number.
    // Token rows and group tables are uploaded once; the draft's calls run on
    // st2 beside the target's, with no host round trip between calls ----
    cudaEventRecord(ev[0], st);
    {
        struct Call {
            int which, m0, G, T;
            size_t t0;
        };
        std::vector<int> meta, tok;
        std::vector<Call> calls;
        std::vector<size_t> off(S + 1, 0);
        for (int sq = 0; sq < S; sq++) off[sq + 1] = off[sq] + (size_t)prompt_len[sq];
        for (int which = 0; which < 2; which++) {
            auto rows_of = [&](int sq) { return prompt_len[sq] - (which == 0 ? 1 : 2); };
            for (int ci = 0;; ci++) {
                // piece ci of every sequence that has one, grouped by length (ascending)
                std::vector<std::pair<int, int>> pcs;   // (length, sequence)
                for (int sq = 0; sq < S; sq++) {
                    const int n = rows_of(sq) - PREFILL_PIECE * ci;
                    if (n > 0) pcs.push_back({n < PREFILL_PIECE ? n : PREFILL_PIECE, sq});
                }
                if (pcs.empty()) break;
                std::stable_sort(pcs.begin(), pcs.end(),
                                 [](const std::pair<int, int> &a, const std::pair<int, int> &b) { return a.first < b.first; });
                for (size_t b = 0; b < pcs.size();) {
                    const int T = pcs[b].first;
                    const int gmax = e->prefill_rows / T > 0 ? e->prefill_rows / T : 1;
                    size_t end = b;
                    while (end < pcs.size() && pcs[end].first == T && (int)(end - b) < gmax) end++;
                    const int G = (int)(end - b);
                    calls.push_back({which, (int)meta.size(), G, T, tok.size()});
                    for (size_t g = b; g < end; g++) meta.push_back(pcs[g].second);
                    for (size_t g = b; g < end; g++) meta.push_back(PREFILL_PIECE * ci);
                    for (size_t g = b; g < end; g++) {
                        const int *src = prompts + off[pcs[g].second] + (size_t)PREFILL_PIECE * ci;
                        tok.insert(tok.end(), src, src + T);
                    }
                    b = end;
                }
            }
        }
        if ((int)meta.size() > e->prefill_cap || tok.size() > e->prefill_tok_cap) {
            vxc_set_error("vxc_spec_generate: prompt chunks exceed the engine's context");
            return -4;
        }
        cudaEvent_t up, join;
        cudaEventCreateWithFlags(&up, cudaEventDisableTiming);
        cudaEventCreateWithFlags(&join, cudaEventDisableTiming);
        if (!meta.empty())
            err = cudaMemcpyAsync(e->prefill_meta, meta.data(), meta.size() * sizeof(int), cudaMemcpyHostToDevice, st);
        if (err == cudaSuccess && !tok.empty())
            err = cudaMemcpyAsync(e->prefill_tok, tok.data(), tok.size() * sizeof(int), cudaMemcpyHostToDevice, st);
        cudaEventRecord(up, st);
        cudaStreamWaitEvent(e->st2, up, 0);
        int rc = 0;
        for (size_t i = 0; i < calls.size() && rc == 0 && err == cudaSuccess; i++) {
            const Call &cl = calls[i];
            const bool tgt = cl.which == 0;
            rc = vxc_forward_prompt(tgt ? e->ts : e->ds, e->prefill_tok + cl.t0, e->prefill_meta + cl.m0,
                                    e->prefill_meta + cl.m0 + cl.G, cl.G, cl.T, tgt ? st : e->st2);
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
                               0.8f, 1, D.seq_id, D.apos, D.n_acc, D.next, st);
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
