// vxc_model.cu — device-resident Llama-family forward pass over many rows and
// sequences (reference src/model.c:391-628, scalar semantics).
//
// Per layer, for M = n_groups * rows_per_group rows:
//   h   = rmsnorm(x) * attn_norm                      (src/model.c:518, src/tensor.c:132-140)
//   qkv = [Wq;Wk;Wv] h                                 fused GEMV (src/model.c:522-536)
//   rope(q,k) at each row's position; k,v -> cache    (src/tensor.c:249-270, src/model.c:291-296)
//   att = softmax(q k^T / sqrt(hd)) v, causal          (src/model.c:299-338)
//   x  += Wo att                                       (out-of-place fix of src/model.c:543-546)
//   h   = rmsnorm(x) * ffn_norm
//   [g;u] = [Wg;Wu] h ; s = silu(g) ; f = |s|<0.01 ? 0 : s*u   (src/model.c:580-585)
//   x  += Wd f                                         (src/model.c:587-589)
// logits = Wout rmsnorm(x) * out_norm for the requested rows (src/model.c:598-615).
//
// RoPE uses a host-built (cos, sin) table computed exactly as the reference
// does (freq = 1/powf(theta, 2i/hd), val = pos*freq, cosf/sinf), and the
// rotation is written with explicitly rounded ops, so it matches the
// reference bit-for-bit.  The KV cache is fp32, head-major
// ([layer][slot][kv head][pos][hd]).
//
// Weights are Q4_0/Q8_0 (tensor-core GEMV, vxc_gemv_tc.cu) or K-quant
// (CUDA-core GEMV on the same activation image, vxc_kquant.cu).  Under tensor
// parallelism (vxc_tp.cu) a net holds this GPU's heads, FFN columns and
// vocabulary rows; the forward then all-reduces the output and down
// projections and gathers the logits, so every GPU ends with the same rows.
#include <climits>
#include "vxc_common.cuh"
#include "vxc_image.cuh"
#include "vxc_kquant.cuh"
#include "vxc_ptx.cuh"
#include "vxc_qmat.cuh"
#include "vxc_internal.h"

#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <atomic>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

struct vxc_layer_dev {
    float *attn_norm, *ffn_norm;   // never NULL (ones when the GGUF has none)
    vxc_qmat *wqkv, *wo, *wgu, *wd;
};

struct vxc_net {
    vxc_net_config cfg;
    int embd_type;
    uint8_t *embd;           // raw GGUF rows
    size_t embd_row_bytes;
    int embd_rows, embd_cols;
    float *out_norm;         // NULL when absent (no final norm, src/model.c:600)
    vxc_qmat *out;           // LM head
    vxc_layer_dev *layers;
    float2 *rope;            // [max_pos][hd/2]
    size_t weight_bytes;
    // tensor parallelism (tp == NULL: the whole model on this GPU)
    const vxc_tp *tp;
    int rank, world;
    int Hl, KHl, Fl, Vl;     // this GPU's q heads, kv heads, FFN columns, vocabulary rows
};

namespace cg = cooperative_groups;

#define VXC_MAX_CHUNKS 64   // row chunks of 64 per forward (max_rows <= 4096)

struct vxc_seqs {
    const vxc_net *net;
    int n_slots, max_ctx, max_rows;
    float *k, *v;            // [L][slot][kv head][pos][hd]
    float *x;                // [max_rows][E] residual stream
    float *qbuf;             // [max_rows][E] rotated queries
    uint8_t *img;            // activation images, one 64-row chunk per img_chunk bytes (GEMV), or
    size_t img_chunk;        // one slab of VXC_GEMM_SLAB rows per (VXC_GEMM_SLAB / 64) * img_chunk (GEMM)
    float *xs;               // [chunks * 64] image prescales
    float *part;             // GEMV partial sums, one slot per chunk
    size_t part_slot;        // floats per chunk slot
    float *xf;               // [VXC_SKINNY_MAX_M][K] fp32 rows for the CUDA-core GEMV of 1-2 rows
    float *attn_part;
    int attn_sl, attn_splits;
    uint64_t tmk[16], tmv[16];   // CUtensorMap of the K and V caches as [rows][hd] (copied to an aligned local per launch)
    float *ar;               // [max_rows][E] all-reduced projection output (tensor parallel)
    float *lg_local, *lg_all;   // local logits [rows][Vl], gathered [world][rows][Vl]
};

// queries per attention CTA: 8 when a kv head has <= 8 queries (verify rows x
// heads per kv head), else 16; the predicated query loops then carry little waste
#define ATTN_QC_MAX 16
#ifndef ATTN_SL_MIN
#define ATTN_SL_MIN 64  // shortest context split
#endif
#ifndef ATTN_MAX_SPLITS
#define ATTN_MAX_SPLITS 16   // context splits at most (before the minimum split lengths below)
#endif
#ifndef ATTN_SL_MIN_WIDE
#define ATTN_SL_MIN_WIDE 128  // ... for head dims >= 128 (fewer splits to merge)
#endif

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
__global__ void k_embed(const uint8_t *__restrict__ embd, int type, size_t row_bytes, int vocab, int E,
                        const int *__restrict__ tokens, float *__restrict__ x, unsigned int *err) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    const int tok = tokens[m];
    float *xr = x + (size_t)m * E;
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) vxc_flag_error(err, VXC_DERR_BAD_TOKEN);
        for (int i = threadIdx.x; i < E; i += blockDim.x) xr[i] = 0.0f;
        return;
    }
    const uint8_t *row = embd + (size_t)tok * row_bytes;
    if (type == 0) {
        const float *f = reinterpret_cast<const float *>(row);
        for (int i = threadIdx.x; i < E; i += blockDim.x) xr[i] = f[i];
        return;
    }
    if (type >= 10 && type <= 15) {   // K-quant rows of E / 256 super-blocks (src/model.c:462-496)
        const int bb = vxc_kq_block_bytes(type);
        for (int i = threadIdx.x; i < E; i += blockDim.x)
            xr[i] = vxc_kq_decode_any(type, row + (size_t)(i / VXC_QK_K) * bb, i % VXC_QK_K);
        return;
    }
    // one thread per element: block b = i/32 (src/quantize.c:578-591, :642-651)
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        int b = i >> 5, j = i & 31;
        if (type == 2) {
            const uint8_t *blk = row + (size_t)b * 18;
            float d = vxc_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
            uint8_t byte = blk[2 + (j >> 1)];
            int q = (j & 1) ? (byte >> 4) : (byte & 0x0F);
            xr[i] = (float)(q - 8) * d;
        } else {
            const uint8_t *blk = row + (size_t)b * 34;
            float d = vxc_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
            xr[i] = (float)(int8_t)blk[2 + j] * d;
        }
    }
}

__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    return t;
}

// Split-K partial sums of a GEMV output, read by its consumer.  Rows are in
// chunks of 64 (one GEMV launch each); chunk c holds ks slices of [Mc][R] at
// base + c * slot.  Slices are added in order, so results are deterministic.
struct Part {
    const float *base;
    size_t slot;
    int R, M, ks_full, ks_last;
    __device__ __forceinline__ float get(int m, int r) const {
        const int c = m >> 6, ml = m & 63;
        const int Mc = min(64, M - (c << 6));
        const int ks = (c == ((M - 1) >> 6)) ? ks_last : ks_full;
        const float *p = base + c * slot + (size_t)ml * R + r;
        float acc = p[0];
        for (int s = 1; s < ks; s++) acc += p[(size_t)s * Mc * R];
        return acc;
    }
};

__device__ __forceinline__ float block_max(float v, float *red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) t = fmaxf(t, red[i]);
    return t;
}

// RoPE of one head of row m (qkv = sum of the fused QKV GEMV's partials):
// blockIdx.x < H: q head -> qbuf; < H + KH: k head -> cache; else v head ->
// cache (head-major [slot][kv head][pos][hd]).  Thread = one (even, odd) pair.
__global__ void k_rope_kv(Part qkv, int T, const int *__restrict__ d_slot, const int *__restrict__ d_pos,
                          const float2 *__restrict__ rope, int max_pos, int H, int KH, int hd,
                          float *__restrict__ qbuf, float *__restrict__ kc, float *__restrict__ vc, int n_slots,
                          int max_ctx, unsigned int *err) {
    pdl_trigger();
    pdl_wait();
    const int head = blockIdx.x, m = blockIdx.y, p = threadIdx.x;
    const int g = m / T, t = m % T;
    const int slot = d_slot[g];
    const int pos = d_pos[g] + t;
    const int E = H * hd, kvd = KH * hd;
    if (pos < 0 || pos >= max_ctx || pos >= max_pos || slot < 0 || slot >= n_slots) {
        if (head == 0 && p == 0) vxc_flag_error(err, VXC_DERR_CTX_FULL);
        return;
    }
    if (2 * p >= hd) return;
    auto cache_row = [&](float *c, int kh) { return c + (((size_t)slot * KH + kh) * max_ctx + pos) * hd; };
    if (head >= H + KH) {
        const int vh = head - H - KH;
        float *dst = cache_row(vc, vh) + 2 * p;
        dst[0] = qkv.get(m, E + kvd + vh * hd + 2 * p);
        dst[1] = qkv.get(m, E + kvd + vh * hd + 2 * p + 1);
        return;
    }
    const float2 c = rope[(size_t)pos * (hd / 2) + p];
    const int col = head < H ? head * hd + 2 * p : E + (head - H) * hd + 2 * p;
    const float a = qkv.get(m, col), b = qkv.get(m, col + 1);
    // a*cr - b*ci ; a*ci + b*cr with the reference's separate roundings (src/tensor.c:262-266)
    const float r0 = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
    const float r1 = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
    float *dst = head < H ? qbuf + (size_t)m * E + col : cache_row(kc, head - H) + 2 * p;
    dst[0] = r0;
    dst[1] = r1;
}

// Decode/verify attention, split over the context (flash-decoding style).
// CTA = (group g, kv head, chunk of <= QC queries) x one split of SL
// positions.  The queries are the rows of group g times the q heads that
// share the kv head (GQA mapping kv_h = h*KH/H, src/model.c:303), so each K/V
// byte of the split is read from HBM once for all of them.
//
// The cache is head-major ([layer][slot][kv head][pos][hd]), so a split's K
// (and V) rows are consecutive rows of one 2-D tensor map [rows][hd].  Tiles
// of ATTN_T rows arrive by TMA (issued by thread 0) in an ATTN_NS-stage ring,
// the K tiles then the V tiles of the split, as hd/32 boxes of 32 floats x
// ATTN_T rows with the 128-byte swizzle (16-byte chunk c of row r stored at
// c ^ (r & 7)), which keeps both access patterns free of bank conflicts.
// Each of the 4 warps owns a quarter of the head dim (QW 16-byte chunks):
//  - scores: lane = position; the warp's partial dot product of every query
//    over its chunks, in order; the softmax pass adds the four partials in
//    warp order, scales, applies the causal mask and forms max and sum of
//    exp(s - max) of the split (one warp per query);
//  - P.V: lane = (row r of each group of RPW rows, chunk of the warp's
//    quarter); rows in order per lane, then the RPW row sums in order.
// So no tile is read twice from shared memory, the warps carry equal work,
// and each warp writes its own chunks of the split's record
// [m, l, -, -, o[hd]] (16-byte aligned) per query: max m, sum l of
// exp(s - m) and o = sum exp(s - m) v.  k_combine_image merges the splits.
// Every wait is bounded: on a timeout the error word gets
// VXC_DERR_TIMEOUT_TMA, the threads keep the CTA's barriers without
// computing, and thread 0 drains the copies in flight.
// Up to 8 queries per kv head the kernel is instantiated for exactly that
// many (no predicated query slots); beyond, in chunks of 16.
#define ATTN_T 32    // cache rows per ring stage
#ifndef ATTN_NS
#define ATTN_NS 2    // ring stages
#endif

// float4 index of chunk c of row r in a ring stage: [hd/32 boxes][ATTN_T rows][8 chunks, swizzled]
__device__ __forceinline__ int attn_chunk(int r, int c) { return (c >> 3) * (ATTN_T * 8) + r * 8 + ((c & 7) ^ (r & 7)); }

// 4 CTAs per SM (128 registers) up to 8 queries; the 16-query form (prompt chunks) keeps 3 so
// that its 16 accumulators per lane stay in registers
template <int HD, int QC>
__global__ void __launch_bounds__(128, QC > 8 ? 3 : 4)
    k_attn(const float *__restrict__ qbuf, int T, const int *__restrict__ d_slot, const int *__restrict__ d_pos,
           int H, int KH, const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, int row0,
           int n_slots, int max_ctx, int SL, int nqc, float *__restrict__ part, unsigned int *err) {
    constexpr int NC = HD / 4;                // float4 chunks per row
    constexpr int QW = NC / 4;                // chunks per warp
    constexpr int RPW = 32 / QW;              // V rows per warp instruction in P.V
    constexpr int SEG = HD / 32;              // boxes per tile
    constexpr int STG = ATTN_T * HD;          // floats per ring stage
    constexpr int PVU = QC > 8 ? 2 : 4;       // P.V rows in flight per lane
    static_assert(HD % 32 == 0 && HD <= 128 && ATTN_T == 32, "head dim / tile");
    extern __shared__ __align__(16) unsigned char sm_raw[];
    // the swizzled boxes need 1024-byte aligned stages
    float *ring = reinterpret_cast<float *>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);   // [ATTN_NS][STG]
    float *qs = ring + ATTN_NS * STG;          // [QC][HD]
    float *sc = qs + QC * HD;                  // [4][QC][SL + 1] partial scores; exp values in [0]
    __shared__ __align__(8) uint64_t full[ATTN_NS], qbar;
    __shared__ float qmax[QC], qsum[QC];
    __shared__ int abort_flag;
    const int G = H / KH, nq = T * G, E = H * HD;
    const int bx = blockIdx.x;
    const int qc = bx % nqc;
    const int kvh = (bx / nqc) % KH;
    const int g = bx / (nqc * KH);
    const int split = blockIdx.y, nsplit = gridDim.y;
    const int q0 = qc * QC;
    // up to 8 queries per kv head the host picks QC = that count, so the query loops are exact
    const int nql = QC <= 8 ? QC : min(QC, nq - q0);
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < ATTN_NS; s++) mbar_init(smem_u32(&full[s]), 1);
        mbar_init(smem_u32(&qbar), 1);
        abort_flag = 0;
        mbar_init_fence();
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    const int slot = d_slot[g];
    const int base = d_pos[g];
    const int p0 = split * SL;
    // exclusive end: causal bound of the group, clamped to the cache
    // (k_rope_kv flags positions outside it; a bad slot reads nothing)
    const int pend = (slot < 0 || slot >= n_slots || base < 0) ? 0 : min(min(p0 + SL, base + T), max_ctx);
    auto part_ptr = [&](int q) {
        return part + ((((size_t)g * KH + kvh) * (size_t)nq + q) * nsplit + split) * (HD + 4);
    };
    if (p0 >= pend) {
        if (tid < nql) {
            float *pp = part_ptr(q0 + tid);
            pp[0] = -INFINITY;
            pp[1] = 0.0f;
        }
        return;
    }
    const int npos = pend - p0;
    const int nt = (npos + ATTN_T - 1) / ATTN_T;
    const int hrow = row0 + (slot * KH + kvh) * max_ctx + p0;   // tensor-map row of the split's first position
    volatile int *abortp = &abort_flag;
    // tile i < nt: K tile i; i >= nt: V tile i - nt (whole boxes land: rows past the split are
    // read, or zero past the tensor)
    auto issue = [&](int i) {
        if (i < 2 * nt) {
            const int s = i % ATTN_NS, t = i < nt ? i : i - nt;
            const uint32_t bar = smem_u32(&full[s]);
            mbar_expect_tx(bar, (uint32_t)(STG * 4));
#pragma unroll
            for (int b = 0; b < SEG; b++)
                tma_load_2d(smem_u32(ring + (size_t)s * STG + b * (ATTN_T * 32)), i < nt ? &tmk : &tmv, b * 32,
                            hrow + t * ATTN_T, bar);
        }
    };
    if (tid == 0) {
        mbar_expect_tx(smem_u32(&qbar), (uint32_t)(nql * HD * 4));
        for (int ql = 0; ql < nql; ql++) {
            const int q = q0 + ql, t = q / G, h = kvh * G + q % G;
            bulk_g2s(smem_u32(qs + (size_t)ql * HD), qbuf + (size_t)(g * T + t) * E + (size_t)h * HD, HD * 4,
                     smem_u32(&qbar));
        }
        for (int i = 0; i < ATTN_NS - 1; i++) issue(i);
    }
    const float scale = 1.0f / sqrtf((float)HD);
    const int SLP = SL + 1;
    const int r = lane / QW, cc = w * QW + lane % QW;   // P.V lane: row r, chunk cc
    const float4 *qv4 = reinterpret_cast<const float4 *>(qs);
    float4 acc[QC];
#pragma unroll
    for (int jq = 0; jq < QC; jq++) acc[jq] = make_float4(0.f, 0.f, 0.f, 0.f);
    bool ok = mbar_wait(smem_u32(&qbar), 0, abortp, err, VXC_DERR_TIMEOUT_TMA);
    int issued = ATTN_NS - 1;
    for (int i = 0; i < 2 * nt; i++) {
        if (tid == 0 && !*abortp) {
            // the stage of tile i - 1 was released by the barrier that ended its iteration
            fence_proxy_async();
            issue(i + ATTN_NS - 1);
            issued = i + ATTN_NS;
        }
        const int s = i % ATTN_NS;
        if (ok) ok = mbar_wait(smem_u32(&full[s]), (i / ATTN_NS) & 1, abortp, err, VXC_DERR_TIMEOUT_TMA);
        const float4 *tile = reinterpret_cast<const float4 *>(ring + (size_t)s * STG);
        if (i == nt && ok) {
            // scores = ((w0 + w1) + w2) + w3, scaled and masked; softmax pieces of the split
            for (int ql = w; ql < nql; ql += 4) {
                float *row = sc + ql * SLP;
                const int lim = base + (q0 + ql) / G - p0;   // last visible position of the split
                float mx = -INFINITY;
                for (int p = lane; p < npos; p += 32) {
                    float v = row[p];
#pragma unroll
                    for (int ww = 1; ww < 4; ww++) v += row[(size_t)ww * QC * SLP + p];
                    v = p <= lim ? v * scale : -INFINITY;
                    row[p] = v;
                    mx = fmaxf(mx, v);
                }
                mx = warp_max(mx);
                float su = 0.0f;
                for (int p = lane; p < npos; p += 32) {
                    const float v = row[p];
                    const float e = (v == -INFINITY) ? 0.0f : expf(v - mx);
                    row[p] = e;
                    su += e;
                }
                su = warp_sum(su);
                if (lane == 0) {
                    qmax[ql] = mx;
                    qsum[ql] = su;
                }
            }
        }
        if (i == nt) __syncthreads();
        if (ok && i < nt) {
            // partial scores over this warp's chunks: lane = position p of the tile
            const int pl = i * ATTN_T + lane;
            if (pl < npos) {
                float a[QC];
#pragma unroll
                for (int jq = 0; jq < QC; jq++) a[jq] = 0.0f;
#pragma unroll 2
                for (int ci = 0; ci < QW; ci++) {
                    const int c = w * QW + ci;
                    const float4 kv = tile[attn_chunk(lane, c)];
#pragma unroll
                    for (int jq = 0; jq < QC; jq++) {
                        if (jq < nql) {
                            const float4 qv = qv4[jq * NC + c];
                            float x = a[jq];
                            x = fmaf(qv.x, kv.x, x);
                            x = fmaf(qv.y, kv.y, x);
                            x = fmaf(qv.z, kv.z, x);
                            x = fmaf(qv.w, kv.w, x);
                            a[jq] = x;
                        }
                    }
                }
                float *dst = sc + (size_t)w * QC * SLP + pl;
#pragma unroll
                for (int jq = 0; jq < QC; jq++)
                    if (jq < nql) dst[jq * SLP] = a[jq];
            }
        } else if (ok && r < RPW) {
            // P.V over this warp's chunks: lane = (row r, chunk cc)
            const int t0 = (i - nt) * ATTN_T, ntp = min(ATTN_T, npos - t0);
            const float *et = sc + t0;
#pragma unroll(PVU)
            for (int p = r; p < ntp; p += RPW) {
                const float4 vv = tile[attn_chunk(p, cc)];
#pragma unroll
                for (int jq = 0; jq < QC; jq++) {
                    if (jq < nql) {
                        const float e = et[jq * SLP + p];
                        acc[jq].x = fmaf(e, vv.x, acc[jq].x);
                        acc[jq].y = fmaf(e, vv.y, acc[jq].y);
                        acc[jq].z = fmaf(e, vv.z, acc[jq].z);
                        acc[jq].w = fmaf(e, vv.w, acc[jq].w);
                    }
                }
            }
        }
        __syncthreads();
    }
    // row sums in order (lanes of row 0 collect rows 1..RPW-1; every lane reads the others' sums
    // before it overwrites its own), then this warp's chunks of the records
#pragma unroll
    for (int jq = 0; jq < QC; jq++) {
        float4 t = acc[jq];
#pragma unroll
        for (int k = 1; k < RPW; k++) {
            t.x += __shfl_down_sync(0xffffffffu, acc[jq].x, k * QW);
            t.y += __shfl_down_sync(0xffffffffu, acc[jq].y, k * QW);
            t.z += __shfl_down_sync(0xffffffffu, acc[jq].z, k * QW);
            t.w += __shfl_down_sync(0xffffffffu, acc[jq].w, k * QW);
        }
        acc[jq] = t;
    }
    if (!*abortp) {
        if (r == 0) {
#pragma unroll
            for (int jq = 0; jq < QC; jq++)
                if (jq < nql) reinterpret_cast<float4 *>(part_ptr(q0 + jq) + 4)[cc] = acc[jq];
        }
        if (tid < nql) {
            float *pp = part_ptr(q0 + tid);
            pp[0] = qmax[tid];
            pp[1] = qsum[tid];
        }
    } else if (tid == 0) {
        // drain (bounded): the query rows and the tiles issued but not waited for
        for (int k = max(0, issued - ATTN_NS); k < issued && k < 2 * nt; k++) {
            const uint64_t t0 = vxc_globaltimer();
            while (!mbar_try(smem_u32(&full[k % ATTN_NS]), (k / ATTN_NS) & 1) && vxc_globaltimer() - t0 < 100000000ull) {}
        }
        const uint64_t t0 = vxc_globaltimer();
        while (!mbar_try(smem_u32(&qbar), 0) && vxc_globaltimer() - t0 < 100000000ull) {}
    }
}

// ---------------------------------------------------------------------------
// Row kernels on thread-block clusters.  A row of M (40 at batch 8 x 5) is
// far too little parallelism for one CTA per row, so each row is spread over
// a cluster of ROW_CL CTAs, each owning a column range (multiple of 8); the
// row-wide sum of squares and max|value| are combined through distributed
// shared memory in fixed rank order (deterministic, identical in every CTA).
// ---------------------------------------------------------------------------
#ifndef ROW_CL
#define ROW_CL 8
#endif
#ifndef ROW_THREADS
#define ROW_THREADS 256
#endif

// Sum (op 0) or max (op 1) of one value per CTA over the cluster; `slot` is
// this reduction's own shared word.  Ends with the values read, so the slot
// may not be rewritten before a later cluster.sync().
__device__ __forceinline__ float cluster_reduce(cg::cluster_group &cl, float v, float *slot, int op) {
    if (threadIdx.x == 0) *slot = v;
    cl.sync();
    float t = op ? 0.0f : 0.0f;
#pragma unroll
    for (int r = 0; r < ROW_CL; r++) {
        const float u = *cl.map_shared_rank(slot, r);
        t = op ? fmaxf(t, u) : t + u;
    }
    return t;
}

__device__ __forceinline__ void col_range(int K, int align, int *k0, int *k1) {
    const int c = blockIdx.x;
    int cw = (K + ROW_CL - 1) / ROW_CL;
    cw = (cw + align - 1) / align * align;
    *k0 = min(K, c * cw);
    *k1 = min(K, *k0 + cw);
}

// Image columns [k0, k1) of row m (vxc_qmat.cuh layout) in chunks of 2^csh
// rows: 64 for the GEMV, VXC_GEMM_SLAB for the GEMM (vxc_gemm_tc.cu).
template <class F>
__device__ __forceinline__ void image_cols(uint8_t *img, size_t chunk_bytes, int csh, int m, int M, int k0, int k1,
                                           float s, F val) {
    const int c = m >> csh, cr = 1 << csh, ml = m & (cr - 1);
    const int N = vxc_img_rows(min(cr, M - (c << csh)));
    uint8_t *base = img + c * chunk_bytes;
    for (int ch = k0 / 8 + threadIdx.x; ch < k1 / 8; ch += blockDim.x) {
        const int b = ch >> 2, cc = ch & 3;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = val(8 * ch + i);
        uint4 hi, lo;
        vxc_hilo8(v, s, hi, lo);
        uint8_t *chunk = base + (size_t)(b * 4 + cc) * 2 * N * 16;
        *reinterpret_cast<uint4 *>(chunk + (size_t)ml * 16) = hi;
        *reinterpret_cast<uint4 *>(chunk + (size_t)(N + ml) * 16) = lo;
    }
}

// The row kernels below write their output for the next GEMV either as its
// tensor-core image (img != NULL, with the row prescale xs) or, when that GEMV
// runs on the CUDA cores (1-2 rows), as fp32 rows xf[m][K] (img == NULL).

// Residual update and RMSNorm into the next GEMV's image:
//   x[src] += sum of the previous GEMV's partials (when add.base != NULL)
//   h = w * (x[src] * (1/sqrt(sum(x^2)/E + 1e-5)))        (src/tensor.c:132-140)
// Output row m (blockIdx.y) reads source row rows[m] (all rows when rows ==
// NULL); x is written back only when write_x.
__global__ void __launch_bounds__(ROW_THREADS) k_norm_image(float *__restrict__ x, Part add,
                                                              const float *__restrict__ w, int E,
                                                              const int *__restrict__ rows, int write_x, int M_out,
                                                              uint8_t *__restrict__ img, size_t chunk_bytes, int csh,
                                                              float *__restrict__ xs, float *__restrict__ xf) {
    extern __shared__ float v[];   // local columns
    __shared__ float red[32], slots[2];
    cg::cluster_group cl = cg::this_cluster();
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.y;
    const int src = rows ? rows[m] : m;
    int k0, k1;
    col_range(E, 8, &k0, &k1);
    float *xr = x + (size_t)src * E;
    float ss = 0.0f;
    for (int i = k0 + threadIdx.x; i < k1; i += blockDim.x) {
        float val = xr[i];
        if (add.base) val = __fadd_rn(val, add.get(src, i));
        if (write_x) xr[i] = val;
        v[i - k0] = val;
        ss = fmaf(val, val, ss);
    }
    ss = cluster_reduce(cl, block_sum(ss, red), &slots[0], 0);
    const float rms = sqrtf(ss / (float)E + 1e-5f);
    const float inv = 1.0f / rms;
    float mx = 0.0f;
    for (int i = k0 + threadIdx.x; i < k1; i += blockDim.x) {
        const float h = rms < 1e-10f ? 0.0f : __fmul_rn(w[i], __fmul_rn(v[i - k0], inv));
        v[i - k0] = h;
        if (!img) xf[(size_t)m * E + i] = h;
        mx = fmaxf(mx, fabsf(h));
    }
    if (img) {
        mx = cluster_reduce(cl, block_max(mx, red), &slots[1], 1);
        const float s = vxc_prescale(mx);
        if (blockIdx.x == 0 && threadIdx.x == 0) xs[m] = s;
        __syncthreads();
        image_cols(img, chunk_bytes, csh, m, M_out, k0, k1, s, [&](int k) { return v[k - k0]; });
    }
    cl.sync();   // peers have read this CTA's slots
}

// f = |silu(g)| < 0.01 ? 0 : silu(g) * u  (src/model.c:580-585, src/tensor.c:71-88, :277)
// from the fused gate/up GEMV's partials, then the image for the down GEMV.
__global__ void __launch_bounds__(ROW_THREADS) k_swiglu_image(Part gu, int F, int M, uint8_t *__restrict__ img,
                                                                size_t chunk_bytes, int csh, float *__restrict__ xs,
                                                                float *__restrict__ xf) {
    extern __shared__ float v[];
    __shared__ float red[32], slots[1];
    cg::cluster_group cl = cg::this_cluster();
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.y;
    int k0, k1;
    col_range(F, 8, &k0, &k1);
    float mx = 0.0f;
    for (int j = k0 + threadIdx.x; j < k1; j += blockDim.x) {
        const float g = gu.get(m, j), u = gu.get(m, F + j);
        const float sl = g / (1.0f + expf(-g));
        const float f = (fabsf(sl) < 0.01f) ? __fmul_rn(sl, 0.0f) : __fmul_rn(sl, u);
        v[j - k0] = f;
        if (!img) xf[(size_t)m * F + j] = f;
        mx = fmaxf(mx, fabsf(f));
    }
    if (img) {
        mx = cluster_reduce(cl, block_max(mx, red), &slots[0], 1);
        const float s = vxc_prescale(mx);
        if (blockIdx.x == 0 && threadIdx.x == 0) xs[m] = s;
        __syncthreads();
        image_cols(img, chunk_bytes, csh, m, M, k0, k1, s, [&](int k) { return v[k - k0]; });
    }
    cl.sync();
}

// Merge of the attention splits for the heads of row m owned by this CTA,
// then the image of the row for the attention-output GEMV:
//   out = (sum_s e^{m_s-M} o_s) / (sum_s e^{m_s-M} l_s + 1e-10)   (vx_softmax's +1e-10, src/tensor.c:168)
// One warp per head; lane s holds split s's weight e^{m_s-M}.
__global__ void __launch_bounds__(ROW_THREADS) k_combine_image(const float *__restrict__ part, int T, int H, int KH,
                                                                 int hd, int nsplit, int M, uint8_t *__restrict__ img,
                                                                 size_t chunk_bytes, int csh, float *__restrict__ xs,
                                                                 float *__restrict__ xf) {
    extern __shared__ float v[];
    __shared__ float red[32], slots[1];
    cg::cluster_group cl = cg::this_cluster();
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.y;
    const int g = m / T, t = m % T;
    const int G = H / KH, nq = T * G;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int rec = hd + 4;
    const int hpc = (H + ROW_CL - 1) / ROW_CL;
    const int h0 = min(H, blockIdx.x * hpc), h1 = min(H, h0 + hpc);
    // warps take (head, part of the head's columns): with fewer heads than warps, P warps share a head
    const int nh = h1 - h0;
    const int P = nh > 0 && nh < nw ? nw / nh : 1;
    float mx = 0.0f;
    for (int it = w; it < nh * P; it += nw) {
        const int h = h0 + it / P, cpart = it % P;
        const int kvh = h / G, q = t * G + (h % G);
        const float *pp = part + (((size_t)g * KH + kvh) * nq + q) * nsplit * rec;
        const float ms = lane < nsplit ? pp[(size_t)lane * rec] : -INFINITY;
        const float Mx = warp_max(ms);
        const float e = (ms == -INFINITY) ? 0.0f : expf(ms - Mx);
        const float Ls = warp_sum(lane < nsplit ? e * pp[(size_t)lane * rec + 1] : 0.0f);
        const float inv = 1.0f / (Ls + 1e-10f);
        // splits past the last one with positions hold no output; the others are read
        // unconditionally (a select, not a branch, drops the weightless ones), so the
        // loads of several splits are in flight together
        const unsigned live = __ballot_sync(0xffffffffu, lane < nsplit && e != 0.0f);
        const int ns = live ? 32 - __clz(live) : 0;
        for (int d = cpart * 32 + lane; d < hd; d += 32 * P) {
            float o = 0.0f;
#pragma unroll 8
            for (int sp = 0; sp < ns; sp++) {
                const float es = __shfl_sync(0xffffffffu, e, sp);
                const float v = pp[(size_t)sp * rec + 4 + d];
                o = fmaf(es, es != 0.0f ? v : 0.0f, o);
            }
            const float val = o * inv;
            v[(h - h0) * hd + d] = val;
            if (!img) xf[(size_t)m * H * hd + h * hd + d] = val;
            mx = fmaxf(mx, fabsf(val));
        }
    }
    if (img) {
        mx = cluster_reduce(cl, block_max(mx, red), &slots[0], 1);
        const float s = vxc_prescale(mx);
        if (blockIdx.x == 0 && threadIdx.x == 0) xs[m] = s;
        __syncthreads();
        image_cols(img, chunk_bytes, csh, m, M, h0 * hd, h1 * hd, s, [&](int k) { return v[k - h0 * hd]; });
    }
    cl.sync();
}

// logits[m][w*Vl + v] = gathered[w][m][v]: the vocabulary shards of the GPUs side by side
__global__ void k_vocab_gather(const float *__restrict__ all, int world, int n_rows, int Vl, float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const size_t V = (size_t)world * Vl, tot = (size_t)n_rows * V;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < tot; i += (size_t)gridDim.x * blockDim.x) {
        const size_t m = i / V, c = i % V, w = c / Vl, v = c % Vl;
        out[i] = all[(w * n_rows + m) * Vl + v];
    }
}

// Greedy token of one logits row, the reference's rule (src/main.c:307-311):
// scanning upward from max = -1e30, the first index whose value is strictly
// greater than every earlier one (NaN never wins; 0 when none exceeds -1e30).
__global__ void __launch_bounds__(1024) k_argmax_row(const float *__restrict__ lg, int V, int *__restrict__ tok) {
    pdl_trigger();
    pdl_wait();
    float best = -1e30f;
    int bi = INT_MAX;
    for (int j = threadIdx.x; j < V; j += blockDim.x) {   // ascending within a thread: > keeps the first
        const float v = lg[j];
        if (v > best) { best = v; bi = j; }
    }
    auto merge = [&]() {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
    };
    merge();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
    if (l == 0) { sv[w] = best; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        best = l < nw ? sv[l] : -1e30f;
        bi = l < nw ? si[l] : INT_MAX;
        merge();
        if (l == 0) *tok = bi == INT_MAX ? 0 : bi;
    }
}

// One step of the greedy loop after the argmax: the token just forwarded is
// now cached (pos + 1); the new token ends the loop if it is eos, else it is
// emitted.  st = {emitted, next position, done}.
__global__ void k_greedy_record(const int *__restrict__ tok, int *__restrict__ st, int *__restrict__ out, int eos,
                                int max_tokens) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0 || st[2]) return;
    st[1] += 1;
    const int t = *tok;
    if (t == eos) {
        st[2] = 1;
        return;
    }
    out[st[0]] = t;
    st[0] += 1;
    if (st[0] >= max_tokens) st[2] = 1;
}

// logits[m][r] = sum of the LM head's partials
__global__ void k_part_out(Part p, int n_rows, float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const size_t n = (size_t)n_rows * p.R;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = p.get((int)(i / p.R), (int)(i % p.R));
}


// ---------------------------------------------------------------------------
// host: upload
// ---------------------------------------------------------------------------
static size_t row_bytes_of(int type, int cols) {
    if (type == 2) return (size_t)(cols / 32) * 18;
    if (type == 8) return (size_t)(cols / 32) * 34;
    if (vxc_is_kquant(type)) return (size_t)(cols / VXC_QK_K) * vxc_kq_block_bytes(type);
    return (size_t)cols * 4;
}

static int upload_f32_or_ones(const vxc_tensor_view *t, int n, float **out) {
    std::vector<float> h(n, 1.0f);
    if (t && t->data && t->type == 0 && t->rows * t->cols >= n) memcpy(h.data(), t->data, (size_t)n * 4);
    VXC_CUDA_OK(cudaMalloc((void **)out, (size_t)n * 4));
    VXC_CUDA_OK(cudaMemcpy(*out, h.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
    return 0;
}

static size_t qmat_bytes(const vxc_qmat *w) { return w ? w->qs_bytes : 0; }

// Where a net's weights come from.  Tensors are numbered as in the GGUF files
// this library writes: 9 per layer (attn_norm, q, k, v, output, ffn_norm,
// gate, up, down), then token_embd (9L), output_norm (9L + 1) and the LM head
// (9L + 2).
struct NetSource {
    virtual ~NetSource() {}
    // GGUF type (0 F32, 2 Q4_0, 8 Q8_0), rows and cols; type -1 when absent
    virtual void shape(int ti, int *type, int *rows, int *cols) const = 0;
    // rows [r0, r0 + nr) x column blocks [b0, b0 + nb) of a Q4_0/Q8_0 tensor
    // as GGUF blocks in device memory (row-major); 0 or an error code
    virtual int blocks(int ti, int r0, int nr, int b0, int nb, uint8_t *dev) const = 0;
    // fp32 vector of n weights, NULL when absent (ones)
    virtual const vxc_tensor_view *f32(int ti) const = 0;
    // the token-embedding table in its GGUF type, rows x row_bytes at dev
    virtual int embedding(uint8_t *dev) const = 0;
};

static size_t block_bytes(int type) { return type == 2 ? 18 : 34; }

// Columns per quantisation block: 32 (Q4_0, Q8_0) or 256 (K-quant super-blocks).
static int block_cols(int type) { return vxc_is_kquant(type) ? VXC_QK_K : 32; }
static size_t unit_bytes(int type) { return vxc_is_kquant(type) ? (size_t)vxc_kq_block_bytes(type) : block_bytes(type); }

// Weights in host memory (GGUF views, e.g. an mmap'd file).
struct HostSource : NetSource {
    const vxc_tensor_view *tok, *onorm, *output;
    const vxc_layer_views *layers;
    int L;
    const vxc_tensor_view *view(int ti) const {
        if (ti == 9 * L) return tok;
        if (ti == 9 * L + 1) return onorm;
        if (ti == 9 * L + 2) return (output && output->data) ? output : tok;   // tied head, src/format.c:238
        const vxc_layer_views &v = layers[ti / 9];
        const vxc_tensor_view *all[9] = {&v.attn_norm, &v.wq, &v.wk, &v.wv, &v.wo, &v.ffn_norm, &v.wg, &v.wu, &v.wd};
        return all[ti % 9];
    }
    void shape(int ti, int *type, int *rows, int *cols) const override {
        const vxc_tensor_view *t = view(ti);
        *type = (t && t->data) ? t->type : -1;
        *rows = t ? t->rows : 0;
        *cols = t ? t->cols : 0;
    }
    int blocks(int ti, int r0, int nr, int b0, int nb, uint8_t *dev) const override {
        const vxc_tensor_view *t = view(ti);
        // b0, nb count 32-column blocks; a K-quant tensor moves whole super-blocks of 8 of them
        const int per = block_cols(t->type) / 32;
        b0 /= per;
        nb /= per;
        const size_t bb = unit_bytes(t->type), nbf = (size_t)t->cols / block_cols(t->type), rb = nbf * bb;
        const uint8_t *src = (const uint8_t *)t->data;
        cudaError_t e;
        if (b0 == 0 && (size_t)nb == nbf) {
            e = cudaMemcpy(dev, src + (size_t)r0 * rb, (size_t)nr * rb, cudaMemcpyHostToDevice);
        } else {
            // a column slice: gather the blocks of each row
            std::vector<uint8_t> buf((size_t)nr * nb * bb);
            for (int r = 0; r < nr; r++)
                memcpy(buf.data() + (size_t)r * nb * bb, src + (size_t)(r0 + r) * rb + (size_t)b0 * bb,
                       (size_t)nb * bb);
            e = cudaMemcpy(dev, buf.data(), buf.size(), cudaMemcpyHostToDevice);
        }
        if (e != cudaSuccess) { vxc_set_error("weight upload: %s", cudaGetErrorString(e)); return -3; }
        return 0;
    }
    const vxc_tensor_view *f32(int ti) const override {
        const vxc_tensor_view *t = view(ti);
        return (t && t->data) ? t : NULL;
    }
    int embedding(uint8_t *dev) const override {
        const size_t eb = row_bytes_of(tok->type, tok->cols) * tok->rows;
        if (cudaMemcpy(dev, tok->data, eb, cudaMemcpyHostToDevice) != cudaSuccess) {
            vxc_set_error("vxc_net_create: embedding upload failed");
            return -3;
        }
        return 0;
    }
};

// Weights generated on the device (vxc_synth.cu), as the GGUF writer would
// have written them for this configuration and seed.
struct SynthSource : NetSource {
    vxc_net_config c;
    int wtype;
    uint64_t seed;
    void shape(int ti, int *type, int *rows, int *cols) const override {
        const int L = c.n_layers, E = c.n_embd, kvd = c.n_kv_heads * c.n_head_dim, F = c.n_ff;
        if (ti >= 9 * L) {
            const int k = ti - 9 * L;
            *type = k == 1 ? 0 : wtype;
            *rows = k == 1 ? 1 : c.n_vocab;
            *cols = E;
            return;
        }
        const int k = ti % 9;
        static const int rows_kind[9] = {0, 1, 2, 2, 1, 0, 3, 3, 1};   // 0 norm, 1 E, 2 kvd, 3 F
        const int rk = rows_kind[k];
        *type = rk == 0 ? 0 : wtype;
        *rows = rk == 0 ? 1 : rk == 1 ? E : rk == 2 ? kvd : F;
        *cols = k == 8 ? F : E;
    }
    int blocks(int ti, int r0, int nr, int b0, int nb, uint8_t *dev) const override {
        int type, rows, cols;
        shape(ti, &type, &rows, &cols);
        return vxc_synth_blocks(type, seed, (uint32_t)ti, r0, nr, cols / 32, b0, nb, dev);
    }
    const vxc_tensor_view *f32(int) const override { return NULL; }
    int embedding(uint8_t *dev) const override {
        return vxc_synth_blocks(wtype, seed, (uint32_t)(9 * c.n_layers), 0, c.n_vocab, c.n_embd / 32, 0,
                                c.n_embd / 32, dev);
    }
};

// Slice of one tensor inside a fused matrix: rows [r0, r0 + nr), column
// blocks [b0, b0 + nb).
struct Piece {
    int ti, r0, nr, b0, nb;
};

// Concatenate pieces by rows (same type, same number of column blocks) and
// build one device matrix from them.
static int upload_pieces(const NetSource &src, const Piece *p, int n, vxc_qmat **out) {
    int type = -1, rows = 0;
    for (int i = 0; i < n; i++) {
        int t, r, c;
        src.shape(p[i].ti, &t, &r, &c);
        if (t < 0) { vxc_set_error("fused matrix parts differ in type/shape or are missing"); return -7; }
        if (t != 2 && t != 8 && !vxc_is_kquant(t)) {
            vxc_set_error("weight type %d not supported on the device (Q4_0, Q8_0, Q2_K..Q8_K)", t);
            return -7;
        }
        if (vxc_is_kquant(t) && (p[i].b0 % 8 || p[i].nb % 8)) {
            vxc_set_error("K-quant matrix slices must be whole 256-column super-blocks");
            return -7;
        }
        if ((i > 0 && p[i].nb != p[0].nb) || p[i].r0 + p[i].nr > r || p[i].b0 + p[i].nb > c / 32) {
            vxc_set_error("fused matrix parts differ in shape or are missing");
            return -7;
        }
        if (i > 0 && t != type) {
            // parts of different K-quant types (e.g. Q4_K query/key with Q6_K value rows) stay
            // separate matrices, stacked by rows
            if (!vxc_is_kquant(t) || !vxc_is_kquant(type)) {
                vxc_set_error("fused matrix parts differ in type (%d, %d)", type, t);
                return -7;
            }
            vxc_qmat *parts[3] = {NULL, NULL, NULL};
            int rc = n > 3 ? -4 : 0;
            for (int k = 0; k < n && rc == 0; k++) rc = upload_pieces(src, &p[k], 1, &parts[k]);
            if (rc == 0) rc = vxc_kquant_stack(parts, n, out);
            if (rc)
                for (int k = 0; k < n; k++) vxc_qmat_destroy(parts[k]);
            return rc;
        }
        type = t;
        rows += p[i].nr;
    }
    const size_t per = (size_t)block_cols(type) / 32, bb = unit_bytes(type);   // per staging unit
    uint8_t *staging = NULL;
    if (cudaMalloc((void **)&staging, (size_t)rows * (p[0].nb / per) * bb) != cudaSuccess) {
        vxc_set_error("vxc_net_create: out of device memory");
        return -3;
    }
    int rc = 0;
    size_t off = 0;
    for (int i = 0; i < n && rc == 0; i++) {
        rc = src.blocks(p[i].ti, p[i].r0, p[i].nr, p[i].b0, p[i].nb, staging + off);
        off += (size_t)p[i].nr * (p[i].nb / per) * bb;
    }
    if (rc == 0)
        rc = vxc_is_kquant(type) ? vxc_kquant_from_device(type, staging, rows, p[0].nb * 32, out)
                                 : vxc_qmat_from_device(type, staging, rows, p[0].nb * 32, out);
    cudaFree(staging);
    return rc;
}

extern "C" int vxc_tp_shard_ranges(const vxc_net_config *cfg, int rank, int world, int *out) {
    if (!cfg || !out || world < 1 || rank < 0 || rank >= world || cfg->n_heads % world ||
        cfg->n_kv_heads % world || cfg->n_ff % (32 * world) || cfg->n_vocab % world || cfg->n_head_dim % 32) {
        vxc_set_error("vxc_tp_shard_ranges: heads, FFN and vocab must split evenly over %d GPUs", world);
        return -4;
    }
    const int E = cfg->n_embd, hd = cfg->n_head_dim, F = cfg->n_ff;
    const int qh = cfg->n_heads / world * hd, kh = cfg->n_kv_heads / world * hd, fl = F / world;
    const int vl = cfg->n_vocab / world;
    const int r[8][4] = {
        {rank * qh, qh, 0, E},   // q: rows of this GPU's heads
        {rank * kh, kh, 0, E},   // k: rows of its kv heads
        {rank * kh, kh, 0, E},   // v
        {0, E, rank * qh, qh},   // output projection: the matching input columns
        {rank * fl, fl, 0, E},   // gate: rows of its FFN columns
        {rank * fl, fl, 0, E},   // up
        {0, E, rank * fl, fl},   // down: the matching input columns
        {rank * vl, vl, 0, E},   // LM head: its vocabulary rows
    };
    memcpy(out, r, sizeof r);
    return 0;
}

// Build a net from a weight source; tp != NULL keeps this GPU's shard only.
static int net_build(const vxc_net_config *cfg, const NetSource &src, const vxc_tp *tp, vxc_net **out) {
    int rc = vxc_require_device();
    if (rc) return rc;
    const int world = vxc_tp_world(tp), rank = vxc_tp_rank(tp);
    if (!cfg || !out || cfg->n_layers <= 0 || cfg->n_heads <= 0 || cfg->n_kv_heads <= 0 ||
        cfg->n_heads % cfg->n_kv_heads || cfg->n_head_dim % 32 || cfg->n_head_dim > 128 ||
        cfg->n_embd != cfg->n_heads * cfg->n_head_dim || cfg->n_embd % 32 || cfg->n_ff % 32) {
        vxc_set_error("vxc_net_create: unsupported configuration");
        return -4;
    }
    if (cfg->n_heads % world || cfg->n_kv_heads % world || cfg->n_ff % (32 * world) || cfg->n_vocab % world) {
        vxc_set_error("vxc_net_create: heads %d/%d, FFN %d and vocab %d must split evenly over %d GPUs",
                      cfg->n_heads, cfg->n_kv_heads, cfg->n_ff, cfg->n_vocab, world);
        return -4;
    }
    const int E = cfg->n_embd, L = cfg->n_layers, hd = cfg->n_head_dim;
    int et, er, ec;
    src.shape(9 * L, &et, &er, &ec);
    if (et < 0 || ec != E || er <= 0) {
        vxc_set_error("vxc_net_create: token embedding missing or not %d wide", E);
        return -4;
    }
    if (et != 0 && et != 2 && et != 8 && !(vxc_is_kquant(et) && E % VXC_QK_K == 0)) {
        vxc_set_error("vxc_net_create: token embedding type %d (width %d) not supported", et, E);
        return -7;
    }
    vxc_net *n = (vxc_net *)calloc(1, sizeof(vxc_net));
    n->cfg = *cfg;
    n->tp = tp;
    n->rank = rank;
    n->world = world;
    n->Hl = cfg->n_heads / world;
    n->KHl = cfg->n_kv_heads / world;
    n->Fl = cfg->n_ff / world;
    n->Vl = cfg->n_vocab / world;
    // embedding rows (raw GGUF, every GPU)
    n->embd_type = et;
    n->embd_rows = er;
    n->embd_cols = ec;
    n->embd_row_bytes = row_bytes_of(et, ec);
    if (cudaMalloc((void **)&n->embd, n->embd_row_bytes * er) != cudaSuccess) {
        vxc_set_error("vxc_net_create: embedding upload failed");
        vxc_net_destroy(n);
        return -3;
    }
    if ((rc = src.embedding(n->embd))) { vxc_net_destroy(n); return rc; }
    {
        int t, r, c;
        src.shape(9 * L + 1, &t, &r, &c);
        if (t >= 0 && (rc = upload_f32_or_ones(src.f32(9 * L + 1), E, &n->out_norm))) {
            vxc_net_destroy(n);
            return rc;
        }
    }
    {
        // tensor parallel: this GPU's vocabulary rows of the LM head
        int t, r, c, sr[8][4];
        src.shape(9 * L + 2, &t, &r, &c);
        Piece p = {9 * L + 2, 0, r, 0, c / 32};
        if (world > 1) {
            vxc_tp_shard_ranges(cfg, rank, world, &sr[0][0]);
            p.r0 = sr[7][0];
            p.nr = sr[7][1];
        }
        if ((rc = upload_pieces(src, &p, 1, &n->out))) { vxc_net_destroy(n); return rc; }
    }
    n->layers = (vxc_layer_dev *)calloc((size_t)L, sizeof(vxc_layer_dev));
    size_t wb = qmat_bytes(n->out) + (size_t)E * 4;
    for (int l = 0; l < L; l++) {
        vxc_layer_dev *d = &n->layers[l];
        const int t0 = 9 * l;
        if ((rc = upload_f32_or_ones(src.f32(t0 + 0), E, &d->attn_norm)) ||
            (rc = upload_f32_or_ones(src.f32(t0 + 5), E, &d->ffn_norm))) { vxc_net_destroy(n); return rc; }
        int ty[9], rw[9], cl[9];
        for (int k = 1; k < 9; k++) src.shape(t0 + k, &ty[k], &rw[k], &cl[k]);
        // whole tensors on one GPU; tensor parallel (Megatron-style): q/k/v rows of this GPU's
        // heads and gate/up rows of its FFN columns (column-parallel); output and down
        // projections keep every row but only the matching input columns (row-parallel,
        // summed over the GPUs afterwards)
        Piece qkv[3] = {{t0 + 1, 0, rw[1], 0, cl[1] / 32}, {t0 + 2, 0, rw[2], 0, cl[2] / 32},
                        {t0 + 3, 0, rw[3], 0, cl[3] / 32}};
        Piece o = {t0 + 4, 0, rw[4], 0, cl[4] / 32};
        Piece gu[2] = {{t0 + 6, 0, rw[6], 0, cl[6] / 32}, {t0 + 7, 0, rw[7], 0, cl[7] / 32}};
        Piece dn = {t0 + 8, 0, rw[8], 0, cl[8] / 32};
        if (world > 1) {
            const int kvd = cfg->n_kv_heads * hd, F = cfg->n_ff;
            const bool ok = rw[1] == E && cl[1] == E && rw[2] == kvd && cl[2] == E && rw[3] == kvd && cl[3] == E &&
                            rw[4] == E && cl[4] == E && rw[6] == F && cl[6] == E && rw[7] == F && cl[7] == E &&
                            rw[8] == E && cl[8] == F;
            bool present = true;
            for (int k = 1; k < 9; k++)
                if (k != 5 && ty[k] < 0) present = false;
            if (!present || !ok) {
                vxc_set_error("vxc_net_create: layer %d lacks a projection the tensor-parallel split needs "
                              "or has an unexpected shape", l);
                vxc_net_destroy(n);
                return -7;
            }
            int sr[8][4];
            vxc_tp_shard_ranges(cfg, rank, world, &sr[0][0]);
            auto piece = [&](int ti, const int *g) { return Piece{ti, g[0], g[1], g[2] / 32, g[3] / 32}; };
            qkv[0] = piece(t0 + 1, sr[0]);
            qkv[1] = piece(t0 + 2, sr[1]);
            qkv[2] = piece(t0 + 3, sr[2]);
            o = piece(t0 + 4, sr[3]);
            gu[0] = piece(t0 + 6, sr[4]);
            gu[1] = piece(t0 + 7, sr[5]);
            dn = piece(t0 + 8, sr[6]);
        }
        if ((rc = upload_pieces(src, qkv, 3, &d->wqkv)) || (rc = upload_pieces(src, &o, 1, &d->wo)) ||
            (rc = upload_pieces(src, gu, 2, &d->wgu)) || (rc = upload_pieces(src, &dn, 1, &d->wd))) {
            vxc_net_destroy(n);
            return rc;
        }
        wb += qmat_bytes(d->wqkv) + qmat_bytes(d->wo) + qmat_bytes(d->wgu) + qmat_bytes(d->wd) + 2ull * E * 4;
    }
    n->weight_bytes = wb;
    // RoPE table exactly as src/tensor.c:180-187 computes it per call
    const int np = hd / 2, P = cfg->max_pos > 0 ? cfg->max_pos : 4096;
    n->cfg.max_pos = P;
    std::vector<float2> tab((size_t)P * np);
    std::vector<float> freq(np);
    for (int i = 0; i < np; i++) freq[i] = 1.0f / powf(cfg->rope_theta, (float)(i * 2) / hd);
    for (int p = 0; p < P; p++)
        for (int i = 0; i < np; i++) {
            float val = p * freq[i];
            tab[(size_t)p * np + i] = make_float2(cosf(val), sinf(val));
        }
    if (cudaMalloc((void **)&n->rope, tab.size() * sizeof(float2)) != cudaSuccess ||
        cudaMemcpy(n->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess) {
        vxc_set_error("vxc_net_create: rope table upload failed");
        vxc_net_destroy(n);
        return -3;
    }
    *out = n;
    return 0;
}

extern "C" int vxc_net_create(const vxc_net_config *cfg, const vxc_tensor_view *tok_embd,
                              const vxc_tensor_view *out_norm, const vxc_tensor_view *output,
                              const vxc_layer_views *layers, vxc_net **out) {
    return vxc_net_create_tp(cfg, tok_embd, out_norm, output, layers, NULL, out);
}

extern "C" int vxc_net_create_tp(const vxc_net_config *cfg, const vxc_tensor_view *tok_embd,
                                 const vxc_tensor_view *out_norm, const vxc_tensor_view *output,
                                 const vxc_layer_views *layers, const vxc_tp *tp, vxc_net **out) {
    if (!cfg || !tok_embd || !tok_embd->data || !layers || !out) {
        vxc_set_error("vxc_net_create: unsupported configuration");
        return -4;
    }
    HostSource src;
    src.tok = tok_embd;
    src.onorm = out_norm;
    src.output = output;
    src.layers = layers;
    src.L = cfg->n_layers;
    return net_build(cfg, src, tp, out);
}

extern "C" int vxc_net_create_synth(const vxc_net_config *cfg, int wtype, uint64_t seed, const vxc_tp *tp,
                                    vxc_net **out) {
    if (!cfg || !out || (wtype != 2 && wtype != 8)) {
        vxc_set_error("vxc_net_create_synth: bad arguments");
        return -4;
    }
    SynthSource src;
    src.c = *cfg;
    src.wtype = wtype;
    src.seed = seed;
    return net_build(cfg, src, tp, out);
}

int vxc_net_world(const vxc_net *n) { return n ? n->world : 1; }

extern "C" void vxc_net_destroy(vxc_net *n) {
    if (!n) return;
    if (n->embd) cudaFree(n->embd);
    if (n->out_norm) cudaFree(n->out_norm);
    vxc_qmat_destroy(n->out);
    if (n->layers) {
        for (int l = 0; l < n->cfg.n_layers; l++) {
            vxc_layer_dev *d = &n->layers[l];
            if (d->attn_norm) cudaFree(d->attn_norm);
            if (d->ffn_norm) cudaFree(d->ffn_norm);
            vxc_qmat_destroy(d->wqkv);
            vxc_qmat_destroy(d->wo);
            vxc_qmat_destroy(d->wgu);
            vxc_qmat_destroy(d->wd);
        }
        free(n->layers);
    }
    if (n->rope) cudaFree(n->rope);
    free(n);
}

extern "C" int vxc_net_config_get(const vxc_net *n, vxc_net_config *cfg) {
    if (!n || !cfg) return -4;
    *cfg = n->cfg;
    return 0;
}

extern "C" size_t vxc_net_weight_bytes(const vxc_net *n) { return n ? n->weight_bytes : 0; }

// ---------------------------------------------------------------------------
// host: sequences + forward
// ---------------------------------------------------------------------------
// Dynamic shared memory of k_attn: ring, query rows, four partial-score rows
// per query (+ alignment of the ring).
static size_t attn_smem(int hd, int SL, int qc) {
    return ((size_t)ATTN_NS * ATTN_T * hd + (size_t)qc * hd + (size_t)4 * qc * (SL + 1)) * sizeof(float) + 1024;
}

static int attn_qc(int nq) { return nq <= 8 ? nq : 16; }

// cuTensorMapEncodeTiled through the runtime's driver entry point table (the
// library links only the static runtime, not libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
    static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
    PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_acquire);
    if (!f) {
        void *p = NULL;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p) {
            cudaGetLastError();
            return NULL;
        }
        f = (PFN_cuTensorMapEncodeTiled_v12000)p;
        fn.store(f, std::memory_order_release);
    }
    return f;
}

// A KV cache as the 2-D tensor [rows][hd] of fp32, read in boxes of 32 floats
// x ATTN_T rows with the 128-byte swizzle (k_attn's ring layout).
static bool attn_tmap(float *base, int hd, uint64_t rows, uint64_t out[16]) {
    PFN_cuTensorMapEncodeTiled_v12000 f = tmap_encode_fn();
    if (!f) return false;
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)hd * sizeof(float)};
    const cuuint32_t box[2] = {32, ATTN_T};
    const cuuint32_t es[2] = {1, 1};
    if (f(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return false;
    static_assert(sizeof(CUtensorMap) == 16 * sizeof(uint64_t), "tensor map size");
    memcpy(out, &m, sizeof m);
    return true;
}

typedef void (*attn_kernel_t)(const float *, int, const int *, const int *, int, int, const CUtensorMap,
                              const CUtensorMap, int, int, int, int, int, float *, unsigned int *);

#define ATTN_K_QC(HD)                  \
    case 1: return k_attn<HD, 1>;      \
    case 2: return k_attn<HD, 2>;      \
    case 3: return k_attn<HD, 3>;      \
    case 4: return k_attn<HD, 4>;      \
    case 5: return k_attn<HD, 5>;      \
    case 6: return k_attn<HD, 6>;      \
    case 7: return k_attn<HD, 7>;      \
    case 8: return k_attn<HD, 8>;      \
    case 16: return k_attn<HD, 16>;    \
    default: return NULL;
static attn_kernel_t attn_kernel(int hd, int qc) {
    switch (hd) {
        case 32: switch (qc) { ATTN_K_QC(32) }
        case 64: switch (qc) { ATTN_K_QC(64) }
        case 96: switch (qc) { ATTN_K_QC(96) }
        case 128: switch (qc) { ATTN_K_QC(128) }
        default: return NULL;
    }
}
#undef ATTN_K_QC

// Kernel launch with programmatic dependent launch: the kernel may start while
// its predecessor finishes; every kernel of the forward calls
// griddepcontrol.wait before touching data.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, ((KArgs)args)...);
    vxc_count_launches(1);
    return e;
}

// Same with a cluster of `clx` CTAs along x (row kernels).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_cluster(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      int clx, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = clx;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, ((KArgs)args)...);
    vxc_count_launches(1);
    return e;
}

// Largest partial-sum slot (floats) any GEMV of the net needs for a chunk of <= 64 rows.
static size_t part_slot_floats(const vxc_net *n) {
    size_t best = 0;
    auto consider = [&](const vxc_qmat *w) {
        if (vxc_is_kquant(w->type) || w->type == VXC_QMAT_STACK) {   // one slice [64][R]
            if ((size_t)64 * w->rows > best) best = (size_t)64 * w->rows;
            return;
        }
        for (int m = 1; m <= 64; m++) {
            VxcGemvPlan p;
            if (vxc_gemv_plan(w, m, &p)) {
                size_t f = (size_t)p.ks * m * w->rows;
                if (f > best) best = f;
            }
        }
        if (vxc_gemm_ok(w)) {   // the GEMM's K-slices of a 64-row chunk
            const size_t f = (size_t)vxc_gemm_slices(w) * 64 * w->rows;
            if (f > best) best = f;
        }
        for (int m = 1; m <= VXC_SKINNY_MAX_M; m++)   // the CUDA-core GEMV of 1-2 rows
            if (vxc_skinny_ok(w, m)) {
                const size_t f = (size_t)vxc_skinny_slices(w) * m * w->rows;
                if (f > best) best = f;
            }
    };
    for (int l = 0; l < n->cfg.n_layers; l++) {
        consider(n->layers[l].wqkv);
        consider(n->layers[l].wo);
        consider(n->layers[l].wgu);
        consider(n->layers[l].wd);
    }
    consider(n->out);
    return (best + 63) & ~(size_t)63;
}

extern "C" int vxc_seqs_create(const vxc_net *net, int n_slots, int max_ctx, int max_rows, vxc_seqs **out) {
    if (!net || !out || n_slots <= 0 || max_ctx <= 0 || max_rows <= 0) { vxc_set_error("vxc_seqs_create: bad args"); return -4; }
    int rc = vxc_require_device();
    if (rc) return rc;
    const vxc_net_config &c = net->cfg;
    if (max_ctx > c.max_pos) { vxc_set_error("vxc_seqs_create: max_ctx %d > rope table %d", max_ctx, c.max_pos); return -4; }
    if (max_rows > 64 * VXC_MAX_CHUNKS) { vxc_set_error("vxc_seqs_create: max_rows %d > %d", max_rows, 64 * VXC_MAX_CHUNKS); return -4; }
    vxc_seqs *s = (vxc_seqs *)calloc(1, sizeof(vxc_seqs));
    s->net = net;
    s->n_slots = n_slots;
    s->max_ctx = max_ctx;
    s->max_rows = max_rows;
    // this GPU's share under tensor parallelism (everything when net->tp == NULL)
    const int E = c.n_embd, kvd = net->KHl * c.n_head_dim, F = net->Fl, hd = c.n_head_dim;
    const int nch = (max_rows + 63) / 64;
    size_t kvn = (size_t)c.n_layers * n_slots * max_ctx * kvd;
    // attention split length: at most 16 splits of >= ATTN_SL_MIN positions (whole
    // tiles).  Short splits and a 2-stage ring keep ~5 CTAs per SM resident, which
    // measured faster on B200 than deeper rings (the kernel is latency-bound per CTA).
    int SL = (max_ctx + ATTN_MAX_SPLITS - 1) / ATTN_MAX_SPLITS;
    SL = ((SL + ATTN_T - 1) / ATTN_T) * ATTN_T;
    const int sl_min = hd >= 128 ? ATTN_SL_MIN_WIDE : ATTN_SL_MIN;
    if (SL < sl_min) SL = sl_min;
    s->attn_sl = SL;
    s->attn_splits = (max_ctx + SL - 1) / SL;
    size_t part = (size_t)max_rows * net->Hl * s->attn_splits * (hd + 4);
    s->img_chunk = (size_t)(E > F ? E : F) / 32 * vxc_img_block_bytes(64);
    s->part_slot = part_slot_floats(net);
    cudaError_t e = cudaSuccess;
#define ALLOC(p, n) if (e == cudaSuccess) e = cudaMalloc((void **)&(p), (n))
    ALLOC(s->k, kvn * 4);
    ALLOC(s->v, kvn * 4);
    ALLOC(s->x, (size_t)max_rows * E * 4);
    ALLOC(s->qbuf, (size_t)max_rows * E * 4);
    ALLOC(s->img, (size_t)nch * s->img_chunk);
    ALLOC(s->xs, (size_t)nch * 64 * 4);
    ALLOC(s->part, (size_t)nch * s->part_slot * 4);
    {
        size_t kmax = (size_t)(E > F ? E : F);
        if ((size_t)net->Hl * hd > kmax) kmax = (size_t)net->Hl * hd;
        ALLOC(s->xf, (size_t)VXC_SKINNY_MAX_M * kmax * 4);
    }
    ALLOC(s->attn_part, part * 4);
    if (net->tp) {
        ALLOC(s->ar, (size_t)max_rows * E * 4);
        ALLOC(s->lg_local, (size_t)max_rows * net->Vl * 4);
        ALLOC(s->lg_all, (size_t)net->world * max_rows * net->Vl * 4);
    }
#undef ALLOC
    if (e == cudaSuccess) e = cudaMemset(s->k, 0, kvn * 4);
    if (e == cudaSuccess) e = cudaMemset(s->v, 0, kvn * 4);
    if (e == cudaSuccess) e = cudaMemset(s->img, 0, (size_t)nch * s->img_chunk);
    if (e == cudaSuccess && !attn_kernel(hd, 16)) {
        vxc_set_error("vxc_seqs_create: head dim %d not supported (32, 64, 96 or 128)", hd);
        vxc_seqs_destroy(s);
        return -7;
    }
    if (e == cudaSuccess && attn_smem(hd, SL, ATTN_QC_MAX) > 227 * 1024) {
        vxc_set_error("vxc_seqs_create: context %d too long for the attention split", max_ctx);
        vxc_seqs_destroy(s);
        return -4;
    }
    // the attention kernel addresses cache rows with 32-bit tensor-map coordinates
    const uint64_t kv_rows = (uint64_t)c.n_layers * n_slots * net->KHl * max_ctx;
    if (e == cudaSuccess && (kv_rows + ATTN_T >= (1ull << 31) || !attn_tmap(s->k, hd, kv_rows, s->tmk) ||
                             !attn_tmap(s->v, hd, kv_rows, s->tmv))) {
        vxc_set_error("vxc_seqs_create: no tensor map for a KV cache of %llu rows of %d", (unsigned long long)kv_rows, hd);
        vxc_seqs_destroy(s);
        return -4;
    }
    if (ROW_CL > 8) {   // clusters above the portable size of 8 must be allowed per kernel
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_norm_image, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_swiglu_image, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_combine_image, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    }
    // The attribute is per kernel (and device), shared by every sequence set of
    // the process, so it is only ever raised: a set with a shorter context
    // must not shrink it under one with a longer context.
    static const int attn_qcs[] = {1, 2, 3, 4, 5, 6, 7, 8, 16};
    for (int qc : attn_qcs) {
        if (e != cudaSuccess) break;
        cudaFuncAttributes fa;
        const int need = (int)attn_smem(hd, SL, qc);
        e = cudaFuncGetAttributes(&fa, attn_kernel(hd, qc));
        if (e == cudaSuccess && fa.maxDynamicSharedSizeBytes < need)
            e = cudaFuncSetAttribute(attn_kernel(hd, qc), cudaFuncAttributeMaxDynamicSharedMemorySize, need);
    }
    if (e != cudaSuccess) {
        vxc_set_error("vxc_seqs_create: %s", cudaGetErrorString(e));
        vxc_seqs_destroy(s);
        return -3;
    }
    *out = s;
    return 0;
}

extern "C" void vxc_seqs_destroy(vxc_seqs *s) {
    if (!s) return;
    void *ptrs[] = {s->k, s->v, s->x, s->qbuf, s->img, s->xs, s->part, s->xf, s->attn_part, s->ar, s->lg_local,
                    s->lg_all};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    free(s);
}

static inline unsigned nblk(size_t n, int t) { return (unsigned)((n + t - 1) / t); }

// ---- optional per-stage device timing of vxc_forward (measurement aid) ----
static bool g_prof = false;
struct ProfEv {
    int stage;
    cudaEvent_t a, b;
};
static std::vector<ProfEv> g_prof_ev;

// Start / end of one timed stage on `st` (no-ops unless enabled, and while
// the stream is being captured into a graph).
static cudaEvent_t prof_begin(cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (!g_prof || cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return NULL;
    cudaEvent_t a = NULL;
    if (cudaEventCreate(&a) != cudaSuccess) return NULL;
    cudaEventRecord(a, st);
    return a;
}

static void prof_end(int stage, cudaEvent_t a, cudaStream_t st) {
    if (!a) return;
    cudaEvent_t b;
    if (cudaEventCreate(&b) != cudaSuccess) {
        cudaEventDestroy(a);
        return;
    }
    cudaEventRecord(b, st);
    g_prof_ev.push_back({stage, a, b});
}

extern "C" void vxc_profile_enable(int on) { g_prof = on != 0; }

extern "C" int vxc_profile_read(double *ms, int n) {
    if (ms)
        for (int i = 0; i < n; i++) ms[i] = 0.0;
    for (const ProfEv &e : g_prof_ev) {
        float t = 0.0f;
        cudaEventSynchronize(e.b);
        if (ms && e.stage < n && cudaEventElapsedTime(&t, e.a, e.b) == cudaSuccess) ms[e.stage] += t;
        cudaEventDestroy(e.a);
        cudaEventDestroy(e.b);
    }
    g_prof_ev.clear();
    return VXC_N_STAGES;
}

// Whether the GEMV of w over M rows runs on the CUDA cores from the fp32 rows
// s->xf (1-2 rows of a Q4_0 / Q8_0 matrix) rather than from the image.
static bool skinny(const vxc_qmat *w, int M) { return vxc_skinny_ok(w, M) != 0; }

// How a matrix multiplies M rows in a forward whose GEMM threshold is
// gemm_min: the tensor-core GEMM (one launch for all rows, image in slabs),
// the CUDA-core GEMV (1-2 rows, fp32 rows in s->xf), or the tensor-core GEMV
// (64-row chunks).  The producer of the rows writes the operand that mode reads.
enum GemvMode { GM_GEMV = 0, GM_SKINNY = 1, GM_GEMM = 2 };
static GemvMode gemv_mode(const vxc_qmat *w, int M, int gemm_min) {
    if (M >= gemm_min && vxc_gemm_ok(w)) return GM_GEMM;
    return skinny(w, M) ? GM_SKINNY : GM_GEMV;
}

// GEMM over all M rows, or GEMV over M rows in chunks of 64 (image chunks ->
// partial slots), or on the CUDA cores from s->xf; returns the Part view of
// its output.
static int gemv_rows(vxc_seqs *s, const vxc_qmat *w, int M, Part *out, cudaStream_t st, int gemm_min) {
    Part p;
    p.base = s->part;
    p.slot = s->part_slot;
    p.R = w->rows;
    p.M = M;
    p.ks_full = p.ks_last = 1;
    const GemvMode mode = gemv_mode(w, M, gemm_min);
    if (mode == GM_GEMM) {
        const int ks = vxc_gemm_slices(w);
        if (s->part_slot < (size_t)ks * 64 * w->rows) {
            vxc_set_error("vxc_forward: partial slot too small");
            return -4;
        }
        if (int rc = vxc_gemm_run(w, s->img, (VXC_GEMM_SLAB / 64) * s->img_chunk, s->xs, M, s->part, s->part_slot,
                                  0, st))
            return rc;
        p.ks_full = p.ks_last = ks;
        *out = p;
        return 0;
    }
    if (mode == GM_SKINNY) {
        const int ks = vxc_skinny_slices(w);
        if ((size_t)ks * M * w->rows > s->part_slot) {
            vxc_set_error("vxc_forward: partial slot too small");
            return -4;
        }
        if (int rc = vxc_skinny_run(w, s->xf, w->cols, M, s->part, st)) return rc;
        p.ks_full = p.ks_last = ks;
        *out = p;
        return 0;
    }
    if (vxc_is_kquant(w->type) || w->type == VXC_QMAT_STACK) {   // CUDA-core K-quant GEMV, one slice
        for (int c = 0; c * 64 < M; c++) {
            const int Mc = M - c * 64 < 64 ? M - c * 64 : 64;
            int rc = vxc_kquant_gemv_image(w, s->img + c * s->img_chunk, vxc_img_rows(Mc), s->xs + c * 64, Mc,
                                           s->part + c * s->part_slot, st);
            if (rc) return rc;
        }
        *out = p;
        return 0;
    }
    for (int c = 0; c * 64 < M; c++) {
        const int Mc = M - c * 64 < 64 ? M - c * 64 : 64;
        VxcGemvPlan pl;
        if (!vxc_gemv_plan(w, Mc, &pl)) {
            vxc_set_error("vxc_forward: no GEMV plan for %d x %d", w->rows, w->cols);
            return -7;
        }
        if ((size_t)pl.ks * Mc * w->rows > s->part_slot) {
            vxc_set_error("vxc_forward: partial slot too small");
            return -4;
        }
        int rc = vxc_gemv_run(w, s->img + c * s->img_chunk, s->xs + c * 64, Mc, s->part + c * s->part_slot, pl, st);
        if (rc) return rc;
        if (Mc == 64) p.ks_full = pl.ks;
        p.ks_last = pl.ks;
    }
    *out = p;
    return 0;
}

// The forward of vxc_forward; matrices multiply M >= gemm_min rows on the GEMM.
static int forward_impl(vxc_seqs *s, const int *d_tokens, const int *d_slot, const int *d_pos, int n_groups,
                        int rows_per_group, const int *d_logit_rows, int n_logit_rows, float *d_logits,
                        void *stream, int gemm_min) {
    if (!s || !d_tokens || !d_slot || !d_pos || n_groups <= 0 || rows_per_group <= 0) {
        vxc_set_error("vxc_forward: bad arguments");
        return -4;
    }
    const int M = n_groups * rows_per_group, T = rows_per_group;
    if (M > s->max_rows || n_logit_rows > s->max_rows || (n_logit_rows > 0 && (!d_logit_rows || !d_logits))) {
        vxc_set_error("vxc_forward: %d rows exceed max_rows %d", M, s->max_rows);
        return -4;
    }
    const vxc_net *n = s->net;
    const vxc_net_config &c = n->cfg;
    // heads, kv heads and FFN columns of this GPU (all of them without tensor parallelism)
    const int E = c.n_embd, H = n->Hl, KH = n->KHl, hd = c.n_head_dim, F = n->Fl;
    const int kvd = KH * hd;
    if (n_logit_rows > 0 && !n->out_norm) {
        vxc_set_error("vxc_forward: models without output_norm are not supported");
        return -7;
    }
    if (n_logit_rows > 0 && n->out->rows != n->Vl) {
        vxc_set_error("vxc_forward: LM head rows %d != vocab %d not supported", n->out->rows, c.n_vocab);
        return -7;
    }
    cudaStream_t st = (cudaStream_t)stream;
    unsigned int *err = vxc_device_error_ptr();
    int rc;
    cudaError_t e;
    // tensor parallel: sum a row-parallel projection's output over the GPUs
    // (its split-K partials first summed here into s->ar), then read it as one slice
    // 0, or the error code with the message set
    auto tp_sum = [&](Part &p) -> int {
        const size_t tot = (size_t)M * E;
        cudaError_t er = launch_pdl(k_part_out, dim3(nblk(tot, 256) < 1184 ? nblk(tot, 256) : 1184), dim3(256), 0,
                                    st, p, M, s->ar);
        if (er != cudaSuccess) {
            vxc_set_error("vxc_forward: %s", cudaGetErrorString(er));
            return -3;
        }
        if (int r = vxc_tp_allreduce_sum(n->tp, s->ar, tot, st)) return r;
        p.base = s->ar;
        p.slot = (size_t)64 * E;
        p.R = E;
        p.M = M;
        p.ks_full = p.ks_last = 1;
        return 0;
    };
    cudaEvent_t pe = prof_begin(st);
    e = launch_pdl(k_embed, dim3(M), dim3(256), 0, st, n->embd, n->embd_type, n->embd_row_bytes,
                               n->embd_rows, E, d_tokens, s->x, err);
    prof_end(0, pe, st);
    const int G = H / KH, nq = T * G, qcn = attn_qc(nq), nqc = (nq + qcn - 1) / qcn;
    const size_t asm_bytes = attn_smem(hd, s->attn_sl, qcn);
    CUtensorMap tmk, tmv;
    memcpy(&tmk, s->tmk, sizeof tmk);
    memcpy(&tmv, s->tmv, sizeof tmv);
    // local columns of a row kernel's CTA (norm: E / ROW_CL, SwiGLU: F / ROW_CL, merge: heads x hd)
    auto cols8 = [](int K) { return ((K + ROW_CL - 1) / ROW_CL + 7) / 8 * 8; };
    size_t row_smem = (size_t)cols8(E);
    if ((size_t)cols8(F) > row_smem) row_smem = cols8(F);
    if ((size_t)((H + ROW_CL - 1) / ROW_CL) * hd > row_smem) row_smem = (size_t)((H + ROW_CL - 1) / ROW_CL) * hd;
    row_smem *= sizeof(float);
    Part prev;
    prev.base = NULL;
    prev.slot = 0;
    prev.R = prev.M = prev.ks_full = prev.ks_last = 0;
    Part pp;
    // where a row kernel writes the operand of the GEMV/GEMM that reads it
    struct ImgOut {
        uint8_t *img;
        size_t bytes;
        int csh;
    };
    auto img_for = [&](const vxc_qmat *w, int rows) -> ImgOut {
        switch (gemv_mode(w, rows, gemm_min)) {
            case GM_GEMM: return {s->img, (VXC_GEMM_SLAB / 64) * s->img_chunk, 8};
            case GM_SKINNY: return {NULL, s->img_chunk, 6};
            default: return {s->img, s->img_chunk, 6};
        }
    };
    static_assert(VXC_GEMM_SLAB == 256, "slab rows = 2^8");
    for (int l = 0; l < c.n_layers && e == cudaSuccess; l++) {
        const vxc_layer_dev *d = &n->layers[l];
        float *kc = s->k + (size_t)l * s->n_slots * s->max_ctx * kvd;
        float *vc = s->v + (size_t)l * s->n_slots * s->max_ctx * kvd;
        pe = prof_begin(st);
        ImgOut io = img_for(d->wqkv, M);
        e = launch_pdl_cluster(k_norm_image, dim3(ROW_CL, M), dim3(ROW_THREADS), row_smem, st, ROW_CL, s->x, prev,
                               d->attn_norm, E, (const int *)NULL, 1, M, io.img, io.bytes, io.csh, s->xs, s->xf);
        prof_end(1, pe, st);
        if (e != cudaSuccess) break;
        pe = prof_begin(st);
        if ((rc = gemv_rows(s, d->wqkv, M, &pp, st, gemm_min))) return rc;
        prof_end(2, pe, st);
        pe = prof_begin(st);
        e = launch_pdl(k_rope_kv, dim3(H + 2 * KH, M), dim3(((hd / 2) + 31) / 32 * 32), 0, st, pp, T, d_slot, d_pos, (const float2 *)n->rope,
                       c.max_pos, H, KH, hd, s->qbuf, kc, vc, s->n_slots, s->max_ctx, err);
        prof_end(3, pe, st);
        if (e != cudaSuccess) break;
        pe = prof_begin(st);
        e = launch_pdl(attn_kernel(hd, qcn), dim3(n_groups * KH * nqc, s->attn_splits), dim3(128), asm_bytes, st,
                       (const float *)s->qbuf, T, d_slot, d_pos, H, KH, tmk, tmv, l * s->n_slots * KH * s->max_ctx,
                       s->n_slots, s->max_ctx, s->attn_sl, nqc, s->attn_part, err);
        prof_end(4, pe, st);
        if (e != cudaSuccess) break;
        pe = prof_begin(st);
        io = img_for(d->wo, M);
        e = launch_pdl_cluster(k_combine_image, dim3(ROW_CL, M), dim3(ROW_THREADS), row_smem, st, ROW_CL,
                               (const float *)s->attn_part, T, H, KH, hd, s->attn_splits, M, io.img, io.bytes,
                               io.csh, s->xs, s->xf);
        prof_end(5, pe, st);
        if (e != cudaSuccess) break;
        pe = prof_begin(st);
        if ((rc = gemv_rows(s, d->wo, M, &pp, st, gemm_min))) return rc;
        if (n->tp && (rc = tp_sum(pp))) return rc;
        prof_end(6, pe, st);
        pe = prof_begin(st);
        io = img_for(d->wgu, M);
        e = launch_pdl_cluster(k_norm_image, dim3(ROW_CL, M), dim3(ROW_THREADS), row_smem, st, ROW_CL, s->x, pp,
                               d->ffn_norm, E, (const int *)NULL, 1, M, io.img, io.bytes, io.csh, s->xs, s->xf);
        prof_end(7, pe, st);
        if (e != cudaSuccess) break;
        pe = prof_begin(st);
        if ((rc = gemv_rows(s, d->wgu, M, &pp, st, gemm_min))) return rc;
        prof_end(8, pe, st);
        pe = prof_begin(st);
        io = img_for(d->wd, M);
        e = launch_pdl_cluster(k_swiglu_image, dim3(ROW_CL, M), dim3(ROW_THREADS), row_smem, st, ROW_CL, pp, F, M,
                               io.img, io.bytes, io.csh, s->xs, s->xf);
        prof_end(9, pe, st);
        if (e != cudaSuccess) break;
        pe = prof_begin(st);
        if ((rc = gemv_rows(s, d->wd, M, &prev, st, gemm_min))) return rc;
        if (n->tp && (rc = tp_sum(prev))) return rc;
        prof_end(10, pe, st);
    }
    if (e == cudaSuccess && n_logit_rows > 0) {
        pe = prof_begin(st);
        const int V = c.n_vocab;
        // last residual update fused with the final norm, for the requested rows only
        const ImgOut lo = img_for(n->out, n_logit_rows);
        e = launch_pdl_cluster(k_norm_image, dim3(ROW_CL, n_logit_rows), dim3(ROW_THREADS), row_smem, st, ROW_CL,
                               s->x, prev, n->out_norm, E, d_logit_rows, 0, n_logit_rows, lo.img, lo.bytes, lo.csh,
                               s->xs, s->xf);
        if (e == cudaSuccess) {
            if ((rc = gemv_rows(s, n->out, n_logit_rows, &pp, st, gemm_min))) return rc;
            const size_t tot = (size_t)n_logit_rows * n->Vl;
            e = launch_pdl(k_part_out, dim3(nblk(tot, 256) < 1184 ? nblk(tot, 256) : 1184), dim3(256), 0, st, pp,
                           n_logit_rows, n->tp ? s->lg_local : d_logits);
            if (e == cudaSuccess && n->tp) {
                // vocabulary-parallel LM head: gather every GPU's rows of the logits
                if (vxc_tp_allgather(n->tp, s->lg_local, s->lg_all, tot, st)) return -3;
                const size_t all = (size_t)n_logit_rows * V;
                e = launch_pdl(k_vocab_gather, dim3(nblk(all, 256) < 1184 ? nblk(all, 256) : 1184), dim3(256), 0, st,
                               (const float *)s->lg_all, n->world, n_logit_rows, n->Vl, d_logits);
            }
        }
        prof_end(11, pe, st);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { vxc_set_error("vxc_forward: %s", cudaGetErrorString(e)); return -3; }
    return 0;
}

extern "C" int vxc_forward(vxc_seqs *s, const int *d_tokens, const int *d_slot, const int *d_pos, int n_groups,
                           int rows_per_group, const int *d_logit_rows, int n_logit_rows, float *d_logits,
                           void *stream) {
    return forward_impl(s, d_tokens, d_slot, d_pos, n_groups, rows_per_group, d_logit_rows, n_logit_rows, d_logits,
                        stream, VXC_GEMM_MIN_ROWS);
}

// The prompt pass of the speculative engine: every Q4_0 / Q8_0 matrix runs on
// the GEMM whatever the row count, so a prompt row's numbers do not depend on
// how the prompts were batched (a row's GEMM result depends on that row only).
int vxc_forward_prompt(vxc_seqs *s, const int *d_tokens, const int *d_slot, const int *d_pos, int n_groups,
                       int rows_per_group, void *stream) {
    return forward_impl(s, d_tokens, d_slot, d_pos, n_groups, rows_per_group, NULL, 0, NULL, stream, 1);
}

// ---------------------------------------------------------------------------
// host-buffer single-sequence path (vx_model_forward)
// ---------------------------------------------------------------------------
extern "C" int vxc_forward_host(vxc_seqs *s, int slot, int pos0, const int *h_tokens, int n_tokens,
                                float *h_logits) {
    if (!s || !h_tokens || n_tokens <= 0 || slot < 0 || slot >= s->n_slots || pos0 < 0) {
        vxc_set_error("vxc_forward_host: bad arguments");
        return -4;
    }
    if (pos0 + n_tokens > s->max_ctx) {
        vxc_set_error("vxc_forward_host: positions %d..%d exceed the context of %d", pos0, pos0 + n_tokens - 1,
                      s->max_ctx);
        return -4;
    }
    const int V = s->net->cfg.n_vocab;
    int *d_i = NULL;
    float *d_l = NULL;
    const int chunk = s->max_rows;
    VXC_CUDA_OK(cudaMalloc((void **)&d_i, (size_t)(chunk + 3) * sizeof(int)));
    if (cudaMalloc((void **)&d_l, (size_t)V * sizeof(float)) != cudaSuccess) {
        cudaFree(d_i);
        vxc_set_error("vxc_forward_host: out of device memory");
        return -3;
    }
    int rc = 0;
    for (int done = 0; done < n_tokens && rc == 0; done += chunk) {
        int n = n_tokens - done < chunk ? n_tokens - done : chunk;
        int meta[3] = {slot, pos0 + done, n - 1};
        if (cudaMemcpy(d_i, h_tokens + done, (size_t)n * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d_i + chunk, meta, sizeof meta, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = -3;
            break;
        }
        const bool last = done + n >= n_tokens;
        rc = vxc_forward(s, d_i, d_i + chunk, d_i + chunk + 1, 1, n, last ? d_i + chunk + 2 : NULL, last ? 1 : 0,
                         last ? d_l : NULL, NULL);
    }
    if (rc == 0 && h_logits && cudaMemcpy(h_logits, d_l, (size_t)V * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = -3;
    if (rc == 0) rc = vxc_check_device_error(NULL);
    cudaFree(d_i);
    cudaFree(d_l);
    return rc;
}

// ---------------------------------------------------------------------------
// greedy decoding on the device (the loop of the reference's CLI,
// src/main.c:283-324, without its second forward of the last prompt token)
// ---------------------------------------------------------------------------
extern "C" int vxc_greedy_generate(vxc_seqs *s, int slot, int pos0, const int *h_prompt, int n_prompt, int *h_out,
                                   int max_tokens, int eos_id, int *n_out, int *pos_out) {
    if (!s || !h_prompt || n_prompt <= 0 || !h_out || max_tokens <= 0 || slot < 0 || slot >= s->n_slots ||
        pos0 < 0) {
        vxc_set_error("vxc_greedy_generate: bad arguments");
        return -4;
    }
    if ((long long)pos0 + n_prompt + max_tokens > s->max_ctx) {
        vxc_set_error("vxc_greedy_generate: %d + %d + %d positions exceed the context of %d", pos0, n_prompt,
                      max_tokens, s->max_ctx);
        return -4;
    }
    const int V = s->net->cfg.n_vocab, chunk = s->max_rows;
    // ints: prompt chunk | chunk meta {slot, pos, last row} | tok | state {n, pos, done} | slot | row 0 | out
    const int o_meta = chunk, o_tok = chunk + 3, o_st = o_tok + 1, o_slot = o_st + 3, o_row = o_slot + 1,
              o_out = o_row + 1;
    int *d_i = NULL;
    float *d_l = NULL;
    cudaStream_t st = NULL;
    cudaGraph_t graph = NULL;
    cudaGraphExec_t exec = NULL;
    cudaError_t e = cudaMalloc((void **)&d_i, (size_t)(o_out + max_tokens) * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc((void **)&d_l, (size_t)V * sizeof(float));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    int rc = e == cudaSuccess ? 0 : -3;
    if (rc) vxc_set_error("vxc_greedy_generate: %s", cudaGetErrorString(e));
    // prompt pass, logits of its last row only
    for (int done = 0; done < n_prompt && rc == 0; done += chunk) {
        const int n = n_prompt - done < chunk ? n_prompt - done : chunk;
        const int meta[3] = {slot, pos0 + done, n - 1};
        e = cudaMemcpyAsync(d_i, h_prompt + done, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_i + o_meta, meta, sizeof meta, cudaMemcpyHostToDevice, st);
        // the host arrays are reused next chunk
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            vxc_set_error("vxc_greedy_generate: %s", cudaGetErrorString(e));
            rc = -3;
            break;
        }
        const bool last = done + n >= n_prompt;
        rc = vxc_forward(s, d_i, d_i + o_meta, d_i + o_meta + 1, 1, n, last ? d_i + o_meta + 2 : NULL, last ? 1 : 0,
                         last ? d_l : NULL, st);
    }
    int state[3] = {0, pos0 + n_prompt - 1, 0};
    if (rc == 0) {
        const int init[6] = {state[0], state[1], state[2], slot, 0, 0};
        e = cudaMemcpyAsync(d_i + o_st, init, 5 * sizeof(int), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = launch_pdl(k_argmax_row, dim3(1), dim3(1024), 0, st, (const float *)d_l, V, d_i + o_tok);
        if (e == cudaSuccess)
            e = launch_pdl(k_greedy_record, dim3(1), dim3(32), 0, st, (const int *)(d_i + o_tok), d_i + o_st,
                           d_i + o_out, eos_id, max_tokens);
        if (e == cudaSuccess) e = cudaMemcpyAsync(state, d_i + o_st, sizeof state, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) { vxc_set_error("vxc_greedy_generate: %s", cudaGetErrorString(e)); rc = -3; }
    }
    // one captured graph per token: forward the last token, argmax, record
    if (rc == 0 && !state[2]) {
        const long long before = vxc_launch_count();
        e = cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed);
        if (e == cudaSuccess) {
            rc = vxc_forward(s, d_i + o_tok, d_i + o_slot, d_i + o_st + 1, 1, 1, d_i + o_row, 1, d_l, st);
            cudaError_t e1 = cudaSuccess, e2 = cudaSuccess;
            if (rc == 0) e1 = launch_pdl(k_argmax_row, dim3(1), dim3(1024), 0, st, (const float *)d_l, V, d_i + o_tok);
            if (rc == 0 && e1 == cudaSuccess)
                e1 = launch_pdl(k_greedy_record, dim3(1), dim3(32), 0, st, (const int *)(d_i + o_tok), d_i + o_st,
                                d_i + o_out, eos_id, max_tokens);
            e2 = cudaStreamEndCapture(st, &graph);
            e = e1 != cudaSuccess ? e1 : e2;
        }
        const long long per_step = vxc_launch_count() - before;
        vxc_count_launches(-per_step);   // captured, not run; each replay counts them
        if (rc == 0 && e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
        if (rc == 0 && e != cudaSuccess) { vxc_set_error("vxc_greedy_generate: graph: %s", cudaGetErrorString(e)); rc = -3; }
        // each replay emits one token until done: max_tokens - 1 replays at most; the
        // host looks at the done flag every 8 replays (a few extra forwards after
        // eos write only positions past the cache length)
        for (int i = 0; rc == 0 && i < max_tokens - 1; i++) {
            e = cudaGraphLaunch(exec, st);
            if (e != cudaSuccess) break;
            vxc_count_launches(per_step);
            if ((i & 7) == 7 || i == max_tokens - 2) {
                e = cudaMemcpyAsync(state, d_i + o_st, sizeof state, cudaMemcpyDeviceToHost, st);
                if (e == cudaSuccess) e = cudaStreamSynchronize(st);
                if (e != cudaSuccess || state[2]) break;
            }
        }
        if (rc == 0 && e != cudaSuccess) { vxc_set_error("vxc_greedy_generate: %s", cudaGetErrorString(e)); rc = -3; }
    }
    if (rc == 0) {
        e = cudaMemcpyAsync(state, d_i + o_st, sizeof state, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e == cudaSuccess && state[0] > 0)
            e = cudaMemcpy(h_out, d_i + o_out, (size_t)state[0] * sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) { vxc_set_error("vxc_greedy_generate: %s", cudaGetErrorString(e)); rc = -3; }
    }
    if (rc == 0) rc = vxc_check_device_error(NULL);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (st) {
        cudaStreamSynchronize(st);
        cudaStreamDestroy(st);
    }
    if (d_i) cudaFree(d_i);
    if (d_l) cudaFree(d_l);
    if (rc == 0) {
        if (n_out) *n_out = state[0];
        if (pos_out) *pos_out = state[1];
    }
    return rc;
}
