// vxc_gemv_tc.cu — Q4_0 / Q8_0 GEMV on the 5th-generation tensor cores
// (reference src/quantize.c:728-750 for Q4_0, src/model.c:234-244 for Q8_0):
//
//   y[m][r] = sum_b d[r][b] * sum_{j<32} (q[r][32b+j] - off) * x[m][32b+j]
//
// Exactness (why not a plain bf16 GEMM).  The weight w = d' * (q - off), with
// d' = d * 2^wshift (vxc_qmat.cuh), has at most 14 (Q4_0) or 18 (Q8_0)
// significant bits, so it is exactly w_hi + w_lo with w_hi = RN_fp16(w) and
// w_lo = w - w_hi (computed by one fused fp16 multiply-add).  The activation
// row is prescaled by a power of two and split into fp16 hi + lo (22
// significant bits; the image layout is in vxc_qmat.cuh).  The products are
// accumulated in fp32 TMEM over the whole K-slice (MMA shape below), so the
// result equals the fp32 reference up to summation order.  A single fp16
// weight or activation would move the logits by ~1e-3 relative through the
// FFN's |silu| < 0.01 row mask (reference src/model.c:583-585).
//
// Work split.  Items are (128-row tile, K-slice of nbs blocks).  CTA c owns
// slice c % ks and the tiles c / ks, c / ks + cps, ...  (cps = CTAs per
// slice), so its slice of the activation image is fetched once (one bulk
// copy per block, one barrier per stage) and stays in shared memory for all
// its tiles.  Each item writes fp32 partial sums part[slice][m][row]; the
// consumer of the GEMV output adds the ks slices in slice order.
//
// MMA shape.  One thread issues one tcgen05.mma per ~200 SM cycles whatever
// N is (16..256, A from TMEM or shared memory; measured on B200), while MMAs
// of different threads overlap, so one issuer cannot keep up with HBM at
// these sizes; several threads issuing into separate accumulators can.  The image
// stacks [x_hi; x_lo] as 2N rows of B, so per K step two MMAs (A = w_hi, then
// A = w_lo) give the hi/lo products in one 2N-column accumulator; the
// epilogue adds column m and N + m.  With GM_LO_HALF_N (the default) the w_lo
// MMA covers the x_hi rows only, dropping w_lo * x_lo (at most 2^-22 of the
// product).
//
// Warp roles (448 threads, one CTA per SM):
//   warp 0      producer: cp.async.bulk of KB weight records per stage into
//               the two groups' halves of a ring of RS stages (weights first:
//               they do not depend on the preceding kernel), then the image
//               slice after griddepcontrol.wait
//   warp 1      TMEM owner
//   warps 2-9   two converter groups (even / odd stages): thread = weight row;
//               raw quants -> w_hi, w_lo fp16 -> tcgen05.st into the group's
//               TMEM A buffer (A operand read from TMEM by the MMA).  Lane 0
//               of the group's first IG warps then issues the MMAs of the
//               stage, issuer i taking blocks i, i+IG, ... into its own
//               accumulator
//   warps 10-13 epilogue: zero the accumulators for the next item, then
//               tcgen05.ld, sum the 2*IG accumulators in a fixed order, scale,
//               store
// TMEM: A buffers 2 x KB*32 columns, 2*IG accumulators x 2N columns.  No TMA
// multicast anywhere.
//
// Every mbarrier wait is bounded (VXC_WAIT_NS); on expiry the CTA records an
// error code, all roles stop, in-flight copies and MMAs are drained (bounded)
// and TMEM is freed.
#include "vxc_common.cuh"
#include "vxc_image.cuh"
#include "vxc_ptx.cuh"
#include "vxc_qmat.cuh"
#include "vxc_internal.h"

#include <atomic>
#include <stdio.h>

#define GM_THREADS 448
#define GM_SMS 148
#define GM_SMEM_DYN (220 * 1024)
#define GM_TMEM_COLS 512u
#define GM_MAXG 48          // image barriers: stages of one K-slice

// Per (quant type, N/16): blocks per stage KB, MMA issuers per converter
// group IG and ring depth RS, such that TMEM holds the two groups' A buffers
// (KB*32 columns each) plus 2*IG accumulators of 2N columns, and ~55-70 KB of
// weights are in flight.
#ifndef GM_PART_COST
#define GM_PART_COST 0.5    // planner weight of a partial-sum byte (written + read) vs an HBM weight byte
#endif
#ifndef GM_IMAGE_COST
#define GM_IMAGE_COST 0.3   // ... of an image byte (read from L2 by every CTA of a slice)
#endif
#ifndef GM_KB_SMALL_N
#define GM_KB_SMALL_N 4     // blocks per stage for N <= 32
#endif
#ifndef GM_RING_BLOCKS
#define GM_RING_BLOCKS 24   // Q4_0 blocks in flight per CTA (Q8_0: two thirds)
#endif
#ifndef GM_LO_HALF_N
#define GM_LO_HALF_N 1      // 1: the w_lo MMA over the x_hi rows only (drops w_lo*x_lo, <= 2^-22 of a
                            // product): 3N instead of 4N accumulator columns of tensor work per K step;
                            // measured 0-3% faster on B200 (the kernel is issue-bound), parity unchanged
#endif
__host__ __device__ constexpr int gm_kb_of(int qt, int nt) {
    return nt == 1 ? (qt == 8 ? 6 : GM_KB_SMALL_N) : nt == 2 ? GM_KB_SMALL_N : nt == 3 ? 5 : 4;
}

template <int QT, int NT>
struct GmCfg {
    static constexpr int QB = QT == 2 ? 16 : 32;
    static constexpr int REC = 128 * QB + 256;
    // Blocks per stage and MMA issuers per converter group, as measured best on
    // B200 within the TMEM budget below: larger stages mean fewer commits and
    // barrier rounds per weight block, more issuers more MMAs in flight.  Above
    // 32 rows one issuer per group (stages of 5 blocks at N = 48, 4 at N = 64:
    // 10-15% faster than 2-block stages with two issuers); up to 16 rows, Q8_0
    // (the draft's matrices) 6-block stages with two issuers (5-11% faster than
    // 4 blocks with four), Q4_0 4 blocks with four.
    static constexpr int KB = gm_kb_of(QT, NT);
    static constexpr int IG = NT == 1 ? (KB == 4 ? 4 : 2) : NT >= 3 ? 1 : 2;
    static constexpr int STAGE = KB * REC;
    static constexpr int RS = (QT == 2 ? GM_RING_BLOCKS : GM_RING_BLOCKS * 2 / 3) / KB / 2 * 2;   // even
    static_assert(2 * KB * 32 + 2 * IG * 32 * NT <= 512, "TMEM budget");
};

struct GmArgs {
    const uint8_t *qs;      // weight records
    int R, nblk, ntile;
    const uint8_t *img;     // activation image, N rows (when x == NULL)
    const float *xs;        // [M] prescales of the image
    const float *x;         // or fp32 activation rows [M][K]: each CTA builds its slice's image
    int M;
    float *part;            // [ks][M][R]
    int ks, nbs;
    float wscale;
    unsigned int *err;
};

// ---------------------------------------------------------------------------
// Dequantisers: raw row-block word(s) -> 4 half2 (q - off) of 8 elements
// ---------------------------------------------------------------------------
__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }
__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }

// Q4_0 permuted word -> (q-8) pairs (8j+2i, 8j+2i+1), i = 0..3.  1024 + q is
// exact in fp16 (magic 0x6400 = 1024.0), and (1024 + q) - 1032 = q - 8.
__device__ __forceinline__ void deq_q4_word(uint32_t w, __half2 *o) {
    const __half2 bias = u2h(0x64086408u);
#pragma unroll
    for (int i = 0; i < 4; i++) o[i] = __hsub2(u2h(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u), bias);
}

// Q8_0: two words (8 int8) -> 4 pairs.  (int8 ^ 0x80) is q + 128 in 0..255;
// 1024 + that is exact, minus 1152 gives q.
__device__ __forceinline__ void deq_q8_words(uint32_t w0, uint32_t w1, __half2 *o) {
    const __half2 bias = u2h(0x64806480u);
    const uint32_t a = w0 ^ 0x80808080u, b = w1 ^ 0x80808080u;
    o[0] = __hsub2(u2h(__byte_perm(a, 0x64646464u, 0x4140)), bias);
    o[1] = __hsub2(u2h(__byte_perm(a, 0x64646464u, 0x4342)), bias);
    o[2] = __hsub2(u2h(__byte_perm(b, 0x64646464u, 0x4140)), bias);
    o[3] = __hsub2(u2h(__byte_perm(b, 0x64646464u, 0x4342)), bias);
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
template <int QT, int NT>
__global__ void __launch_bounds__(GM_THREADS, 1) k_qgemv_mma(const GmArgs a) {
    using C = GmCfg<QT, NT>;
    constexpr int N = 16 * NT, NP = 2 * N;   // B = [x_hi; x_lo]: NP rows
    constexpr int KB = C::KB, RS = C::RS, IG = C::IG, ACOL = KB * 32, NACC = 2 * IG, RSG = RS / 2;
    static_assert(RS % 2 == 0 && RS >= 2, "ring: two equal halves, one per converter group");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[2 * RS + 6 + GM_MAXG];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ float xinv[N];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ks = a.ks;
    const int slice = blockIdx.x % ks;
    const int cps = gridDim.x / ks;
    const int r0 = blockIdx.x / ks;
    const int b0 = slice * a.nbs;
    const int nb = min(a.nbs, a.nblk - b0);
    const int nst = (nb + KB - 1) / KB;
    const int nitems = (r0 < a.ntile && nb > 0) ? (a.ntile - 1 - r0) / cps + 1 : 0;
    const int total = nitems * nst;
    const int ngroups = nst >= 2 ? 2 : 1;      // converter groups with stages in every item

    uint8_t *Bs = smem;                                   // nbs blocks x 128*N bytes
    uint8_t *Raw = Bs + (size_t)a.nbs * 128 * N;          // RS stages

    const uint32_t bar0 = smem_u32(bars);
    auto raw_full = [&](int s) { return bar0 + 8u * s; };
    auto raw_empty = [&](int s) { return bar0 + 8u * (RS + s); };
    auto a_empty = [&](int j) { return bar0 + 8u * (2 * RS + j); };
    const uint32_t acc_full = bar0 + 8u * (2 * RS + 2);
    const uint32_t acc_empty = bar0 + 8u * (2 * RS + 3);
    const uint32_t fin_bar = bar0 + 8u * (2 * RS + 4);
    auto b_full = [&](int g) { return bar0 + 8u * (2 * RS + 6 + g); };

    if (tid == 0) {
        for (int s = 0; s < RS; s++) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), 128);
        }
        for (int j = 0; j < 2; j++) mbar_init(a_empty(j), IG);
        mbar_init(acc_full, IG * ngroups);
        mbar_init(acc_empty, 128);
        mbar_init(fin_bar, NACC);
        for (int g = 0; g < GM_MAXG; g++) mbar_init(b_full(g), 1);
        abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), GM_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_trigger();
    const uint32_t tmem_base = tmem_slot;
    volatile int *abortp = &abort_flag;
    unsigned int *err = a.err;

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            // each converter group has its own RS/2 ring slots, used in order, so a
            // group never waits on a slot phase that the other group still owns
            int q = 0;
            int last_phase[RS];
            for (int i = 0; i < RS; i++) last_phase[i] = -1;
            auto slot_of = [&](int qq, int &slot, int &phase) {
                const int item = qq / nst, gl = qq % nst, g = gl & 1;
                const int u = item * ((nst - g + 1) / 2) + (gl >> 1);
                slot = g * RSG + u % RSG;
                phase = u / RSG;
            };
            auto issue = [&](int qq) -> bool {
                int sl, ph;
                slot_of(qq, sl, ph);
                if (ph >= 1 && !mbar_wait(raw_empty(sl), (ph - 1) & 1, abortp, err, VXC_DERR_TIMEOUT_TMA))
                    return false;
                const int item = qq / nst, g = qq % nst;
                const int tile = r0 + item * cps;
                const int kbn = min(KB, nb - g * KB);
                const uint8_t *src = a.qs + ((size_t)tile * a.nblk + b0 + g * KB) * C::REC;
                mbar_expect_tx(raw_full(sl), (uint32_t)(kbn * C::REC));
                bulk_g2s(smem_u32(Raw + (size_t)sl * C::STAGE), src, (uint32_t)(kbn * C::REC), raw_full(sl));
                last_phase[sl] = ph;
                return true;
            };
            // weights do not depend on the preceding kernel: fill the free slots now
            for (; q < total; q++) {
                int sl, ph;
                slot_of(q, sl, ph);
                if (ph >= 1) break;
                issue(q);
            }
            pdl_wait();
            if (total > 0 && !a.x) {
                // the image slice, one barrier per stage so the first MMAs need not wait for all of it
                for (int g = 0; g < nst; g++) {
                    const int kbn = min(KB, nb - g * KB);
                    mbar_expect_tx(b_full(g), (uint32_t)(kbn * 128 * N));
                    for (int kb = 0; kb < kbn; kb++) {
                        const int b = g * KB + kb;
                        bulk_g2s(smem_u32(Bs + (size_t)b * 128 * N), a.img + (size_t)(b0 + b) * 128 * N, 128 * N,
                                 b_full(g));
                    }
                }
            }
            for (; q < total; q++)
                if (!issue(q)) break;
            if (*abortp) {
                // drain (bounded): the last stage issued into each slot, and the image
                for (int sl = 0; sl < RS; sl++) {
                    if (last_phase[sl] < 0) continue;
                    const uint64_t t0 = vxc_globaltimer();
                    while (!mbar_try(raw_full(sl), last_phase[sl] & 1) && vxc_globaltimer() - t0 < 100000000ull) {}
                }
                for (int g = 0; total > 0 && g < nst; g++) {
                    const uint64_t t0 = vxc_globaltimer();
                    while (!mbar_try(b_full(g), 0) && vxc_globaltimer() - t0 < 100000000ull) {}
                }
            }
        }
    } else if (warp >= 2 && warp < 10) {
        // ----------------- converters + MMA issue (lane 0 of the first IG warps of a group) -----------------
        const int group = (warp - 2) >> 2;
        const int kw = (warp - 2) & 3;            // warp within the group
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t tlane = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const bool issuer = kw < IG && lane == 0;
        const uint32_t idesc = (1u << 4) | ((uint32_t)(NP >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        // the w_lo MMA: all 2N rows of B, or (GM_LO_HALF_N) the first N, the x_hi parts
        const uint32_t idesc_lo =
            GM_LO_HALF_N ? (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24) : idesc;
        const uint32_t bbase = smem_u32(Bs);
        const uint32_t dcol = tmem_base + 2 * ACOL + (group * IG + kw) * NP;
        const int per_item = (nst - group + 1) / 2;   // this group's stages per item
        bool ok = true;
        for (int item = 0; item < nitems && ok; item++) {
            for (int gl = group; gl < nst; gl += 2) {
                const int u = item * per_item + (gl >> 1);   // this group's stage count (A buffer, ring slot)
                const int s = group * RSG + u % RSG;
                const int kbn = min(KB, nb - gl * KB);
                bool w_ok = mbar_wait_warp(raw_full(s), (u / RSG) & 1, abortp, err, VXC_DERR_TIMEOUT_TMA);
                uint32_t qw[KB][C::QB / 4];
                uint32_t dh[KB];
                if (w_ok) {
                    const uint8_t *st = Raw + (size_t)s * C::STAGE;
#pragma unroll
                    for (int kb = 0; kb < KB; kb++) {
                        if (kb < kbn) {
                            const uint8_t *rec = st + kb * C::REC;
                            const uint4 *qp = reinterpret_cast<const uint4 *>(rec + row * C::QB);
#pragma unroll
                            for (int v = 0; v < C::QB / 16; v++) {
                                const uint4 w4 = qp[v];
                                qw[kb][4 * v] = w4.x;
                                qw[kb][4 * v + 1] = w4.y;
                                qw[kb][4 * v + 2] = w4.z;
                                qw[kb][4 * v + 3] = w4.w;
                            }
                            const uint32_t h = reinterpret_cast<const uint16_t *>(rec + 128 * C::QB)[row];
                            dh[kb] = h | (h << 16);
                        }
                    }
                    mbar_arrive(raw_empty(s));
                }
                // the MMAs of this group's previous stage have finished reading its A buffer
                if (w_ok && u >= 1) w_ok = mbar_wait_warp(a_empty(group), (u - 1) & 1, abortp, err, VXC_DERR_TIMEOUT_MMA);
                if (w_ok) {
                    tc_fence_after();
#pragma unroll
                    for (int kb = 0; kb < KB; kb++) {
                        if (kb < kbn) {
                            const __half2 d2 = u2h(dh[kb]);
                            uint32_t hi[16], lo[16];
#pragma unroll
                            for (int c = 0; c < 4; c++) {
                                __half2 qh[4];
                                if (QT == 2) deq_q4_word(qw[kb][c], qh);
                                else deq_q8_words(qw[kb][2 * c], qw[kb][2 * c + 1], qh);
#pragma unroll
                                for (int i = 0; i < 4; i++) {
                                    const __half2 h = __hmul2(qh[i], d2);
                                    hi[4 * c + i] = h2u(h);
                                    lo[4 * c + i] = h2u(__hfma2(qh[i], d2, __hneg2(h)));
                                }
                            }
                            const uint32_t col = tlane + group * ACOL + kb * 32;
                            tmem_st16(col, hi);
                            tmem_st16(col + 16, lo);
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                }
                // all four warps of the group have written their quarter of the A buffer (or
                // all stop together: the decision is the same in every warp of the group)
                ok = bar_and(2 + group, 128, w_ok && !*abortp);
                if (!ok) break;
                if (issuer) {
                    tc_fence_after();
                    bool iok = true;
                    // the accumulators were zeroed by the epilogue of the previous item
                    if (gl == group) iok = mbar_wait(acc_empty, item & 1, abortp, err, VXC_DERR_TIMEOUT_MMA);
                    if (iok && item == 0) iok = mbar_wait(b_full(gl), 0, abortp, err, VXC_DERR_TIMEOUT_TMA);
                    if (iok) {
                        tc_fence_after();
                        for (int kb = kw; kb < kbn; kb += IG) {
                            const int bl = gl * KB + kb;
#pragma unroll
                            for (int kk = 0; kk < 2; kk++) {
                                const uint32_t ahi = tmem_base + group * ACOL + kb * 32 + kk * 8;
                                const uint64_t bd =
                                    sdesc(bbase + (uint32_t)((bl * 4 + 2 * kk) * NP * 16), NP * 16, 128);
                                mma_f16_ts(dcol, ahi, bd, idesc, 1u);
                                mma_f16_ts(dcol, ahi + 16, bd, idesc_lo, 1u);
                            }
                        }
                    }
                    mma_commit(a_empty(group));
                    if (gl + 2 >= nst) mma_commit(acc_full);   // this group's last stage of the item
                }
                __syncwarp();
            }
        }
        if (issuer) {
            // nothing this thread issued may still run when TMEM is freed
            mma_commit(fin_bar);
            const uint64_t t0 = vxc_globaltimer();
            while (!mbar_try(fin_bar, 0) && vxc_globaltimer() - t0 < 100000000ull) {}
        }
    } else if (warp >= 10) {
        // ------------------------------ epilogue ------------------------------
        const int quarter = warp & 3;
        const int trow = quarter * 32 + lane;
        const uint32_t tlane = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const int M = a.M;
        uint32_t zero[16];
#pragma unroll
        for (int i = 0; i < 16; i++) zero[i] = 0u;
        // zero the accumulators (the MMAs always accumulate), then hand them to the issuers
#pragma unroll
        for (int c = 0; c < NACC * NP / 16; c++) tmem_st16(tlane + 2 * ACOL + c * 16, zero);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(acc_empty);
        pdl_wait();   // xs / x come from the preceding kernel; part may still be read by it
        if (a.x) {
            // fp32 rows in: build this slice's image in shared memory with a prescale of
            // its own per row (the partials are divided by it, so slices may differ)
            const int K = a.nblk * 32, k0 = b0 * 32, kl = nb * 32;
            const int et = tid - 320;
            for (int m = warp - 10; m < M; m += 4) {
                const float *xr = a.x + (size_t)m * K + k0;
                float mx = 0.0f;
                for (int k = lane; k < kl; k += 32) mx = fmaxf(mx, fabsf(xr[k]));
                mx = warp_max(mx);
                if (lane == 0) xinv[m] = vxc_prescale(mx);   // the prescale for now
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            for (int it = et; it < nb * 4 * M; it += 128) {
                const int m = it % M, rest = it / M, c = rest & 3, b = rest >> 2;
                const float4 *src = reinterpret_cast<const float4 *>(a.x + (size_t)m * K + k0 + b * 32 + c * 8);
                const float4 v0 = src[0], v1 = src[1];
                const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                uint4 hi, lo;
                vxc_hilo8(v, xinv[m], hi, lo);
                uint8_t *chunk = Bs + (size_t)(b * 4 + c) * NP * 16;
                *reinterpret_cast<uint4 *>(chunk + (size_t)m * 16) = hi;
                *reinterpret_cast<uint4 *>(chunk + (size_t)(N + m) * 16) = lo;
            }
            fence_proxy_async();   // generic-proxy stores -> the MMAs' async-proxy reads
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (et == 0)
                for (int g = 0; g < nst && total > 0; g++) mbar_arrive(b_full(g));
            for (int m = et; m < N; m += 128) xinv[m] = m < M ? a.wscale / xinv[m] : 0.0f;
        } else {
            for (int m = tid - 320; m < N; m += 128) xinv[m] = m < M ? a.wscale / a.xs[m] : 0.0f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        for (int item = 0; item < nitems; item++) {
            bool ok = mbar_wait_warp(acc_full, item & 1, abortp, err, VXC_DERR_TIMEOUT_EPI);
            if (!ok) break;
            tc_fence_after();
            // y[m] = sum over accumulators of (acc[m] + acc[N + m]), fixed order
            float y[N];
#pragma unroll
            for (int m = 0; m < N; m++) y[m] = 0.0f;
#pragma unroll
            for (int c = 0; c < NACC * NP / 16; c++) {
                uint32_t v[16];
                tmem_ld16(tlane + 2 * ACOL + c * 16, v);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; e++) y[(c * 16 + e) % N] += __uint_as_float(v[e]);
                tmem_st16(tlane + 2 * ACOL + c * 16, zero);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(acc_empty);
            const int row = (r0 + item * cps) * 128 + trow;
            if (row < a.R) {
                float *dst = a.part + (size_t)slice * M * a.R + row;
#pragma unroll
                for (int m = 0; m < N; m++)
                    if (m < M) dst[(size_t)m * a.R] = y[m] * xinv[m];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, GM_TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int gm_stage(int qt, int nt) { return gm_kb_of(qt, nt) * (128 * (qt == 2 ? 16 : 32) + 256); }
static int gm_rs(int qt, int nt) {
    return (qt == 2 ? GM_RING_BLOCKS : GM_RING_BLOCKS * 2 / 3) / gm_kb_of(qt, nt) / 2 * 2;
}

static size_t gm_smem(int qt, int nt, int nbs) {
    return (size_t)nbs * 128 * 16 * nt + (size_t)gm_rs(qt, nt) * gm_stage(qt, nt);
}

// Plan: pick the K-slice count minimising the busiest CTA's stages plus the
// partial-sum traffic (served mostly from L2).
bool vxc_gemv_plan(const vxc_qmat *w, int M, VxcGemvPlan *p) {
    if (!w || M < 1 || M > 64) return false;
    const int nt = (M + 15) / 16, N = 16 * nt, KB = gm_kb_of(w->type, nt);
    const long avail = GM_SMEM_DYN - (long)gm_rs(w->type, nt) * gm_stage(w->type, nt);
    int nbs_max = (int)(avail / (128L * N));
    if (nbs_max > GM_MAXG * KB) nbs_max = GM_MAXG * KB;
    if (nbs_max < 1) return false;
    double best = 1e30;
    int bks = 0, bnbs = 0, bcps = 0;
    const int ks_lo = (w->nblk + nbs_max - 1) / nbs_max;
    for (int ks = ks_lo; ks <= w->nblk && ks <= GM_SMS; ks++) {
        const int nbs = (w->nblk + ks - 1) / ks;
        const int kse = (w->nblk + nbs - 1) / nbs;
        if (kse != ks) continue;
        int cps = GM_SMS / ks;
        if (cps > w->ntile) cps = w->ntile;
        if (cps < 1) continue;
        const int tpc = (w->ntile + cps - 1) / cps;
        // in units of one Q4_0 block-record time per SM: the busiest CTA's weight
        // blocks, its pipeline fill per item, and the L2 traffic of the partial
        // sums (written + read) and of the image slices (read by every CTA of a slice)
        const double unit = (double)GM_SMS * (128 * 18);
        const double blocks = (double)tpc * nbs;
        const double part = ks > 1 ? GM_PART_COST * ks * (double)M * w->rows * 8.0 / unit : 0.0;
        const double image = GM_IMAGE_COST * (double)ks * cps * nbs * 128.0 * N / unit;
        const double cost = blocks + tpc * 2.0 * KB + part + image;
        if (cost < best - 1e-9) {
            best = cost;
            bks = ks;
            bnbs = nbs;
            bcps = cps;
        }
    }
    if (!bks) return false;
    p->nt = nt;
    p->ks = bks;
    p->nbs = bnbs;
    p->grid = bks * bcps;
    p->smem = gm_smem(w->type, nt, bnbs);
    return p->smem <= GM_SMEM_DYN;
}

template <int QT, int NT>
static cudaError_t launch_mma(const GmArgs &ga, const VxcGemvPlan &p, cudaStream_t st) {
    // the attribute is per device: a process that drives several GPUs sets it on each
    static std::atomic<uint64_t> attr_set{0};   // bit d: set on device d
    int dev = 0;
    cudaError_t ea = cudaGetDevice(&dev);
    if (ea != cudaSuccess) return ea;
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t)1 << dev : 0;
    if (!bit || !(attr_set.load(std::memory_order_acquire) & bit)) {
        ea = cudaFuncSetAttribute(k_qgemv_mma<QT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, GM_SMEM_DYN);
        if (ea != cudaSuccess) return ea;
        if (bit) attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(GM_THREADS);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_qgemv_mma<QT, NT>, ga);
    vxc_count_launches(1);
    return e;
}

int vxc_gemv_run(const vxc_qmat *w, const uint8_t *img, const float *xs, int M, float *part,
                 const VxcGemvPlan &p, cudaStream_t st, const float *x) {
    if (p.nt != (M + 15) / 16 || p.ks < 1 || p.grid < p.ks || p.smem > GM_SMEM_DYN) {
        vxc_set_error("vxc_gemv_run: plan does not match M = %d", M);
        return -4;
    }
    GmArgs ga;
    ga.qs = w->qs;
    ga.R = w->rows;
    ga.nblk = w->nblk;
    ga.ntile = w->ntile;
    ga.img = img;
    ga.xs = xs;
    ga.x = x;
    ga.M = M;
    ga.part = part;
    ga.ks = p.ks;
    ga.nbs = p.nbs;
    ga.wscale = w->wscale;
    ga.err = vxc_device_error_ptr();
    cudaError_t e;
    if (w->type == 2) {
        switch (p.nt) {
            case 1: e = launch_mma<2, 1>(ga, p, st); break;
            case 2: e = launch_mma<2, 2>(ga, p, st); break;
            case 3: e = launch_mma<2, 3>(ga, p, st); break;
            default: e = launch_mma<2, 4>(ga, p, st); break;
        }
    } else {
        switch (p.nt) {
            case 1: e = launch_mma<8, 1>(ga, p, st); break;
            case 2: e = launch_mma<8, 2>(ga, p, st); break;
            case 3: e = launch_mma<8, 3>(ga, p, st); break;
            default: e = launch_mma<8, 4>(ga, p, st); break;
        }
    }
    if (e != cudaSuccess) {
        vxc_set_error("vxc_gemv_run: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}

// Up to this many rows the GEMV builds its K-slices' operand from the fp32
// rows itself (measured faster: no separate image kernel); above it a
// separate kernel writes the image once for all CTAs.
#define GM_SELF_IMAGE_ROWS 16

// Workspace of the public entry point for one chunk of M <= 64 rows:
// [image 128*N per block][prescales, 256 B] when M > GM_SELF_IMAGE_ROWS, then
// the split-K partial sums ks*M*R fp32 when ks > 1.
static size_t img_bytes(const vxc_qmat *w, int M) {
    return M > GM_SELF_IMAGE_ROWS ? (size_t)w->nblk * vxc_img_block_bytes(vxc_img_rows(M)) + 256 : 0;
}

static size_t chunk_ws_bytes(const vxc_qmat *w, int M) {
    VxcGemvPlan p;
    if (!vxc_gemv_plan(w, M, &p)) return 0;
    return img_bytes(w, M) + (p.ks > 1 ? (size_t)p.ks * M * w->rows * sizeof(float) : 0);
}

// Workspace of the GEMM path (M >= VXC_GEMM_MIN_ROWS): the image in slabs,
// then the M prescales (each 256-byte aligned), then the K-slices' partial
// sums [ks][M][R] when ks > 1 (one slice is written to y directly).
static size_t gemm_img_bytes(const vxc_qmat *w, int M) {
    return (vxc_gemm_image_bytes(w->cols, M) + 255) & ~(size_t)255;
}
static size_t gemm_ws_bytes(const vxc_qmat *w, int M) {
    const int ks = vxc_gemm_slices(w);
    return gemm_img_bytes(w, M) + (((size_t)M * sizeof(float) + 255) & ~(size_t)255) +
           (ks > 1 ? (size_t)ks * M * w->rows * sizeof(float) : 0);
}

extern "C" size_t vxc_qgemv_workspace_bytes(const vxc_qmat *w, int M) {
    if (!w || M <= 0 || vxc_is_kquant(w->type)) return 0;
    if (M >= VXC_GEMM_MIN_ROWS && vxc_gemm_ok(w)) {
        const size_t g = gemm_ws_bytes(w, M);
        const size_t simt = vxc_qgemv_simt_ws(w, M);
        return g > simt ? g : simt;
    }
    const int mc = M < 64 ? M : 64;
    size_t b = chunk_ws_bytes(w, mc);
    if (M > 64 && M % 64) {
        size_t t = chunk_ws_bytes(w, M % 64);
        if (t > b) b = t;
    }
    // the same scratch also serves vxc_qgemv_simt and the skinny GEMV's partials
    const size_t simt = vxc_qgemv_simt_ws(w, M);
    if (simt > b) b = simt;
    if (vxc_skinny_ok(w, M)) {
        const int ks = vxc_skinny_slices(w);
        const size_t sk = ks > 1 ? (size_t)ks * M * w->rows * sizeof(float) : 0;
        if (sk > b) b = sk;
    }
    return b;
}

extern "C" int vxc_qgemv(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
                         size_t workspace_bytes, void *stream) {
    if (!w || !x || !y || M <= 0) { vxc_set_error("vxc_qgemv: bad arguments"); return -4; }
    if (((uintptr_t)x & 15) != 0) { vxc_set_error("vxc_qgemv: x must be 16-byte aligned"); return -4; }
    if (((uintptr_t)workspace & 15) != 0) { vxc_set_error("vxc_qgemv: workspace must be 16-byte aligned"); return -4; }
    cudaStream_t st = (cudaStream_t)stream;
    if (vxc_is_kquant(w->type)) return vxc_kquant_gemv(w, x, M, y, st);   // no workspace
    if (vxc_skinny_ok(w, M)) {   // few rows: CUDA-core kernel, HBM-bound
        const int ks = vxc_skinny_slices(w);
        const size_t need = ks > 1 ? (size_t)ks * M * w->rows * sizeof(float) : 0;
        if ((need && !workspace) || need > workspace_bytes) {
            vxc_set_error("vxc_qgemv: workspace %zu < %zu bytes", workspace_bytes, need);
            return -4;
        }
        float *part = ks > 1 ? (float *)workspace : y;
        int rc = vxc_skinny_run(w, x, w->cols, M, part, st);
        if (rc == 0 && ks > 1) rc = vxc_launch_splitk_reduce(part, ks, M, w->rows, y, st);
        return rc;
    }
    if (M >= VXC_GEMM_MIN_ROWS && vxc_gemm_ok(w)) {   // many rows: the tensor-core GEMM, weights read once per slab
        const size_t ib = gemm_img_bytes(w, M), need = gemm_ws_bytes(w, M);
        if (!workspace || need > workspace_bytes) {
            vxc_set_error("vxc_qgemv: workspace %zu < %zu bytes", workspace_bytes, need);
            return -4;
        }
        uint8_t *img = (uint8_t *)workspace;
        float *xs = (float *)(img + ib);
        float *part = (float *)(img + ib + (((size_t)M * sizeof(float) + 255) & ~(size_t)255));
        const int ks = vxc_gemm_slices(w);
        const size_t slab = (size_t)w->nblk * 128 * VXC_GEMM_SLAB;
        for (int m0 = 0; m0 < M; m0 += VXC_GEMM_SLAB) {
            const int ms = M - m0 < VXC_GEMM_SLAB ? M - m0 : VXC_GEMM_SLAB;
            const int rc = vxc_launch_act_image(x + (size_t)m0 * w->cols, ms, w->cols,
                                                img + (size_t)(m0 / VXC_GEMM_SLAB) * slab, xs + m0, st);
            if (rc) return rc;
        }
        if (ks == 1) return vxc_gemm_run(w, img, slab, xs, M, y, (size_t)64 * w->rows, 0, st);
        int rc = vxc_gemm_run(w, img, slab, xs, M, part, (size_t)64 * w->rows, (size_t)M * w->rows, st);
        if (rc == 0) rc = vxc_launch_splitk_reduce(part, ks, M, w->rows, y, st);
        return rc;
    }
    for (int m0 = 0; m0 < M; m0 += 64) {
        const int mc = M - m0 < 64 ? M - m0 : 64;
        VxcGemvPlan p;
        if (!vxc_gemv_plan(w, mc, &p)) { vxc_set_error("vxc_qgemv: no plan for %d x %d", w->rows, w->cols); return -7; }
        const size_t need = chunk_ws_bytes(w, mc);
        if ((need && !workspace) || need > workspace_bytes) {
            vxc_set_error("vxc_qgemv: workspace %zu < %zu bytes", workspace_bytes, need);
            return -4;
        }
        const float *xm = x + (size_t)m0 * w->cols;
        const size_t ib = img_bytes(w, mc);
        float *part = p.ks > 1 ? (float *)((uint8_t *)workspace + ib) : y + (size_t)m0 * w->rows;
        int rc;
        if (mc <= GM_SELF_IMAGE_ROWS) {
            rc = vxc_gemv_run(w, NULL, NULL, mc, part, p, st, xm);
        } else {
            uint8_t *img = (uint8_t *)workspace;
            float *xs = (float *)(img + ib - 256);
            rc = vxc_launch_act_image(xm, mc, w->cols, img, xs, st);
            if (rc == 0) rc = vxc_gemv_run(w, img, xs, mc, part, p, st);
        }
        if (rc == 0 && p.ks > 1) rc = vxc_launch_splitk_reduce(part, p.ks, mc, w->rows, y + (size_t)m0 * w->rows, st);
        if (rc) return rc;
    }
    return 0;
}

// ---------------------------------------------------------------------------
// vxc_qgemv_noalloc: vxc_qgemv for callers that cannot allocate device
// memory — for instance a host application that owns the whole device
// memory budget and forbids libraries to call cudaMalloc, or a latency-bound
// caller that cannot afford cudaMalloc's implicit device synchronisation.
// The scratch (activation image, prescales and split-K partial sums) lives in
// one static device array of VXC_QGEMV_NOALLOC_BYTES, which every GPU that
// loads this library holds until the process exits.  Nothing in it has to
// start at zero: every byte a call reads was written earlier by the same
// call.  All calls on a device share the array, so calls whose GPU work
// overlaps (different streams without ordering between them) race on it.
// The array's device address is looked up on the first call on each device
// (with that device current) and cached with the context it belongs to; a
// device reset that recreates the primary context makes the next call look
// it up again.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_qgemv_scratch[VXC_QGEMV_NOALLOC_BYTES];

struct NoallocSlot {
    std::atomic<void *> ptr{nullptr};   // device address of g_qgemv_scratch
    std::atomic<void *> ctx{nullptr};   // the context it belongs to
};
static NoallocSlot g_qgemv_scratch_slot[64];

extern "C" int vxc_qgemv_noalloc(const vxc_qmat *w, const float *x, int M, float *y, void *stream) {
    if (!w || !x || !y || M <= 0) {
        vxc_set_error("vxc_qgemv_noalloc: bad arguments");
        return -4;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        vxc_set_error("vxc_qgemv_noalloc: no current CUDA device");
        return -7;
    }
    const size_t need = vxc_qgemv_workspace_bytes(w, M);
    if (need > VXC_QGEMV_NOALLOC_BYTES) {
        vxc_set_error("vxc_qgemv_noalloc: %d x %d with %d rows needs %zu bytes of scratch; the static limit is %zu",
                      w->rows, w->cols, M, need, (size_t)VXC_QGEMV_NOALLOC_BYTES);
        return -4;
    }
    NoallocSlot &slot = g_qgemv_scratch_slot[dev];
    void *ctx = vxc_current_context();
    void *p = slot.ptr.load(std::memory_order_acquire);
    if (!p || slot.ctx.load(std::memory_order_acquire) != ctx) {
        // set-up, once per device (and context), with that device current: the
        // host-side name of the array is not a device address.  Two threads that
        // get here together store the same address.
        p = NULL;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_qgemv_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();   // do not leave the error for a later call to report
            vxc_set_error("vxc_qgemv_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
            return -3;
        }
        slot.ctx.store(ctx, std::memory_order_release);
        slot.ptr.store(p, std::memory_order_release);
    }
    return vxc_qgemv(w, x, M, y, p, VXC_QGEMV_NOALLOC_BYTES, stream);
}
