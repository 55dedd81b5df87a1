// vxc_gemm_tc.cu — Q4_0 / Q8_0 matrix product for many activation rows
// (the prompt pass and verifies of 64 rows and more) on the tcgen05 tensor
// cores.  The arithmetic is the reference's (src/quantize.c:728-750 for
// Q4_0, dequantise + src/tensor.c:103-120 for Q8_0, src/model.c:234-244):
//
//   y[m][r] = sum_b d[r][b] * sum_{j<32} (q[r][32b+j] - off) * x[m][32b+j]
//
// made exact in the same way as the GEMV of vxc_gemv_tc.cu: the weight
// w = d' * (q - off) is exactly w_hi + w_lo in fp16, the activation row is
// prescaled by a power of two and split into fp16 hi + lo, and the products
// w_hi*x_hi + w_hi*x_lo + w_lo*x_hi (w_lo*x_lo, at most 2^-22 of a product,
// is dropped) are accumulated in fp32 TMEM.  K is cut into slices of at most
// GG_KC blocks, each summed in its own accumulator and written as a partial
// sum; the consumer adds the slices in order.  (The tensor core's fp32
// accumulation loses about an ulp of the running sum per MMA, so one
// accumulator over K = 11008 drifted to 4e-5 of max|y|; slices of 2048
// columns keep it near 5e-6.)  The slice count depends on K only, so a row's
// result depends only on that row and the same token gives the same numbers
// in any batch.
//
// Why a second kernel.  The GEMV converts every weight once per 64 activation
// rows and keeps the converted tile in TMEM, which leaves room for
// accumulators of at most 64 rows.  Here the converted weights go to shared
// memory and the accumulators fill TMEM: each CTA tile is 256 weight rows
// (two 128-row weight tiles) x one slab of up to 256 activation rows, so
// every weight byte is read and converted once per 256 rows, and every MMA
// is 128 x N x 16 with N up to 256 (the largest shape of one instruction).
//
// Operands (canonical K-major, no swizzle: 8-row x 16-byte core matrices).
//   B, activations: the image slab as the producing kernel wrote it
//     (vxc_qmat.cuh layout with N = padded slab rows): per 32-column block,
//     4 chunks x [N hi rows; N lo rows] x 16 bytes, one bulk copy per block.
//   A, weights: per block and weight tile, [4 chunks][128 rows] x 16 bytes
//     of w_hi and the same of w_lo, written by the converter threads.
// Per 16-column step and weight tile: three MMAs into one N-column
// accumulator, (w_hi, x_hi), (w_hi, x_lo), (w_lo, x_hi).
//
// Roles (448 threads = 14 warps, one CTA per SM):
//   warp 0       producer: weight records of a stage (bulk copies issued
//                before griddepcontrol.wait for the first stages: weights do
//                not depend on the preceding kernel), then the image block
//   warp 1       TMEM owner (512 columns: two accumulators of 256)
//   warps 2-9    converters, thread = (weight tile, row): raw quants ->
//                w_hi, w_lo fp16 -> shared memory
//   warps 10-13  epilogue (tcgen05.ld of its lane quarter, scale, store);
//                lane 0 of warps 10 and 11 issues the MMAs of weight tile
//                0 and 1
// CTA tiles are (weight pair, slab, K-slice), slab-major; a CTA walks its
// tiles' blocks as one sequence of stages.
// Ring of RS stages (one 32-column block each); a stage's A and B slots are
// released together by the issuers' tcgen05.commit.  No multicast anywhere.
// Every mbarrier wait is bounded (VXC_WAIT_NS); on expiry the CTA records an
// error code, all roles stop, in-flight copies and MMAs are drained
// (bounded) and TMEM is freed.
#include "vxc_common.cuh"
#include "vxc_ptx.cuh"
#include "vxc_qmat.cuh"
#include "vxc_internal.h"

#include <atomic>

#define GG_THREADS 448         // warp 0 producer, 1 TMEM, 2-9 converters, 10-13 epilogue
#define GG_EPI_WARP0 10        // the epilogue's named barrier counts warps GG_EPI_WARP0.. to the last
static_assert(GG_THREADS == (GG_EPI_WARP0 + 4) * 32, "roles: 14 warps");
#define GG_SMS 148
#define GG_RS 3                 // ring stages
#define GG_SLAB VXC_GEMM_SLAB   // activation rows per CTA tile (one MMA's N)
#define GG_ATILE 8192           // bytes of one 128 x 32 fp16 operand (w_hi or w_lo of one tile)
#define GG_KC 64                // 32-column blocks per K-slice at most

template <int QT>
struct GgCfg {
    static constexpr int QB = QT == 2 ? 16 : 32;
    static constexpr int REC = 128 * QB + 256;
    static constexpr int A_SLOT = 2 * 2 * GG_ATILE;           // 2 weight tiles x (hi, lo)
    static constexpr int B_SLOT = 128 * GG_SLAB;              // one block of a full slab
    static constexpr int RAW_SLOT = 2 * REC;                  // 2 weight tiles' records
    static constexpr int SMEM = GG_RS * (A_SLOT + B_SLOT + RAW_SLOT);
    static_assert(RAW_SLOT % 128 == 0, "slot alignment");
    static_assert(SMEM <= 224 * 1024, "shared memory");
};

struct GgArgs {
    const uint8_t *qs;      // weight records (vxc_qmat.cuh)
    int R, nblk, ntile;
    const uint8_t *img;     // activation image: slab s at img + s * slab_bytes
    size_t slab_bytes;
    const float *xs;        // [M] prescales of the image rows
    int M;
    int ks, nbs;            // K-slices, blocks per slice
    float *out;             // slice s of row m: out[(m >> 6) * slot + s * sst + (m & 63) * R + r]
    size_t slot;
    size_t sstride;         // sst = sstride, or (rows of m's 64-row chunk) * R when 0
    float wscale;
    unsigned int *err;
};

__device__ __forceinline__ __half2 gg_u2h(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }
__device__ __forceinline__ uint32_t gg_h2u(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (both fp16), fp32 accumulate.
__device__ __forceinline__ void mma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Eight weights (elements 8c..8c+7 of a row-block) -> 4 half2 (q - off):
// Q4_0 from one permuted word, Q8_0 from two words (vxc_qmat.cuh layout).
__device__ __forceinline__ void gg_deq_q4(uint32_t w, __half2 *o) {
    const __half2 bias = gg_u2h(0x64086408u);   // 1024 + 8
#pragma unroll
    for (int i = 0; i < 4; i++) o[i] = __hsub2(gg_u2h(((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u), bias);
}
__device__ __forceinline__ void gg_deq_q8(uint32_t w0, uint32_t w1, __half2 *o) {
    const __half2 bias = gg_u2h(0x64806480u);   // 1024 + 128
    const uint32_t a = w0 ^ 0x80808080u, b = w1 ^ 0x80808080u;
    o[0] = __hsub2(gg_u2h(__byte_perm(a, 0x64646464u, 0x4140)), bias);
    o[1] = __hsub2(gg_u2h(__byte_perm(a, 0x64646464u, 0x4342)), bias);
    o[2] = __hsub2(gg_u2h(__byte_perm(b, 0x64646464u, 0x4140)), bias);
    o[3] = __hsub2(gg_u2h(__byte_perm(b, 0x64646464u, 0x4342)), bias);
}

template <int QT>
__global__ void __launch_bounds__(GG_THREADS, 1) k_qgemm_mma(const GgArgs a) {
    using C = GgCfg<QT>;
    constexpr int RS = GG_RS;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[5 * RS + 3];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ float xinv_buf[2][GG_SLAB];   // per tile, double-buffered: written while the last tile's is read

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.nblk;
    const int nwp = (a.ntile + 1) / 2;                 // weight-tile pairs
    const int nsl = (a.M + GG_SLAB - 1) / GG_SLAB;     // activation slabs
    const int ntiles = nwp * nsl * a.ks;
    const int nmine = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    uint8_t *Aring = smem;
    uint8_t *Bring = Aring + RS * C::A_SLOT;
    uint8_t *Raw = Bring + RS * C::B_SLOT;

    const uint32_t bar0 = smem_u32(bars);
    auto raw_full = [&](int s) { return bar0 + 8u * s; };
    auto raw_empty = [&](int s) { return bar0 + 8u * (RS + s); };
    auto b_full = [&](int s) { return bar0 + 8u * (2 * RS + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (3 * RS + s); };
    auto st_empty = [&](int s) { return bar0 + 8u * (4 * RS + s); };
    const uint32_t acc_full = bar0 + 8u * (5 * RS);
    auto fin_bar = [&](int i) { return bar0 + 8u * (5 * RS + 1 + i); };

    // tile t of this CTA's i-th turn: slab-major, then slice, so the CTAs
    // running together share a slab slice (read once) and stream the weight
    // pairs (L2-resident).  Blocks [b0, b0 + nb) of K.
    auto tile_of = [&](int i, int &wp, int &sl, int &ksl, int &b0, int &nb) {
        const int t = (int)blockIdx.x + i * (int)gridDim.x;
        wp = t % nwp;
        const int rest = t / nwp;
        ksl = rest % a.ks;
        sl = rest / a.ks;
        b0 = ksl * a.nbs;
        nb = min(a.nbs, nblk - b0);
    };

    if (tid == 0) {
        for (int s = 0; s < RS; s++) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), 256);
            mbar_init(b_full(s), 1);
            mbar_init(a_full(s), 256);
            mbar_init(st_empty(s), 2);
        }
        mbar_init(acc_full, 2);
        mbar_init(fin_bar(0), 1);
        mbar_init(fin_bar(1), 1);
        abort_flag = 0;
        mbar_init_fence();
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), 512u);
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
            int raw_phase[RS], b_phase[RS];
            for (int s = 0; s < RS; s++) raw_phase[s] = b_phase[s] = -1;
            // stage q = block b of tile i: weight records of the pair's tiles
            auto raw_issue = [&](int q, int wp, int b) {
                const int s = q % RS;
                const int ntw = min(2, a.ntile - 2 * wp);
                mbar_expect_tx(raw_full(s), (uint32_t)(ntw * C::REC));
                for (int tw = 0; tw < ntw; tw++)
                    bulk_g2s(smem_u32(Raw + s * C::RAW_SLOT + tw * C::REC),
                             a.qs + ((size_t)(2 * wp + tw) * nblk + b) * C::REC, (uint32_t)C::REC, raw_full(s));
                raw_phase[s] = q / RS;
            };
            {   // weights first: they do not depend on the preceding kernel
                int q = 0;
                for (int i = 0; i < nmine && q < RS; i++) {
                    int wp, sl, ksl, b0, nb;
                    tile_of(i, wp, sl, ksl, b0, nb);
                    for (int b = b0; b < b0 + nb && q < RS; b++, q++) raw_issue(q, wp, b);
                }
            }
            pdl_wait();
            bool pok = true;
            int q = 0;
            for (int i = 0; i < nmine && pok; i++) {
                int wp, sl, ksl, b0, nb;
                tile_of(i, wp, sl, ksl, b0, nb);
                const int nrow = vxc_img_rows(min(GG_SLAB, a.M - sl * GG_SLAB));
                const uint32_t bytes = (uint32_t)(128 * nrow);
                for (int b = b0; b < b0 + nb; b++, q++) {
                    const int s = q % RS, u = q / RS;
                    if (q >= RS) {
                        if (!mbar_wait(raw_empty(s), (u - 1) & 1, abortp, err, VXC_DERR_TIMEOUT_TMA)) { pok = false; break; }
                        raw_issue(q, wp, b);
                        if (!mbar_wait(st_empty(s), (u - 1) & 1, abortp, err, VXC_DERR_TIMEOUT_MMA)) { pok = false; break; }
                    }
                    mbar_expect_tx(b_full(s), bytes);
                    bulk_g2s(smem_u32(Bring + s * C::B_SLOT), a.img + sl * a.slab_bytes + (size_t)b * 128 * nrow,
                             bytes, b_full(s));
                    b_phase[s] = u;
                }
            }
            if (*abortp) {
                // drain (bounded): the last copies issued into every slot
                for (int s = 0; s < RS; s++) {
                    const uint64_t t0 = vxc_globaltimer();
                    if (raw_phase[s] >= 0)
                        while (!mbar_try(raw_full(s), raw_phase[s] & 1) && vxc_globaltimer() - t0 < 100000000ull) {}
                    if (b_phase[s] >= 0)
                        while (!mbar_try(b_full(s), b_phase[s] & 1) && vxc_globaltimer() - t0 < 100000000ull) {}
                }
            }
        }
    } else if (warp >= 2 && warp < GG_EPI_WARP0) {
        // ------------------------------ converters ------------------------------
        const int ct = tid - 64, tw = ct >> 7, r = ct & 127;
        bool cok = true;
        int q = 0;
        for (int i = 0; i < nmine && cok; i++) {
          int wp, sl, ksl, b0, nb;
          tile_of(i, wp, sl, ksl, b0, nb);
          const bool have = 2 * wp + tw < a.ntile;
          for (int b = 0; b < nb; b++, q++) {
            const int s = q % RS, u = q / RS;
            if (!mbar_wait(raw_full(s), u & 1, abortp, err, VXC_DERR_TIMEOUT_TMA)) { cok = false; break; }
            uint32_t qw[C::QB / 4];
            uint32_t dh = 0;
            if (have) {
                const uint8_t *rec = Raw + s * C::RAW_SLOT + tw * C::REC;
                const uint4 *qp = reinterpret_cast<const uint4 *>(rec + r * C::QB);
#pragma unroll
                for (int v = 0; v < C::QB / 16; v++) {
                    const uint4 w4 = qp[v];
                    qw[4 * v] = w4.x;
                    qw[4 * v + 1] = w4.y;
                    qw[4 * v + 2] = w4.z;
                    qw[4 * v + 3] = w4.w;
                }
                const uint32_t h = reinterpret_cast<const uint16_t *>(rec + 128 * C::QB)[r];
                dh = h | (h << 16);
            }
            mbar_arrive(raw_empty(s));
            // the MMAs of this slot's previous stage have finished reading it
            if (q >= RS && !mbar_wait(st_empty(s), (u - 1) & 1, abortp, err, VXC_DERR_TIMEOUT_MMA)) { cok = false; break; }
            if (have) {
                const __half2 d2 = gg_u2h(dh);
                uint8_t *ahi = Aring + s * C::A_SLOT + (2 * tw) * GG_ATILE + r * 16;
                uint8_t *alo = ahi + GG_ATILE;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    __half2 qh[4];
                    if (QT == 2) gg_deq_q4(qw[c], qh);
                    else gg_deq_q8(qw[2 * c], qw[2 * c + 1], qh);
                    uint32_t hi[4], lo[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const __half2 h = __hmul2(qh[k], d2);
                        hi[k] = gg_h2u(h);
                        lo[k] = gg_h2u(__hfma2(qh[k], d2, __hneg2(h)));
                    }
                    *reinterpret_cast<uint4 *>(ahi + c * 128 * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4 *>(alo + c * 128 * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                }
            }
            fence_proxy_async();   // generic-proxy stores -> the MMAs' async-proxy reads
            mbar_arrive(a_full(s));
          }
        }
    } else if (warp >= GG_EPI_WARP0) {
        // ------------------- epilogue; lane 0 of warps 10, 11 issues the MMAs -------------------
        const int quarter = warp & 3, et = tid - 32 * GG_EPI_WARP0;
        const bool issuer = warp < GG_EPI_WARP0 + 2 && lane == 0;
        const int itw = warp - GG_EPI_WARP0;         // the issuer's weight tile
        const uint32_t tlane = tmem_base + ((uint32_t)(quarter * 32) << 16);
        pdl_wait();   // xs comes from the preceding kernel, which may still read `out`
        bool ok = true;
        int qbase = 0;   // stages of the tiles before tile i
        for (int i = 0; i < nmine; i++) {
            int wp, sl, ksl, b0, nb;
            tile_of(i, wp, sl, ksl, b0, nb);
            const int ntw = min(2, a.ntile - 2 * wp);
            const int msl = min(GG_SLAB, a.M - sl * GG_SLAB);
            const int nrow = vxc_img_rows(msl);
            float *xinv = xinv_buf[i & 1];
            for (int n = et; n < GG_SLAB; n += 128) xinv[n] = n < msl ? a.wscale / a.xs[sl * GG_SLAB + n] : 0.0f;
            // xinv written; the previous tile's accumulators all read
            ok = bar_and(1, 128, ok && !*abortp);
            if (!ok) break;
            if (issuer) {
                tc_fence_after();
                const uint32_t idesc = (1u << 4) | ((uint32_t)(nrow >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
                const uint32_t dcol = tmem_base + (uint32_t)(itw * 256);
                const uint32_t lbo_b = (uint32_t)(2 * nrow * 16);
                bool iok = true;
                for (int b = 0; b < nb; b++) {
                    const int q = qbase + b, s = q % RS, u = q / RS;
                    iok = mbar_wait(a_full(s), u & 1, abortp, err, VXC_DERR_TIMEOUT_MMA) &&
                          mbar_wait(b_full(s), u & 1, abortp, err, VXC_DERR_TIMEOUT_TMA);
                    if (!iok) break;
                    tc_fence_after();
                    if (itw < ntw) {
                        const uint32_t abase = smem_u32(Aring + s * C::A_SLOT + (2 * itw) * GG_ATILE);
                        const uint32_t bbase = smem_u32(Bring + s * C::B_SLOT);
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            const uint64_t ah = sdesc(abase + kk * 2 * 2048, 2048, 128);
                            const uint64_t al = sdesc(abase + GG_ATILE + kk * 2 * 2048, 2048, 128);
                            const uint64_t bh = sdesc(bbase + kk * 2 * lbo_b, lbo_b, 128);
                            const uint64_t bl = sdesc(bbase + kk * 2 * lbo_b + nrow * 16, lbo_b, 128);
                            mma_f16_ss(dcol, ah, bh, idesc, (b | kk) != 0 ? 1u : 0u);
                            mma_f16_ss(dcol, ah, bl, idesc, 1u);
                            mma_f16_ss(dcol, al, bh, idesc, 1u);
                        }
                    }
                    mma_commit(st_empty(s));   // this stage's A and B slots are free once these MMAs end
                }
                mma_commit(acc_full);
            }
            __syncwarp();
            qbase += nb;
            ok = mbar_wait_warp(acc_full, i & 1, abortp, err, VXC_DERR_TIMEOUT_EPI);
            if (ok) {
                tc_fence_after();
                for (int tw = 0; tw < ntw; tw++) {
                    const int row = (2 * wp + tw) * 128 + quarter * 32 + lane;
                    float *dst = a.out + row;
                    for (int cc = 0; cc < nrow / 16; cc++) {
                        uint32_t v[16];
                        tmem_ld16(tlane + (uint32_t)(tw * 256 + cc * 16), v);
                        tmem_wait_ld();
                        tmem_pin<16>(v);
                        if (row < a.R) {
#pragma unroll
                            for (int e = 0; e < 16; e++) {
                                const int n = cc * 16 + e;
                                if (n < msl) {
                                    const int m = sl * GG_SLAB + n, c = m >> 6;
                                    const size_t sst = a.sstride ? a.sstride : (size_t)min(64, a.M - 64 * c) * a.R;
                                    dst[(size_t)c * a.slot + ksl * sst + (size_t)(m & 63) * a.R] =
                                        __uint_as_float(v[e]) * xinv[n];
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
            }
        }
        if (issuer) {
            // nothing this thread issued may still run when TMEM is freed
            mma_commit(fin_bar(itw));
            const uint64_t t0 = vxc_globaltimer();
            while (!mbar_try(fin_bar(itw), 0) && vxc_globaltimer() - t0 < 100000000ull) {}
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512u);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int QT>
static cudaError_t launch_gemm(const GgArgs &ga, int grid, cudaStream_t st) {
    // the attribute is per device: a process that drives several GPUs sets it on each
    static std::atomic<uint64_t> attr_set{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t)1 << dev : 0;
    if (!bit || !(attr_set.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(k_qgemm_mma<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, GgCfg<QT>::SMEM);
        if (e != cudaSuccess) return e;
        if (bit) attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GG_THREADS);
    cfg.dynamicSmemBytes = GgCfg<QT>::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k_qgemm_mma<QT>, ga);
    vxc_count_launches(1);
    return e;
}

int vxc_gemm_ok(const vxc_qmat *w) { return w && (w->type == 2 || w->type == 8) ? 1 : 0; }

// K-slices of the GEMM for a matrix (its K only) and blocks per slice.
static void gemm_split(const vxc_qmat *w, int *ks, int *nbs) {
    int k = (w->nblk + GG_KC - 1) / GG_KC;
    const int b = (w->nblk + k - 1) / k;
    *ks = (w->nblk + b - 1) / b;
    *nbs = b;
}

int vxc_gemm_slices(const vxc_qmat *w) {
    if (!vxc_gemm_ok(w)) return 0;
    int ks, nbs;
    gemm_split(w, &ks, &nbs);
    return ks;
}

size_t vxc_gemm_image_bytes(int K, int M) {
    if (M <= 0 || K <= 0 || K % 32) return 0;
    const int nsl = (M + GG_SLAB - 1) / GG_SLAB;
    const size_t slab = (size_t)(K / 32) * 128 * GG_SLAB;
    return slab * (nsl - 1) + (size_t)(K / 32) * 128 * vxc_img_rows(M - (nsl - 1) * GG_SLAB);
}

int vxc_gemm_run(const vxc_qmat *w, const uint8_t *img, size_t slab_bytes, const float *xs, int M, float *out,
                 size_t slot, size_t sstride, cudaStream_t st) {
    if (!vxc_gemm_ok(w) || !img || !xs || !out || M < 1) {
        vxc_set_error("vxc_gemm_run: bad arguments");
        return -4;
    }
    int ks, nbs;
    gemm_split(w, &ks, &nbs);
    // a chunk's slices [ks][rows][R] must fit its slot, or slices of sstride apart the whole output
    const size_t need = sstride ? (size_t)64 * w->rows : (size_t)ks * 64 * w->rows;
    if (slab_bytes < (size_t)w->nblk * 128 * GG_SLAB || (M > 64 && slot < need) ||
        (sstride && ks > 1 && sstride < (size_t)M * w->rows) || (((uintptr_t)img | slab_bytes) & 15)) {
        vxc_set_error("vxc_gemm_run: slab %zu bytes or output slot %zu floats too small, or image misaligned",
                      slab_bytes, slot);
        return -4;
    }
    GgArgs ga;
    ga.qs = w->qs;
    ga.R = w->rows;
    ga.nblk = w->nblk;
    ga.ntile = w->ntile;
    ga.img = img;
    ga.slab_bytes = slab_bytes;
    ga.xs = xs;
    ga.M = M;
    ga.ks = ks;
    ga.nbs = nbs;
    ga.out = out;
    ga.slot = slot;
    ga.sstride = sstride;
    ga.wscale = w->wscale;
    ga.err = vxc_device_error_ptr();
    const long ntiles = (long)((w->ntile + 1) / 2) * ((M + GG_SLAB - 1) / GG_SLAB) * ks;
    const int grid = (int)(ntiles < GG_SMS ? ntiles : GG_SMS);
    const cudaError_t e = w->type == 2 ? launch_gemm<2>(ga, grid, st) : launch_gemm<8>(ga, grid, st);
    if (e != cudaSuccess) {
        vxc_set_error("vxc_gemm_run: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}
