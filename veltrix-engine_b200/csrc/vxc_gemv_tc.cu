// vxc_gemv_tc.cu — Q4_0 / Q8_0 GEMV on the 5th-generation tensor cores.
//
// y[m][r] = sum_b d[r][b] * D_b[r][m],  D_b[r][m] = sum_{j<32} (q[r][32b+j]-off) * x[m][32b+j]
//
// Exactness strategy (why not a plain bf16 GEMM): the 32 integer weights of a
// block are exact in fp16, and the activation row is prescaled by a power of
// two (exact) and split into fp16 hi + lo parts (22 significant bits).  Both
// parts go through `tcgen05.mma.kind::f16` into the same fp32 TMEM
// accumulator, one fresh accumulator per 32-element block.  The fp16 block
// scale d is applied in fp32 by the epilogue (`tcgen05.ld` + FFMA).  Folding d
// into an fp16 weight, or using a single fp16/bf16 activation, moves the
// logits by ~1e-3 relative through the FFN's |silu| < 0.01 row mask
// (reference src/model.c:583-585); this scheme stays at fp32 level.
//
// CTA = one 128-row weight tile x one K-slice of `nbs` blocks, 6 warps:
//   warps 0-3  row threads: thread t owns weight row t of the tile.  They
//              expand raw nibbles/int8 to fp16 into the A stage (K-major,
//              no swizzle), then run the epilogue of the previous stage.
//   warp 4     TMA producer: cp.async.bulk of raw quant + scale bytes into a
//              ring of RS stages (the tile's K-range is contiguous in HBM).
//   warp 5     TMEM owner; lane 0 issues the MMAs and tcgen05.commit.
// The activation operand B (all nbs blocks, hi and lo) is built once per CTA
// in shared memory.  No TMA multicast anywhere (multi-GPU safe).
//
// Every mbarrier wait is bounded (VXC_WAIT_NS); on expiry the CTA records an
// error code, stops issuing work, drains what it issued and frees its TMEM.
#include "vxc_common.cuh"
#include "vxc_qmat.cuh"
#include "vxc_internal.h"

#include <stdio.h>

#define TC_KB 2          // blocks per pipeline stage
#define TC_RS 6          // raw-weight ring stages
#define TC_ROWS 128

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait.  Returns false when the CTA is aborting (this wait expired,
// or another role's did).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                          unsigned int *err, unsigned int code) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
        if ((it & 255u) == 255u) {
            uint64_t now = vxc_globaltimer();
            if (t0 == 0) t0 = now;
            else if (now - t0 > VXC_WAIT_NS) {
                *abort_flag = 1;
                vxc_flag_error(err, code);
                return false;
            }
        }
    }
}

// Warp-uniform wait for the row threads: every lane waits, and the warp
// proceeds only if all lanes saw the phase complete, so .sync.aligned
// tcgen05 instructions that follow are executed by all lanes or by none.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                               unsigned int *err, unsigned int code) {
    bool ok = mbar_wait(bar, parity, abort_flag, err, code);
    return __all_sync(0xffffffffu, ok) != 0;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major, no-swizzle shared-memory matrix descriptor: core matrices of
// 8 rows x 16 bytes; LBO = byte distance between the two 16-byte K chunks of
// one MMA-K step, SBO = byte distance between consecutive 8-row groups.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;   // descriptor version for sm_100
    return d;                 // base offset 0, layout SWIZZLE_NONE
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Dequantisers: raw row-block -> 4 x 16-byte chunks of fp16 (elements 8c..8c+7)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}

// Q4_0 permuted word -> 4 half2 (q-8) of elements (8j+2i, 8j+2i+1), i=0..3.
__device__ __forceinline__ uint4 deq_q4_word(uint32_t w) {
    const uint32_t magic = 0x64006400u;     // fp16 1024.0 in both halves
    const uint32_t bias = 0x64086408u;      // fp16 1032.0 = 1024 + 8
    uint4 o;
    o.x = h2_sub((w & 0x000F000Fu) | magic, bias);
    o.y = h2_sub(((w >> 4) & 0x000F000Fu) | magic, bias);
    o.z = h2_sub(((w >> 8) & 0x000F000Fu) | magic, bias);
    o.w = h2_sub(((w >> 12) & 0x000F000Fu) | magic, bias);
    return o;
}

// Q8_0 two words (8 int8) -> 4 half2.
__device__ __forceinline__ uint4 deq_q8_words(uint32_t w0, uint32_t w1) {
    const uint32_t bias = 0x64806480u;      // fp16 1152.0 = 1024 + 128
    uint32_t a = w0 ^ 0x80808080u, b = w1 ^ 0x80808080u;
    uint4 o;
    o.x = h2_sub(__byte_perm(a, 0x64646464u, 0x4140), bias);
    o.y = h2_sub(__byte_perm(a, 0x64646464u, 0x4342), bias);
    o.z = h2_sub(__byte_perm(b, 0x64646464u, 0x4140), bias);
    o.w = h2_sub(__byte_perm(b, 0x64646464u, 0x4342), bias);
    return o;
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
struct TcSmem {
    uint32_t raw_full[TC_RS], raw_empty[TC_RS];
    uint32_t a_full[2], mma_done[2], acc_empty[2];
    uint32_t final_bar;
};

template <int QT, int NT>   // QT: 2 (Q4_0) or 8 (Q8_0); N = 16*NT activation columns
__global__ void __launch_bounds__(192, 1)
k_qgemv_tc(const uint8_t *__restrict__ qs, const uint16_t *__restrict__ sc, int R, int nblk,
           const float *__restrict__ x, int M, float *__restrict__ out, int nbs, unsigned int *err) {
    constexpr int N = 16 * NT;
    constexpr int QB = QT == 2 ? 16 : 32;                 // quant bytes per row-block
    constexpr int RAW_Q = TC_KB * TC_ROWS * QB;            // quant bytes per stage
    constexpr int RAW_S = TC_KB * TC_ROWS * 2;             // scale bytes per stage
    constexpr int A_STAGE = TC_KB * 4 * TC_ROWS * 16;      // fp16 A bytes per stage
    constexpr uint32_t TMEM_COLS = (2 * TC_KB * N <= 32) ? 32 : (2 * TC_KB * N <= 64) ? 64
                                  : (2 * TC_KB * N <= 128) ? 128 : (2 * TC_KB * N <= 256) ? 256 : 512;

    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bars[TC_RS * 2 + 7];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ int stages_consumed;
    __shared__ float xscale[N];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, slice = blockIdx.y;
    const int b0 = slice * nbs;
    const int nb = min(nbs, nblk - b0);        // blocks in this slice (even)
    const int NG = nb / TC_KB;
    const int K = nblk * 32;

    uint8_t *Bs = smem;                                     // nb*8 chunks x N rows x 16 B
    uint8_t *As = Bs + (size_t)nbs * 8 * N * 16;            // 2 stages
    uint8_t *RawQ = As + 2 * A_STAGE;                       // TC_RS stages
    uint8_t *RawS = RawQ + TC_RS * RAW_Q;

    const uint32_t bar0 = smem_u32(bars);
    auto raw_full = [&](int s) { return bar0 + 8u * s; };
    auto raw_empty = [&](int s) { return bar0 + 8u * (TC_RS + s); };
    auto a_full = [&](int j) { return bar0 + 8u * (2 * TC_RS + j); };
    auto mma_done = [&](int j) { return bar0 + 8u * (2 * TC_RS + 2 + j); };
    auto acc_empty = [&](int j) { return bar0 + 8u * (2 * TC_RS + 4 + j); };
    const uint32_t final_bar = bar0 + 8u * (2 * TC_RS + 6);

    if (tid == 0) {
        for (int s = 0; s < TC_RS; s++) { mbar_init(raw_full(s), 1); mbar_init(raw_empty(s), 128); }
        for (int j = 0; j < 2; j++) { mbar_init(a_full(j), 128); mbar_init(mma_done(j), 1); mbar_init(acc_empty(j), 128); }
        mbar_init(final_bar, 1);
        abort_flag = 0;
        stages_consumed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;
    volatile int *abortp = &abort_flag;

    if (warp == 4) {
        // ------------------------------ producer -------------------------------
        if (lane == 0) {
            int issued = 0;
            for (int g = 0; g < NG; g++) {
                int s = g % TC_RS;
                if (g >= TC_RS && !mbar_wait(raw_empty(s), ((g - TC_RS) / TC_RS) & 1, abortp, err, VXC_DERR_TIMEOUT_TMA))
                    break;
                size_t slot = ((size_t)tile * nblk + b0 + (size_t)g * TC_KB) * TC_ROWS;
                mbar_expect_tx(raw_full(s), RAW_Q + RAW_S);
                bulk_g2s(smem_u32(RawQ + s * RAW_Q), qs + slot * QB, RAW_Q, raw_full(s));
                bulk_g2s(smem_u32(RawS + s * RAW_S), sc + slot, RAW_S, raw_full(s));
                issued = g + 1;
            }
            if (*abortp) {
                // drain: wait (bounded) for copies that no row thread consumed
                for (int g = stages_consumed; g < issued; g++) {
                    uint64_t t0 = vxc_globaltimer();
                    while (!mbar_try(raw_full(g % TC_RS), (g / TC_RS) & 1) &&
                           vxc_globaltimer() - t0 < 100000000ull) {}
                }
            }
        }
    } else if (warp < 4) {
        // ------------------------------ row threads ----------------------------
        // 1. activation operand B: per-row power-of-two prescale, fp16 hi/lo
        for (int m = warp; m < N; m += 4) {
            float mx = 0.0f;
            if (m < M)
                for (int j = lane; j < nb * 32; j += 32) mx = fmaxf(mx, fabsf(x[(size_t)m * K + (size_t)b0 * 32 + j]));
            mx = warp_max(mx);
            if (lane == 0) {
                int e = 0;
                if (mx > 0.0f) { frexpf(mx, &e); e = 15 - e; }
                e = max(-120, min(120, e));
                xscale[m] = ldexpf(1.0f, e);
            }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        for (int i = tid; i < N * nb * 4; i += 128) {
            int m = i % N, rest = i / N;
            int c = rest & 3, b = rest >> 2;              // chunk of 8 elements within block b
            uint4 hi = make_uint4(0, 0, 0, 0), lo = make_uint4(0, 0, 0, 0);
            if (m < M) {
                const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)m * K + (size_t)(b0 + b) * 32 + c * 8);
                float4 v0 = src[0], v1 = src[1];
                float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                float s = xscale[m];
                uint32_t h[4], l[4];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    float a0 = v[2 * k] * s, a1 = v[2 * k + 1] * s;
                    __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
                    __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
                    h[k] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                    l[k] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
                }
                hi = make_uint4(h[0], h[1], h[2], h[3]);
                lo = make_uint4(l[0], l[1], l[2], l[3]);
            }
            *reinterpret_cast<uint4 *>(Bs + ((size_t)(b * 8 + c) * N + m) * 16) = hi;
            *reinterpret_cast<uint4 *>(Bs + ((size_t)(b * 8 + 4 + c) * N + m) * 16) = lo;
        }
        fence_proxy_async();
        asm volatile("bar.sync 2, 160;" ::: "memory");     // B ready -> MMA warp

        float yacc[N];
#pragma unroll
        for (int m = 0; m < N; m++) yacc[m] = 0.0f;
        float dprev[TC_KB], dcur[TC_KB];
        const uint32_t trow = tmem_base + ((uint32_t)(warp * 32) << 16);

        auto epilogue = [&](int g, const float *dsc) -> bool {
            int j = g & 1;
            if (!mbar_wait_warp(mma_done(j), (g >> 1) & 1, abortp, err, VXC_DERR_TIMEOUT_EPI)) return false;
            tc_fence_after();
#pragma unroll
            for (int kb = 0; kb < TC_KB; kb++) {
                float dv[N];
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
                    tmem_ld16(trow + (uint32_t)((j * TC_KB + kb) * N + nt * 16), &dv[nt * 16]);
                tmem_wait_ld();
#pragma unroll
                for (int m = 0; m < N; m++) yacc[m] = fmaf(dsc[kb], dv[m], yacc[m]);
            }
            tc_fence_before();
            mbar_arrive(acc_empty(j));
            return true;
        };

        bool ok = true;
        for (int g = 0; g < NG && ok; g++) {
            int s = g % TC_RS;
            if (!mbar_wait_warp(raw_full(s), (g / TC_RS) & 1, abortp, err, VXC_DERR_TIMEOUT_TMA)) { ok = false; break; }
            uint32_t qw[TC_KB][QB / 4];
#pragma unroll
            for (int kb = 0; kb < TC_KB; kb++) {
                const uint4 *src = reinterpret_cast<const uint4 *>(RawQ + s * RAW_Q + (kb * TC_ROWS + tid) * QB);
#pragma unroll
                for (int v = 0; v < QB / 16; v++) {
                    uint4 q = src[v];
                    qw[kb][4 * v] = q.x; qw[kb][4 * v + 1] = q.y; qw[kb][4 * v + 2] = q.z; qw[kb][4 * v + 3] = q.w;
                }
                dcur[kb] = vxc_h2f(reinterpret_cast<const uint16_t *>(RawS + s * RAW_S)[kb * TC_ROWS + tid]);
            }
            mbar_arrive(raw_empty(s));
            if (tid == 0) atomicAdd(&stages_consumed, 1);
            int j = g & 1;
            uint8_t *Aj = As + j * A_STAGE;
#pragma unroll
            for (int kb = 0; kb < TC_KB; kb++)
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint4 h = QT == 2 ? deq_q4_word(qw[kb][c]) : deq_q8_words(qw[kb][2 * c], qw[kb][2 * c + 1]);
                    *reinterpret_cast<uint4 *>(Aj + ((kb * 4 + c) * TC_ROWS + tid) * 16) = h;
                }
            fence_proxy_async();
            mbar_arrive(a_full(j));
            if (g > 0 && !epilogue(g - 1, dprev)) { ok = false; break; }
#pragma unroll
            for (int kb = 0; kb < TC_KB; kb++) dprev[kb] = dcur[kb];
        }
        if (ok && NG > 0) ok = epilogue(NG - 1, dprev);
        const int row = tile * TC_ROWS + tid;
        if (ok && row < R) {
            float *dst = gridDim.y == 1 ? out : out + (size_t)slice * M * R;
#pragma unroll
            for (int m = 0; m < N; m++)
                if (m < M) dst[(size_t)m * R + row] = yacc[m] / xscale[m];
        }
    } else {
        // ------------------------------ MMA warp -------------------------------
        asm volatile("bar.sync 2, 160;" ::: "memory");
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);
            const uint32_t bbase = smem_u32(Bs), abase = smem_u32(As);
            int issued = 0;
            for (int g = 0; g < NG; g++) {
                int j = g & 1;
                if (!mbar_wait(a_full(j), (g >> 1) & 1, abortp, err, VXC_DERR_TIMEOUT_MMA)) break;
                if (g >= 2 && !mbar_wait(acc_empty(j), ((g - 2) >> 1) & 1, abortp, err, VXC_DERR_TIMEOUT_MMA)) break;
                tc_fence_after();
#pragma unroll
                for (int kb = 0; kb < TC_KB; kb++) {
                    const uint32_t dacc = tmem_base + (uint32_t)((j * TC_KB + kb) * N);
                    const int bl = g * TC_KB + kb;
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        uint64_t ad = sdesc(abase + j * A_STAGE + (kb * 4 + 2 * kk) * TC_ROWS * 16, TC_ROWS * 16, 128);
                        uint64_t bh = sdesc(bbase + (bl * 8 + 2 * kk) * N * 16, N * 16, 128);
                        uint64_t blo = sdesc(bbase + (bl * 8 + 4 + 2 * kk) * N * 16, N * 16, 128);
                        mma_f16(dacc, ad, bh, idesc, kk > 0 ? 1u : 0u);
                        mma_f16(dacc, ad, blo, idesc, 1u);
                    }
                }
                mma_commit(mma_done(j));
                issued = g + 1;
            }
            // make sure nothing this thread issued is still running before TMEM is freed
            mma_commit(final_bar);
            uint64_t t0 = vxc_globaltimer();
            while (!mbar_try(final_bar, 0) && vxc_globaltimer() - t0 < 100000000ull) {}
            (void)issued;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct TcPlan {
    int nt;     // N / 16
    int nbs;    // blocks per slice (even)
    int ks;     // slices
    size_t smem;
};

static size_t tc_smem_bytes(int qt, int N, int nbs) {
    int QB = qt == 2 ? 16 : 32;
    size_t b = (size_t)nbs * 8 * N * 16;
    size_t a = 2ull * TC_KB * 4 * TC_ROWS * 16;
    size_t raw = (size_t)TC_RS * (TC_KB * TC_ROWS * QB + TC_KB * TC_ROWS * 2);
    return b + a + raw + 1024;
}

static bool tc_plan(const vxc_qmat *w, int M, TcPlan *p) {
    if (M < 1 || M > 64 || (w->nblk % TC_KB) != 0) return false;
    int nt = (M + 15) / 16;
    int N = 16 * nt;
    int nbs_max = (96 * 1024) / (N * 128);
    nbs_max -= nbs_max % TC_KB;
    if (nbs_max < TC_KB) return false;
    int ks_min = (w->nblk + nbs_max - 1) / nbs_max;
    int ks = (2 * 148 + w->ntile - 1) / w->ntile;
    if (ks < ks_min) ks = ks_min;
    if (ks > w->nblk / TC_KB) ks = w->nblk / TC_KB;
    int nbs = (w->nblk + ks - 1) / ks;
    nbs += nbs % TC_KB;
    if (nbs > nbs_max) nbs = nbs_max;
    ks = (w->nblk + nbs - 1) / nbs;
    p->nt = nt;
    p->nbs = nbs;
    p->ks = ks;
    p->smem = tc_smem_bytes(w->type, N, nbs);
    return true;
}

template <int QT, int NT>
static cudaError_t launch_tc(const vxc_qmat *w, const float *x, int M, float *dst, const TcPlan &p,
                             cudaStream_t st) {
    static bool attr_set = false;   // one flag per template instance
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(k_qgemv_tc<QT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    dim3 grid(w->ntile, p.ks);
    (k_qgemv_tc<QT, NT><<<grid, 192, p.smem, st>>>(w->qs, w->sc, w->rows, w->nblk, x, M, dst, p.nbs,
                                                   vxc_device_error_ptr()), vxc_count_launches(1));
    return cudaGetLastError();
}

extern "C" size_t vxc_qgemv_workspace_bytes(const vxc_qmat *w, int M) {
    if (!w || M <= 0) return 0;
    TcPlan p;
    if (M <= 64 && tc_plan(w, M, &p)) return p.ks > 1 ? (size_t)p.ks * M * w->rows * sizeof(float) : 0;
    if (M > 64) {
        // processed in chunks of 64 rows
        TcPlan q;
        if (tc_plan(w, 64, &q)) return q.ks > 1 ? (size_t)q.ks * 64 * w->rows * sizeof(float) : 0;
    }
    return vxc_qgemv_simt_ws(w, M);
}

static int qgemv_tc_chunk(const vxc_qmat *w, const float *x, int M, float *y, void *ws, size_t wsb,
                          cudaStream_t st) {
    TcPlan p;
    if (!tc_plan(w, M, &p)) return 1;   // not handled here
    size_t need = p.ks > 1 ? (size_t)p.ks * M * w->rows * sizeof(float) : 0;
    if (need > wsb || (need && !ws)) {
        vxc_set_error("vxc_qgemv: workspace %zu < %zu bytes", wsb, need);
        return -4;
    }
    float *dst = p.ks > 1 ? (float *)ws : y;
    cudaError_t e;
    if (w->type == 2) {
        switch (p.nt) {
            case 1: e = launch_tc<2, 1>(w, x, M, dst, p, st); break;
            case 2: e = launch_tc<2, 2>(w, x, M, dst, p, st); break;
            case 3: e = launch_tc<2, 3>(w, x, M, dst, p, st); break;
            default: e = launch_tc<2, 4>(w, x, M, dst, p, st); break;
        }
    } else {
        switch (p.nt) {
            case 1: e = launch_tc<8, 1>(w, x, M, dst, p, st); break;
            case 2: e = launch_tc<8, 2>(w, x, M, dst, p, st); break;
            case 3: e = launch_tc<8, 3>(w, x, M, dst, p, st); break;
            default: e = launch_tc<8, 4>(w, x, M, dst, p, st); break;
        }
    }
    if (e != cudaSuccess) { vxc_set_error("vxc_qgemv: %s", cudaGetErrorString(e)); return -3; }
    if (p.ks > 1) return vxc_launch_splitk_reduce(dst, p.ks, M, w->rows, y, st);
    return 0;
}

extern "C" int vxc_qgemv(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
                         size_t workspace_bytes, void *stream) {
    if (!w || !x || !y || M <= 0) { vxc_set_error("vxc_qgemv: bad arguments"); return -4; }
    if (((uintptr_t)x & 15) != 0) { vxc_set_error("vxc_qgemv: x must be 16-byte aligned"); return -4; }
    cudaStream_t st = (cudaStream_t)stream;
    for (int m0 = 0; m0 < M; m0 += 64) {
        int mc = M - m0 < 64 ? M - m0 : 64;
        int rc = qgemv_tc_chunk(w, x + (size_t)m0 * w->cols, mc, y + (size_t)m0 * w->rows, workspace,
                                workspace_bytes, st);
        if (rc == 1)
            rc = vxc_qgemv_simt(w, x + (size_t)m0 * w->cols, mc, y + (size_t)m0 * w->rows, workspace,
                                workspace_bytes, stream);
        if (rc) return rc;
    }
    return 0;
}
