// vxc_gemv_skinny.cu — CUDA-core GEMV of a Q4_0 / Q8_0 matrix with one or
// two activation rows (M <= VXC_SKINNY_MAX_M: a draft step of one sequence,
// or target-only decoding), judged against HBM bandwidth.  With more rows
// the tensor-core kernel (vxc_gemv_tc.cu) is faster: here every weight costs
// M fused multiply-adds on the CUDA cores.
//
// Math (reference src/quantize.c:728-750 for Q4_0, src/model.c:234-244 for
// Q8_0):  y[m][r] = sum_b d[r][b] * sum_{j<32} (q[r][32b+j] - off) x[m][32b+j]
// with the per-block inner sums in fp32 and the block terms accumulated in
// fp32; only the summation order differs from the reference.
//
// Work split.  The work is cut into units of 32 rows x one K-slice of bps
// blocks (bps a multiple of SK_WARPS * SK_BPS); a persistent CTA of SK_WARPS
// warps takes units blockIdx.x, blockIdx.x + gridDim.x, ..., and within a
// unit warp w takes the pairs of consecutive blocks 2w, 2w + 2 SK_WARPS, ...
// Each warp streams its block pairs through its own ring of shared-memory
// slots with cp.async (per block the unit's 32 rows of one record, one
// contiguous span, plus their 32 scales), so all but one slot stay in flight
// per warp across unit boundaries; two blocks per step halve the per-element
// cost of the ring and cursor bookkeeping.  The
// first copies are issued before griddepcontrol.wait: the weights do not
// depend on the kernel that produces x.  Lane l covers rows rr, rr + 8,
// rr + 16, rr + 24 of the unit (rr = l / 4) and the element group g = l % 4
// (elements 8g..8g+7 of every 32-column block); it reads two float4 of every
// activation row per block, shared by its four rows.  At the end of a unit
// the 4 lanes of a row (shuffles) and the warps (shared memory) are summed;
// K-slices (ks > 1) leave fp32 partials part[slice][m][row] that the consumer
// adds, as the tensor-core GEMV's.  ks depends on the matrix shape only,
// never on M, and M = 1 and M = 2 share one accumulation order, so a row's
// result does not depend on how many rows share the launch.
//
// Dequantisation without conversion instructions.  A byte b placed in the
// low byte of the bit pattern of 2^23 is the float 2^23 + b exactly (it lands
// in the lowest significand bits of that binade), so one byte permute makes
// the float and one packed add of -(2^23 + off) gives b - off.  Q4_0 nibbles
// are first split into bytes (two masks and a shift per 8 elements); Q8_0
// bytes are made unsigned by flipping their top bits.  The products and sums
// run as packed fp32 pairs (FFMA2), two elements per instruction.
#include "vxc_common.cuh"
#include "vxc_qmat.cuh"
#include "vxc_ptx.cuh"
#include "vxc_internal.h"

#include <stdio.h>
#include <atomic>

#define SK_WARPS 8

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// 2^e as an fp32 bit pattern
#define SK_POW2(e) ((uint32_t)(127 + (e)) << 23)

// Q4_0: the 8 elements of word w (elements 8g + 2i, 8g + 2i + 1 in pair i).
// The low and high nibbles are split into bytes, and each byte is placed into
// the low byte of the pattern of 2^23 by one byte permute (PRMT), so every
// element uses the same magic constant and the same packed offset.
__device__ __forceinline__ void sk_dequant_q4(uint32_t w, float2 (&f)[4]) {
    const uint32_t lo = w & 0x0F0F0F0Fu;          // bytes: elements 0, 4, 1, 5 (of 8g..8g+7)
    const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;   // bytes: elements 2, 6, 3, 7
    const uint32_t k = SK_POW2(23);
    const float c = -(8388608.0f + 8.0f);
    const float2 off = f2(c, c);
    // selector 0x744b: byte b of the word, two zero bytes of k, then k's top byte
    f[0] = __fadd2_rn(f2(__uint_as_float(__byte_perm(lo, k, 0x7440)), __uint_as_float(__byte_perm(lo, k, 0x7442))), off);
    f[1] = __fadd2_rn(f2(__uint_as_float(__byte_perm(hi, k, 0x7440)), __uint_as_float(__byte_perm(hi, k, 0x7442))), off);
    f[2] = __fadd2_rn(f2(__uint_as_float(__byte_perm(lo, k, 0x7441)), __uint_as_float(__byte_perm(lo, k, 0x7443))), off);
    f[3] = __fadd2_rn(f2(__uint_as_float(__byte_perm(hi, k, 0x7441)), __uint_as_float(__byte_perm(hi, k, 0x7443))), off);
}

// Q8_0: 4 int8 elements of word w (natural order) as pairs (0,1), (2,3): the
// top bits flipped (unsigned = value + 128), each byte permuted into 2^23's pattern.
__device__ __forceinline__ void sk_dequant_q8(uint32_t w, float2 &p01, float2 &p23) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t k = SK_POW2(23);
    const float c = -(8388608.0f + 128.0f);
    const float2 off = f2(c, c);
    p01 = __fadd2_rn(f2(__uint_as_float(__byte_perm(u, k, 0x7440)), __uint_as_float(__byte_perm(u, k, 0x7441))), off);
    p23 = __fadd2_rn(f2(__uint_as_float(__byte_perm(u, k, 0x7442)), __uint_as_float(__byte_perm(u, k, 0x7443))), off);
}

// the lane's 8 products w * x for one activation row (x0, x1 = its 8 values),
// summed in two interleaved halves
__device__ __forceinline__ float2 sk_dot8(const float2 (&f)[4], float4 x0, float4 x1) {
    float2 p = __fmul2_rn(f[0], f2(x0.x, x0.y));
    p = __ffma2_rn(f[1], f2(x0.z, x0.w), p);
    p = __ffma2_rn(f[2], f2(x1.x, x1.y), p);
    return __ffma2_rn(f[3], f2(x1.z, x1.w), p);
}

template <int QT>
__device__ __forceinline__ void sk_dequant(const uint32_t (&q)[QT == 2 ? 1 : 2], float2 (&f)[4]) {
    if (QT == 2) {
        sk_dequant_q4(q[0], f);
    } else {
        sk_dequant_q8(q[0], f[0], f[1]);
        sk_dequant_q8(q[QT == 2 ? 0 : 1], f[2], f[3]);
    }
}

__device__ __forceinline__ void sk_cp16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void sk_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void sk_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Rows per lane, rows of a unit, blocks per pipeline step.
#define SK_RPL 4
#define SK_UROWS (8 * SK_RPL)
#define SK_BPS 2

// CTAs per SM the kernel is built for (registers).
template <int MAXM>
struct SkOcc {
    static constexpr int CTAS = 4;
};

// Ring slot of one warp: SK_BPS consecutive blocks, each the quants of the
// unit's rows in one record followed by their scales.
template <int QT, int MAXM>
struct SkSlot {
    static constexpr int QB = QT == 2 ? 16 : 32;
    static constexpr int QBYTES = SK_UROWS * QB;
    static constexpr int BLK = QBYTES + SK_UROWS * 2;   // 576 or 1088, multiples of 16
    static constexpr int BYTES = SK_BPS * BLK;
    static constexpr int BUDGET = 225 * 1024 / SkOcc<MAXM>::CTAS - 2048 - SK_WARPS * SK_UROWS * MAXM * 4;
    static constexpr int STAGES = BUDGET / (SK_WARPS * BYTES) < 8 ? BUDGET / (SK_WARPS * BYTES) : 8;
    static constexpr size_t SMEM = (size_t)SK_WARPS * STAGES * BYTES + (size_t)SK_WARPS * SK_UROWS * MAXM * 4;
};

template <int QT, int MAXM>
__global__ void __launch_bounds__(SK_WARPS * 32, SkOcc<MAXM>::CTAS)
    k_qgemv_skinny(const uint8_t *__restrict__ qs, int R, int nblk, float wscale, const float *__restrict__ x,
                   int ldx, int M, float *__restrict__ out, int bps, int ks) {
    using Sl = SkSlot<QT, MAXM>;
    constexpr int RPL = SK_RPL, ROWS = SK_UROWS;
    constexpr int QB = Sl::QB, SLOT = Sl::BYTES, S = Sl::STAGES;
    constexpr int REC = VXC_TILE_ROWS * QB + 256;
    constexpr int NW = QT == 2 ? 1 : 2;
    static_assert(S >= 3, "ring too small");
    static_assert(MAXM <= VXC_SKINNY_MAX_M, "activation rows held in registers");
    extern __shared__ __align__(16) uint8_t sk_smem[];     // [SK_WARPS][S][SLOT], then red
    float *red = reinterpret_cast<float *>(sk_smem + SK_WARPS * S * SLOT);   // [SK_WARPS][ROWS * MAXM]
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, rr = lane >> 2, g = lane & 3;
    const int G = (R + ROWS - 1) / ROWS;
    const int n_units = G * ks;
    const int my_units = (int)blockIdx.x < n_units ? (n_units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nbw = bps / (SK_WARPS * SK_BPS);   // steps per unit
    uint8_t *ring = sk_smem + (size_t)w * S * SLOT;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    // cursor over this warp's steps: unit (uu-th of this CTA), step kb in it,
    // first block b of the step
    struct Cur {
        int uu, kb, b, rg, sl;
    };
    auto unit_start = [&](Cur &c) {
        const int u = (int)blockIdx.x + c.uu * (int)gridDim.x;
        c.rg = u / ks;
        c.sl = u - c.rg * ks;
        c.b = c.sl * bps + w * SK_BPS;
        c.kb = 0;
    };
    auto advance = [&](Cur &c) {
        if (++c.kb == nbw) {
            c.uu++;
            unit_start(c);
        } else {
            c.b += SK_WARPS * SK_BPS;
        }
    };
    Cur ic, cc;
    ic.uu = cc.uu = 0;
    unit_start(ic);
    unit_start(cc);
    int islot = 0, cslot = 0;
    auto issue = [&]() {
        if (ic.uu < my_units) {
            const int r0 = ic.rg * ROWS;
            const uint8_t *rec0 = qs + ((size_t)(r0 / VXC_TILE_ROWS) * nblk + ic.b) * REC;
            const int tr0 = r0 % VXC_TILE_ROWS;
            const uint32_t dst = ring_s + islot * SLOT;
#pragma unroll
            for (int k = 0; k < SK_BPS; k++)
                if (ic.b + k < nblk) {
                    const uint8_t *rec = rec0 + (size_t)k * REC;
#pragma unroll
                    for (int c = lane; c < Sl::QBYTES / 16; c += 32)
                        sk_cp16(dst + k * Sl::BLK + 16 * c, rec + tr0 * QB + 16 * c);
                    if (lane < ROWS * 2 / 16)
                        sk_cp16(dst + k * Sl::BLK + Sl::QBYTES + 16 * lane,
                                rec + VXC_TILE_ROWS * QB + tr0 * 2 + 16 * lane);
                }
            advance(ic);
        }
        sk_commit();   // one group per step, empty or not, so the waits below count steps
        islot = islot + 1 == S ? 0 : islot + 1;
    };
    // packed accumulators (even / odd element halves) for every M: one
    // accumulation order, so a row's result does not depend on M
    float2 acc[RPL][MAXM];
#pragma unroll
    for (int i = 0; i < RPL; i++)
#pragma unroll
        for (int m = 0; m < MAXM; m++) acc[i][m] = f2(0.0f, 0.0f);
    auto accum = [&](float2 &a, float d, float2 p) { a = __ffma2_rn(f2(d, d), p, a); };
    // the weights do not depend on the preceding kernel: start their copies,
    // then wait for it before reading x or writing the output
#pragma unroll
    for (int j = 0; j < S - 1; j++) issue();
    pdl_trigger();
    pdl_wait();
    const int J = my_units * nbw;
    for (int j = 0; j < J; j++) {
        issue();
        sk_wait<S - 1>();
        __syncwarp();
#pragma unroll
        for (int k = 0; k < SK_BPS; k++) {
            const int b = cc.b + k;
            if (b < nblk) {
                const uint8_t *blk = ring + cslot * SLOT + k * Sl::BLK;
                const uint16_t *sc = reinterpret_cast<const uint16_t *>(blk + Sl::QBYTES);
                const float *xb = x + (size_t)b * 32 + g * 8;
                auto rowq = [&](int i, uint32_t (&q)[NW]) {
                    if constexpr (QT == 2) {
                        q[0] = reinterpret_cast<const uint32_t *>(blk + (rr + 8 * i) * QB)[g];
                    } else {
                        const uint2 u2 = reinterpret_cast<const uint2 *>(blk + (rr + 8 * i) * QB)[g];
                        q[0] = u2.x;
                        q[NW - 1] = u2.y;
                    }
                };
                // every activation row of the block in registers, rows outer
                float4 xr[MAXM][2];
#pragma unroll
                for (int m = 0; m < MAXM; m++)
                    if (m < M) {
                        xr[m][0] = __ldg(reinterpret_cast<const float4 *>(xb + (size_t)m * ldx));
                        xr[m][1] = __ldg(reinterpret_cast<const float4 *>(xb + (size_t)m * ldx) + 1);
                    }
#pragma unroll
                for (int i = 0; i < RPL; i++) {
                    uint32_t q[NW];
                    rowq(i, q);
                    float2 f[4];
                    sk_dequant<QT>(q, f);
                    const float d = vxc_h2f(sc[rr + 8 * i]);
#pragma unroll
                    for (int m = 0; m < MAXM; m++)
                        if (m < M) accum(acc[i][m], d, sk_dot8(f, xr[m][0], xr[m][1]));
                }
            }
        }
        __syncwarp();   // every lane has read the slot before a later step refills it
        cslot = cslot + 1 == S ? 0 : cslot + 1;
        if (cc.kb == nbw - 1) {   // end of a unit: the 4 lanes of a row, then the warps
#pragma unroll
            for (int i = 0; i < RPL; i++)
#pragma unroll
                for (int m = 0; m < MAXM; m++) {
                    float v = acc[i][m].x + acc[i][m].y;
                    acc[i][m] = f2(0.0f, 0.0f);
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    if (g == 0) red[(w * ROWS + rr + 8 * i) * MAXM + m] = v;
                }
            __syncthreads();
            const int r0 = cc.rg * ROWS;
            for (int t = threadIdx.x; t < ROWS * M; t += blockDim.x) {
                const int m = t / ROWS, row = t % ROWS;
                float v = red[row * MAXM + m];
#pragma unroll
                for (int i = 1; i < SK_WARPS; i++) v += red[(i * ROWS + row) * MAXM + m];
                if (r0 + row < R) out[((size_t)cc.sl * M + m) * R + r0 + row] = v * wscale;
            }
            __syncthreads();   // red is refilled at the next unit's end
        }
        advance(cc);
    }
    sk_wait<0>();   // no copy is left in flight at exit
}

static int sk_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
            sms = n;
        else
            sms = 148;
    }
    return sms;
}

#define SK_CTAS_SPLIT 4   // CTAs per SM assumed when choosing K-slices (the same for every M)

// K-slices: the number of slices ks (bps blocks each, a multiple of
// SK_WARPS * SK_BPS, at least 2 steps per warp when the matrix is sliced)
// whose units spread most evenly over the persistent CTAs, from the shape alone.
static void sk_split(const vxc_qmat *w, int *ks_out, int *bps_out) {
    const int q = SK_WARPS * SK_BPS;
    const long slots = (long)sk_sms() * SK_CTAS_SPLIT;
    const long G = (w->rows + SK_UROWS - 1) / SK_UROWS;
    int best_ks = 1, best_bps = (w->nblk + q - 1) / q * q;
    double best = -1.0;
    for (int ks = 1; ks <= 16; ks++) {
        const int bps = ((w->nblk + ks - 1) / ks + q - 1) / q * q;
        const int k = (w->nblk + bps - 1) / bps;
        if (k != ks) continue;
        if (ks > 1 && bps < 2 * q) break;
        const long units = G * k, rounds = (units + slots - 1) / slots;
        const double eff = (double)units / (double)(rounds * slots);
        if (eff > best + 0.02) {   // a clearly better spread; otherwise fewer slices
            best = eff;
            best_ks = k;
            best_bps = bps;
        }
    }
    *ks_out = best_ks;
    *bps_out = best_bps;
}

int vxc_skinny_ok(const vxc_qmat *w, int M) {
    return w && (w->type == 2 || w->type == 8) && M >= 1 && M <= VXC_SKINNY_MAX_M;
}

int vxc_skinny_slices(const vxc_qmat *w) {
    int ks, bps;
    sk_split(w, &ks, &bps);
    return ks;
}

template <int QT, int MAXM>
static cudaError_t sk_launch(const vxc_qmat *w, const float *x, int ldx, int M, float *out, int ks, int bps,
                             cudaStream_t st) {
    using Sl = SkSlot<QT, MAXM>;
    // the shared-memory limit is a per-kernel, per-device attribute
    static std::atomic<uint64_t> attr_set{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t)1 << dev : 0;
    if (!bit || !(attr_set.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(k_qgemv_skinny<QT, MAXM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Sl::SMEM);
        if (e != cudaSuccess) return e;
        if (bit) attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    const long units = (long)((w->rows + SK_UROWS - 1) / SK_UROWS) * ks;
    const long slots = (long)sk_sms() * SkOcc<MAXM>::CTAS;
    const unsigned grid = (unsigned)(units < slots ? units : slots);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(SK_WARPS * 32);
    cfg.dynamicSmemBytes = Sl::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // may start while the producer of x drains
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k_qgemv_skinny<QT, MAXM>, w->qs, w->rows, w->nblk, w->wscale, x, ldx, M, out, bps,
                           ks);
    vxc_count_launches(1);
    return e;
}

// out = partials [ks][M][R] (the output itself when ks == 1); returns 0 or an
// error code with the message set.
int vxc_skinny_run(const vxc_qmat *w, const float *x, int ldx, int M, float *out, cudaStream_t st) {
    if (!vxc_skinny_ok(w, M) || ((uintptr_t)x & 15) || (ldx & 3)) {
        vxc_set_error("vxc_skinny_run: unsupported arguments (type %d, M %d)", w ? w->type : -1, M);
        return -4;
    }
    int ks, bps;
    sk_split(w, &ks, &bps);
    cudaError_t e;
    if (w->type == 2)
        e = M == 1 ? sk_launch<2, 1>(w, x, ldx, M, out, ks, bps, st) : sk_launch<2, 2>(w, x, ldx, M, out, ks, bps, st);
    else
        e = M == 1 ? sk_launch<8, 1>(w, x, ldx, M, out, ks, bps, st) : sk_launch<8, 2>(w, x, ldx, M, out, ks, bps, st);
    if (e != cudaSuccess) {
        vxc_set_error("vxc_skinny_run: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}
