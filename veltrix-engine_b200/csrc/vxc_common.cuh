// vxc_common.cuh — shared device helpers for the Veltrix B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define VXC_CUDA_OK(expr)                                                       \
    do {                                                                        \
        cudaError_t _e = (expr);                                                \
        if (_e != cudaSuccess) {                                                \
            vxc_set_error("%s:%d %s: %s", __FILE__, __LINE__, #expr,            \
                          cudaGetErrorString(_e));                              \
            return -3;                                                          \
        }                                                                       \
    } while (0)

// Error text of the last failing vxc_* call on this host thread.
void vxc_set_error(const char *fmt, ...);

// Device-side error word (one per device, allocated at vxc_device_init and
// passed to kernels).  Kernels never trap: a wait that runs out of time, or an
// input outside the kernel's contract, records a code there and the kernel
// returns.  The host reads it after synchronising (vxc_check_device_error).
#define VXC_DERR_TIMEOUT_TMA 1u
#define VXC_DERR_TIMEOUT_MMA 2u
#define VXC_DERR_BAD_TOKEN 4u
#define VXC_DERR_BAD_SHAPE 8u
#define VXC_DERR_CTX_FULL 16u
#define VXC_DERR_TIMEOUT_EPI 32u

__device__ __forceinline__ void vxc_flag_error(unsigned int *err, unsigned int code) {
    if (err) atomicOr(err, code);
}

// Wall-clock budget for any spin-wait inside a kernel.
#define VXC_WAIT_NS 2000000000ull

__device__ __forceinline__ uint64_t vxc_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11) keyed by (seed, position, sequence,
// purpose); must agree with the CPU oracle bit-for-bit.
// ---------------------------------------------------------------------------
#define VXC_PURPOSE_DRAFT 1u
#define VXC_PURPOSE_ACCEPT 2u
#define VXC_PURPOSE_RESAMPLE 3u

__host__ __device__ __forceinline__ uint32_t vxc_philox_u32(uint64_t seed, uint32_t pos, uint32_t seq,
                                                            uint32_t purpose) {
    uint32_t c0 = pos, c1 = seq, c2 = purpose, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

// exp for the sampler: Cody-Waite reduction with a two-part ln 2 (Cody &
// Waite 1980) and the degree-7 Taylor polynomial of e^r by Horner with FMA,
// scaled by 2^k through the exponent field.  Written with explicitly rounded
// operations so no contraction changes it; bit-identical to the CPU oracle.
// Branch-free: arguments at or below -80 (and NaN) are clamped, evaluated and
// then replaced by 0; positive arguments are clamped to 0.
__device__ __forceinline__ float vxc_expf_canon(float x) {
    const bool zero = !(x > -80.0f);
    x = fminf(fmaxf(x, -80.0f), 0.0f);
    // k = nearest integer (ties to even) to x log2(e), |x log2(e)| < 116:
    // adding 1.5 * 2^23 leaves k in the low significand bits, and removing it
    // again gives k as a float (the classic round-by-magic-constant method).
    const float big = __fadd_rn(__fmul_rn(x, 1.44269504088896341f), 12582912.0f);
    const float kf = __fsub_rn(big, 12582912.0f);
    float r = __fmaf_rn(kf, -0.693145751953125f, x);
    r = __fmaf_rn(kf, -1.42860682030941723212e-6f, r);
    float p = 1.98412698412698413e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    // 2^k: the bits of big are those of 1.5 * 2^23 + k
    const uint32_t k127 = __float_as_uint(big) - 0x4B400000u + 127u;
    const float e = __fmul_rn(p, __uint_as_float(k127 << 23));
    return zero ? 0.0f : e;
}

// Integer sampling weight of one logit: trunc(exp((l - max) / T) * 2^32).
// The scaling by 2^32 is exact; the conversion truncates.
__device__ __forceinline__ uint64_t vxc_weight(float l, float mx, float invT) {
    const float z = __fmul_rn(__fsub_rn(l, mx), invT);
    return (uint64_t)__fmul_rn(vxc_expf_canon(z), 4294967296.0f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// fp16 bit pattern -> fp32 (exact for every non-NaN code, as the reference's
// vx_fp16_to_fp32, src/quantize.c:37-57).
__device__ __forceinline__ float vxc_h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
