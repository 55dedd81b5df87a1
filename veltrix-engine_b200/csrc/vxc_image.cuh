// vxc_image.cuh — writers of the tensor-core GEMV's activation image (layout
// in vxc_qmat.cuh): per-row power-of-two prescale and the exact fp16 hi/lo
// split.  Used by the generic image kernel and by the fused producers of the
// forward pass (norm, SwiGLU, attention combine).
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

// 2^e with max|x| * 2^e in [2^14, 2^15) (1 for an all-zero row).
__device__ __forceinline__ float vxc_prescale(float mx) {
    if (!(mx > 0.0f) || !isfinite(mx)) return 1.0f;
    int e;
    frexpf(mx, &e);
    e = 15 - e;
    e = max(-120, min(120, e));
    return ldexpf(1.0f, e);
}

// 8 values -> fp16 hi = RN(v*s), lo = RN(v*s - hi), packed pairwise.
__device__ __forceinline__ void vxc_hilo8(const float *v, float s, uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float a0 = v[2 * k] * s, a1 = v[2 * k + 1] * s;
        const __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
        const __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
        h[k] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        l[k] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Row m of the image for a K-long row whose element k is val(k); called by
// every thread of the CTA (any block size).
template <class F>
__device__ __forceinline__ void vxc_image_row(uint8_t *__restrict__ img, int N, int m, int K, float s, F val) {
    for (int ch = threadIdx.x; ch < K / 8; ch += blockDim.x) {
        const int b = ch >> 2, c = ch & 3;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = val(8 * ch + i);
        uint4 hi, lo;
        vxc_hilo8(v, s, hi, lo);
        uint8_t *chunk = img + (size_t)(b * 4 + c) * 2 * N * 16;
        *reinterpret_cast<uint4 *>(chunk + (size_t)m * 16) = hi;
        *reinterpret_cast<uint4 *>(chunk + (size_t)(N + m) * 16) = lo;
    }
}
