// vxc_synth.cu — synthetic weights generated in device memory.
//
// The same numbers as the library's GGUF writer (host/vxh_synth.c): element
// e of tensor ti is the Box-Muller normal from Philox4x32-10 keyed by (seed,
// ti, e / 4), times 0.02, and every 32 elements are quantised with the
// reference's Q4_0 rule (src/quantize.c:88-114) or the GGML Q8_0 rule.  The
// integer and fp32 steps are the writer's; the double-precision log, sqrt,
// cos and sin are the device's, so an element can differ from the file by
// one rounding of a double, which only matters where the fp32 value or a
// quantisation step sits on a boundary.  A timing run of a 70B-shaped model
// then needs no 41 GB checkpoint on the host: each GPU writes just the rows
// and column blocks of its shard.
#include "vxc_common.cuh"
#include "vxc_internal.h"

namespace {

__device__ __forceinline__ void philox10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint64_t seed,
                                         uint32_t out[4]) {
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; r++) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c1 = lo1;
        c3 = lo0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

// Elements 4q..4q+3 of tensor ti (the writer's normals4).
__device__ __forceinline__ void normals4(uint64_t seed, uint32_t ti, uint64_t q, float *z) {
    uint32_t w[4];
    philox10((uint32_t)q, (uint32_t)(q >> 32), ti, 0x5EEDu, seed, w);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const double u1 = ((double)w[2 * h] + 0.5) * (1.0 / 4294967296.0);
        const double u2 = ((double)w[2 * h + 1] + 0.5) * (1.0 / 4294967296.0);
        const double r = sqrt(-2.0 * log(u1));
        z[2 * h] = (float)(r * cos(6.283185307179586 * u2) * 0.02f);
        z[2 * h + 1] = (float)(r * sin(6.283185307179586 * u2) * 0.02f);
    }
}

// Truncating fp32 -> fp16 (the reference's encoder, src/quantize.c:17-35).
__device__ __forceinline__ uint16_t f2h_trunc(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t s = (x >> 31) & 1u, e = (x >> 23) & 0xFFu, m = x & 0x7FFFFFu;
    if (e == 0) return (uint16_t)(s << 15);
    if (e == 0xFF) return (uint16_t)((s << 15) | (0x1Fu << 10) | (m >> 13));
    const int ne = (int)e - 127 + 15;
    if (ne <= 0) return (uint16_t)(s << 15);
    if (ne >= 31) return (uint16_t)((s << 15) | (0x1Fu << 10));
    return (uint16_t)((s << 15) | ((uint32_t)ne << 10) | (m >> 13));
}

// One GGUF block per thread: out[r][c] for rows row0.. and blocks blk0.. of a
// tensor whose rows hold nblk_full blocks.
template <int QT>
__global__ void k_synth_blocks(uint64_t seed, uint32_t ti, long long row0, int nrows, int nblk_full, int blk0,
                               int nblk, uint8_t *__restrict__ out) {
    constexpr int BB = QT == 2 ? 18 : 34;
    const long long total = (long long)nrows * nblk;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / nblk, c = i % nblk;
        const uint64_t b = (uint64_t)(row0 + r) * nblk_full + blk0 + c;
        float x[32];
#pragma unroll
        for (int q = 0; q < 8; q++) normals4(seed, ti, b * 8 + q, x + 4 * q);
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
        uint8_t *o = out + (size_t)i * BB;
        if (QT == 2) {
            float d = amax / 7.0f;
            if (d < 1e-10f) d = 1e-10f;
            const uint16_t h = f2h_trunc(d);
            o[0] = (uint8_t)h;
            o[1] = (uint8_t)(h >> 8);
            const float id = 1.0f / d;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                int a = (int)(x[j] * id), e = (int)(x[j + 1] * id);
                a = a < -8 ? -8 : a > 7 ? 7 : a;
                e = e < -8 ? -8 : e > 7 ? 7 : e;
                o[2 + j / 2] = (uint8_t)((uint8_t)(a + 8) | ((uint8_t)(e + 8) << 4));
            }
        } else {
            const float d = amax / 127.0f;
            const uint16_t h = f2h_trunc(d);
            o[0] = (uint8_t)h;
            o[1] = (uint8_t)(h >> 8);
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                float v = roundf(x[j] * id);
                v = v > 127.0f ? 127.0f : v < -127.0f ? -127.0f : v;
                o[2 + j] = (uint8_t)(int8_t)v;
            }
        }
    }
}

}  // namespace

int vxc_synth_blocks(int type, uint64_t seed, uint32_t ti, long long row0, int nrows, int nblk_full, int blk0,
                     int nblk, uint8_t *dev_out) {
    if ((type != 2 && type != 8) || nrows <= 0 || nblk <= 0 || blk0 < 0 || blk0 + nblk > nblk_full || !dev_out) {
        vxc_set_error("vxc_synth_blocks: bad arguments");
        return -4;
    }
    const long long total = (long long)nrows * nblk;
    const long long want = (total + 255) / 256;
    const unsigned grid = (unsigned)(want < 148 * 16 ? want : 148 * 16);
    if (type == 2) k_synth_blocks<2><<<grid, 256>>>(seed, ti, row0, nrows, nblk_full, blk0, nblk, dev_out);
    else k_synth_blocks<8><<<grid, 256>>>(seed, ti, row0, nrows, nblk_full, blk0, nblk, dev_out);
    vxc_count_launches(1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        vxc_set_error("vxc_synth_blocks: %s", cudaGetErrorString(e));
        return -3;
    }
    return 0;
}
