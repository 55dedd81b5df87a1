// vxc_qmat.cuh — device layout of a GGUF Q4_0 / Q8_0 weight matrix, and of
// the activation image the tensor-core GEMV reads.
//
// Weights.  The GGUF bytes stay the interface (18-byte Q4_0 and 34-byte Q8_0
// blocks, reference include/quantize.h:5-10 and :34-38).  On upload the
// matrix is cut into 128-row tiles and stored as one record per
// (tile, 32-column block), records of a tile contiguous along K, so that any
// K-range of a tile is one contiguous span (one bulk copy):
//
//   record(t, b) at qs + (t * nblk + b) * REC
//     [128 rows][QB bytes]   quants of rows 128t..128t+127, QB = 16 or 32
//     [128 rows] fp16        the block scale d of each row, times 2^wshift
//   REC = 128 * QB + 256     (2304 bytes for Q4_0, 4352 for Q8_0)
//
// Rows past R in the last tile are zero.  The scales are stored multiplied
// by 2^wshift (exact: a power of two), chosen per matrix so that
// |d * q| * 2^wshift < 2^15 for every block; results are multiplied by
// wscale = 2^-wshift.  Within a Q4_0 row-block the 32 nibbles are permuted so
// that 32-bit word j (bytes 4j..4j+3) holds elements 8j..8j+7 as: element
// 8j+2i in bits [4i, 4i+4) and element 8j+2i+1 in bits [16+4i, 20+4i),
// i = 0..3; (w >> 4i) & 0x000F000F then yields the pair (8j+2i, 8j+2i+1) in
// the two 16-bit halves.  GGUF order is the reference's interleaved one:
// element 2b is the low nibble of byte b, 2b+1 the high nibble
// (src/quantize.c:584-588).
//
// Activation image (the MMA's B operand, built by the producer of the
// activations): N rows (N = 16 * ceil(M / 16)), each row m prescaled by
// xs[m] = 2^e (max|x[m]| * 2^e in [2^14, 2^15)) and split into fp16
// hi = RN(x * xs) and lo = RN(x * xs - hi).  Per 32-column block b the image
// holds 4 chunks c (elements 8c..8c+7) of 2N rows x 16 bytes: rows 0..N-1
// the hi parts, rows N..2N-1 the lo parts:
//   byte offset ((b * 4 + c) * 2N + n) * 16
// This is the K-major, no-swizzle canonical layout of tcgen05 (8-row core
// matrices, 16-byte rows) for a 2N-row B operand, so one MMA multiplies the
// weights by both parts, and a slice of blocks is one contiguous span.
#pragma once
#include <stddef.h>
#include <stdint.h>

#define VXC_TILE_ROWS 128

struct vxc_qmat {
    int type;           // 2 = Q4_0, 8 = Q8_0; 10..15 K-quant; VXC_QMAT_STACK: parts below
    int rows, cols;     // R, K (K % 32 == 0)
    int nblk;           // K / 32
    int ntile;          // ceil(R / 128)
    int qb;             // quant bytes per row-block (16 or 32)
    int rec;            // bytes per record
    int wshift;         // scales stored times 2^wshift
    float wscale;       // 2^-wshift
    uint8_t *qs;        // device records
    size_t qs_bytes;
    // VXC_QMAT_STACK: K-quant matrices of different types stacked by rows
    // (e.g. Q4_K query/key and Q6_K value rows); part i fills output rows
    // [part_row0[i], part_row0[i] + parts[i]->rows)
    int nparts;
    vxc_qmat *parts[3];
    int part_row0[3];
};
#define VXC_QMAT_STACK 100

// Image bytes of one 32-column block for N padded rows.
__host__ __device__ static inline size_t vxc_img_block_bytes(int N) { return (size_t)N * 128; }
__host__ __device__ static inline int vxc_img_rows(int M) { return 16 * ((M + 15) / 16); }
