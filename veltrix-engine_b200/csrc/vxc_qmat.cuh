// vxc_qmat.cuh — device layout of a GGUF Q4_0 / Q8_0 weight matrix.
//
// The GGUF bytes stay the interface (18-byte Q4_0 and 34-byte Q8_0 blocks,
// reference include/quantize.h:5-10 and :34-38); on upload they are split
// into a quant plane and a scale plane, tiled by 128 rows so that every
// 16-byte chunk a kernel loads is aligned and a tile's K-range is one
// contiguous byte span (one bulk copy):
//
//   qs: [tile][block][128 rows][QB bytes]   QB = 16 (Q4_0) or 32 (Q8_0)
//   sc: [tile][block][128 rows] fp16        the block scale d
//
// Rows past R in the last tile are zero.  Within a Q4_0 row-block the 32
// nibbles are permuted so that 32-bit word j (bytes 4j..4j+3) holds elements
// 8j..8j+7 as: element 8j+2i in bits [4i, 4i+4) and element 8j+2i+1 in bits
// [16+4i, 20+4i), i = 0..3.  (w >> 4i) & 0x000F000F then yields the pair
// (8j+2i, 8j+2i+1) in the two 16-bit halves, which is what the fp16
// dequantiser consumes.  GGUF order is the reference's interleaved one:
// element 2b is the low nibble of byte b, 2b+1 the high nibble
// (src/quantize.c:584-588).
#pragma once
#include <stdint.h>

#define VXC_TILE_ROWS 128

struct vxc_qmat {
    int type;           // 2 = Q4_0, 8 = Q8_0
    int rows, cols;     // R, K (K % 32 == 0)
    int nblk;           // K / 32
    int ntile;          // ceil(R / 128)
    int qb;             // bytes per row-block in qs (16 or 32)
    uint8_t *qs;        // device
    uint16_t *sc;       // device
    size_t qs_bytes, sc_bytes;
};
