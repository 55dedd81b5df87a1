"""Synthetic quantised matrices of the microbenchmark configuration
(Q4_0: nibbles uniform 0..15, scale fp16(|N(0,1)|*0.02); Q8_0: int8 uniform
-127..127, scale fp16(|N(0,1)|*0.002)), as raw GGUF blocks."""
import numpy as np


def q4_0_blocks(rows, cols, rng):
    nb = cols // 32
    d = (np.abs(rng.standard_normal((rows, nb))) * 0.02).astype(np.float16)
    qs = rng.integers(0, 256, size=(rows, nb, 16), dtype=np.uint8)
    blk = np.empty((rows, nb, 18), dtype=np.uint8)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    blk[:, :, 2:] = qs
    return blk


def q8_0_blocks(rows, cols, rng):
    nb = cols // 32
    d = (np.abs(rng.standard_normal((rows, nb))) * 0.002).astype(np.float16)
    qs = rng.integers(-127, 128, size=(rows, nb, 32), dtype=np.int8)
    blk = np.empty((rows, nb, 34), dtype=np.uint8)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    blk[:, :, 2:] = qs.view(np.uint8)
    return blk


def dequant(qtype, blk):
    """Exact float64 dequantisation (reference src/quantize.c:578-591, :642-651)."""
    rows, nb, _ = blk.shape
    d = blk[:, :, 0:2].copy().view(np.float16).astype(np.float64)[:, :, 0]
    if qtype == 2:
        qs = blk[:, :, 2:]
        lo = (qs & 0x0F).astype(np.int64) - 8
        hi = (qs >> 4).astype(np.int64) - 8
        q = np.stack([lo, hi], axis=-1).reshape(rows, nb, 32)
    else:
        q = blk[:, :, 2:].view(np.int8).astype(np.int64)
    return (q * d[:, :, None]).reshape(rows, nb * 32)
