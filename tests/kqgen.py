"""Random K-quant super-blocks for the tests (test infrastructure only)."""
import numpy as np

TYPES = {10: ("q2_K", 84), 11: ("q3_K", 110), 12: ("q4_K", 144), 13: ("q5_K", 176), 14: ("q6_K", 210),
         15: ("q8_K", 292)}


def fp16_bits(v):
    return np.asarray(v, np.float16).view(np.uint16)


def random_blocks(t, nblocks, rng):
    """Random bytes with finite, moderate scale fields."""
    bb = TYPES[t][1]
    b = rng.integers(0, 256, (nblocks, bb), dtype=np.uint8)
    d = fp16_bits(np.abs(rng.standard_normal(nblocks)) * 0.01 + 1e-3)
    dm = fp16_bits(np.abs(rng.standard_normal(nblocks)) * 0.01)
    put16 = lambda off, v: b.__setitem__((slice(None), slice(off, off + 2)), v.view(np.uint8).reshape(-1, 2))
    if t == 10:
        put16(80, d)
        put16(82, dm)
    elif t == 11:
        put16(108, d)
    elif t in (12, 13):
        put16(0, d)
        put16(2, dm)
    elif t == 14:
        put16(208, d)
    else:
        f = (np.abs(rng.standard_normal(nblocks)) * 0.01 + 1e-3).astype(np.float32)
        b[:, 0:4] = f.view(np.uint8).reshape(-1, 4)
    return np.ascontiguousarray(b)
