"""K-quant oracle (oracle/vxo_kquant.c) pinned bit for bit to the
reference's own K-quant code (src/quantize.c, compiled by oracle/Makefile),
on random super-blocks of every type the reference's GEMV dispatches
(src/model.c:222-233): Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K.

- vxo_dequant_kquant == vx_dequantize_row_<type>
- vxo_gemv_kquant_shipped == vx_gemv_<type> (Q8_K-quantised activations and
  integer dots for Q2_K/Q3_K/Q4_K, blockwise dequant for the rest)
- vxo_gemv_kquant == the reference's blockwise GEMV, i.e. vx_gemv_<type> for
  Q5_K/Q6_K/Q8_K; for Q4_K the shipped dot leaves out half of every
  super-block, which the last test records.
"""
import ctypes

import numpy as np
import pytest

from _paths import oracle, ref, ref_available
from kqgen import TYPES, random_blocks

pytestmark = pytest.mark.skipif(not ref_available(), reason="reference build unavailable")
vp = lambda a: a.ctypes.data_as(ctypes.c_void_p)


def libs():
    O, R = oracle(), ref()
    O.vxo_dequant_kquant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    for f in (O.vxo_gemv_kquant, O.vxo_gemv_kquant_shipped):
        f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    for t, (nm, _) in TYPES.items():
        getattr(R, f"vx_dequantize_row_{nm}").argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        getattr(R, f"vx_gemv_{nm}").argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                               ctypes.c_int]
    return O, R


@pytest.mark.parametrize("t", sorted(TYPES))
def test_dequant_bit_exact(t):
    O, R = libs()
    rng = np.random.default_rng(t)
    nb = 64
    blk = random_blocks(t, nb, rng)
    a = np.zeros(nb * 256, np.float32)
    b = np.full(nb * 256, np.nan, np.float32)
    getattr(R, f"vx_dequantize_row_{TYPES[t][0]}")(vp(blk), vp(a), nb * 256)
    assert O.vxo_dequant_kquant(t, vp(blk), vp(b), nb * 256) == 0
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("t", sorted(TYPES))
def test_gemv_bit_exact_with_shipped(t):
    O, R = libs()
    rng = np.random.default_rng(100 + t)
    rows, cols = 37, 1024
    w = random_blocks(t, rows * cols // 256, rng)
    x = rng.standard_normal(cols).astype(np.float32)
    x[5:300] *= 0                       # an all-zero Q8_K block and ragged values
    ya = np.zeros(rows, np.float32)
    yb = np.full(rows, np.nan, np.float32)
    getattr(R, f"vx_gemv_{TYPES[t][0]}")(vp(w), vp(x), vp(ya), rows, cols)
    assert O.vxo_gemv_kquant_shipped(t, vp(w), vp(x), vp(yb), rows, cols) == 0
    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
    # the dequant GEMV is the reference's own for the blockwise types
    if t in (13, 14, 15):
        yc = np.full(rows, np.nan, np.float32)
        assert O.vxo_gemv_kquant(t, vp(w), vp(x), vp(yc), rows, cols) == 0
        assert np.array_equal(ya.view(np.uint32), yc.view(np.uint32))


def test_dequant_gemv_is_dequant_dot():
    """vxo_gemv_kquant = dequantised weights . x (float64 check, all types)."""
    O, _ = libs()
    rng = np.random.default_rng(7)
    rows, cols = 9, 512
    for t in TYPES:
        w = random_blocks(t, rows * cols // 256, rng)
        x = rng.standard_normal(cols).astype(np.float32)
        W = np.zeros(rows * cols, np.float32)
        assert O.vxo_dequant_kquant(t, vp(w), vp(W), rows * cols) == 0
        y = np.zeros(rows, np.float32)
        assert O.vxo_gemv_kquant(t, vp(w), vp(x), vp(y), rows, cols) == 0
        want = W.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
        assert np.max(np.abs(y - want)) <= 1e-5 * max(1.0, np.max(np.abs(want))), t


def test_shipped_q4k_dot_leaves_out_half_of_each_superblock():
    """As shipped, the Q4_K GEMV ignores elements 128..255 of each super-block:
    changing only those weights leaves its output unchanged."""
    O, R = libs()
    rng = np.random.default_rng(11)
    rows, cols = 4, 512
    w = random_blocks(12, rows * cols // 256, rng)
    x = rng.standard_normal(cols).astype(np.float32)
    y1, y2 = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
    R.vx_gemv_q4_K(vp(w), vp(x), vp(y1), rows, cols)
    w2 = w.copy()
    w2[:, 16 + 64:16 + 128] ^= 0x55         # nibbles of elements 128..255 (qs bytes 64..127)
    R.vx_gemv_q4_K(vp(w2), vp(x), vp(y2), rows, cols)
    assert np.array_equal(y1, y2)
    d1, d2 = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
    O.vxo_gemv_kquant(12, vp(w), vp(x), vp(d1), rows, cols)
    O.vxo_gemv_kquant(12, vp(w2), vp(x), vp(d2), rows, cols)
    assert not np.array_equal(d1, d2)
