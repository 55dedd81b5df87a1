"""Pin the CPU oracle (oracle/, a C restatement) against the reference itself.

The reference's own sources are compiled by oracle/Makefile into
oracle/_ref/libvxref.so (scalar build, the out-of-place attn_o fix applied by
symbol interposition).  Every restated function must agree bit-for-bit with
the reference function it restates; the only exception is vx_gemv_q4_0, whose
summation order differs from the dequant+vx_gemv_f32 path that
vx_model_forward actually uses, so it is held to fp32 rounding.
"""
import ctypes

import numpy as np
import pytest

from _paths import oracle, ref, ref_available
from qgen import q4_0_blocks, q8_0_blocks

pytestmark = pytest.mark.skipif(not ref_available(), reason="reference build not available")

f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


@pytest.fixture(scope="module")
def O():
    return oracle()


@pytest.fixture(scope="module")
def R():
    return ref()


def test_fp16_decode_all_codes(O, R):
    codes = [c for c in range(65536) if not ((c >> 10) & 0x1F == 31 and c & 0x3FF)]  # skip NaN payloads
    a = np.array([O.vxo_fp16_to_fp32(c) for c in codes], dtype=np.float32)
    b = np.array([R.vx_fp16_to_fp32(c) for c in codes], dtype=np.float32)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # and it is the exact IEEE decode
    assert np.array_equal(a.view(np.uint32), np.array(codes, dtype=np.uint16).view(np.float16).astype(np.float32).view(np.uint32))


def test_fp16_truncating_encode(O, R):
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-6, 1e-3, 1.0, 1e3, 1e5)])
    for x in xs[::7]:
        assert O.vxo_fp32_to_fp16_trunc(float(x)) == R.vx_fp32_to_fp16(float(x))


def test_quantize_q4_0(O, R):
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(32 * 512) * 0.02).astype(np.float32)
    a = np.zeros(512 * 18, np.uint8)
    b = np.zeros(512 * 18, np.uint8)
    O.vxo_quantize_row_q4_0(f32p(x), f32p(a), x.size)
    R.vx_quantize_row_q4_0(f32p(x), f32p(b), x.size)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("qt", [2, 8])
def test_dequant(O, R, qt):
    rng = np.random.default_rng(3)
    blk = (q4_0_blocks if qt == 2 else q8_0_blocks)(64, 256, rng)
    n = 64 * 256
    a = np.zeros(n, np.float32)
    b = np.zeros(n, np.float32)
    (O.vxo_dequant_q4_0 if qt == 2 else O.vxo_dequant_q8_0)(f32p(blk), f32p(a), n)
    (R.vx_dequantize_row_q4_0 if qt == 2 else R.vx_dequantize_row_q8_0)(f32p(blk), f32p(b), n)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("qt", [2, 8])
def test_gemv_matches_reference_path(O, R, qt):
    """Oracle GEMV == reference dequantise + vx_gemv_f32 (src/model.c:216-219,
    :235-241), bit for bit."""
    rng = np.random.default_rng(4)
    rows, cols = 96, 512
    blk = (q4_0_blocks if qt == 2 else q8_0_blocks)(rows, cols, rng)
    x = rng.standard_normal(cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    O.vxo_qgemv(qt, f32p(blk), f32p(x), f32p(y), 1, rows, cols)
    A = np.zeros(rows * cols, np.float32)
    (R.vx_dequantize_row_q4_0 if qt == 2 else R.vx_dequantize_row_q8_0)(f32p(blk), f32p(A), rows * cols)
    yr = np.zeros(rows, np.float32)
    R.vx_gemv_f32(f32p(yr), f32p(A), f32p(x), rows, cols)
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
    if qt == 2:   # the fused scalar kernel: same math, different order
        yq = np.zeros(rows, np.float32)
        R.vx_gemv_q4_0(f32p(blk), f32p(x), f32p(yq), rows, cols)
        assert np.max(np.abs(yq - y)) <= 1e-5 * np.max(np.abs(y))


def test_rms_norm_softmax_silu(O, R):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    a = np.zeros_like(x); b = np.zeros_like(x)
    O.vxo_rms_norm(f32p(a), f32p(x), f32p(w), x.size)
    R.vx_rms_norm(f32p(b), f32p(x), f32p(w), x.size)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    a = x.copy(); b = x.copy()
    O.vxo_softmax(f32p(a), a.size); R.vx_softmax(f32p(b), b.size)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    a = x.copy(); b = x.copy()
    O.vxo_silu(f32p(a), a.size); R.vx_silu(f32p(b), b.size)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("heads,kv,hd,theta,pos", [(8, 8, 32, 1e4, 0), (8, 8, 32, 1e4, 37), (32, 4, 64, 1e4, 511),
                                                    (64, 8, 128, 5e5, 4095)])
def test_rope(O, R, heads, kv, hd, theta, pos):
    rng = np.random.default_rng(6)
    q = rng.standard_normal(heads * hd).astype(np.float32)
    k = rng.standard_normal(kv * hd).astype(np.float32)
    qa, ka, qb, kb = q.copy(), k.copy(), q.copy(), k.copy()
    O.vxo_rope(f32p(qa), f32p(ka), pos, heads, kv, hd, theta)
    R.vx_rope(f32p(qb), f32p(kb), pos, heads, kv, hd, 0, theta)
    assert np.array_equal(qa.view(np.uint32), qb.view(np.uint32))
    assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32))
