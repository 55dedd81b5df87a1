"""Whole-model forwards with K-quant weights: the oracle (oracle/vxo_fwd.c,
K-quant rows decoded as the reference decodes them) against the reference
build (oracle/_ref/libvxref.so, with the out-of-place fix P1 extended to the
blockwise K-quant GEMVs) on the tiny target's shape, every 2-D tensor of one
K-quant type.

- Q5_K, Q6_K, Q8_K: the reference's own GEMV is dequant-then-dot, so the
  logits agree to 1e-5 x max|logit| (summation order only).
- Q3_K: the reference rounds the activations to int8 first (finding KQ1):
  a difference of about 1e-2, recorded between 1e-4 and 0.1.
- Q2_K and Q4_K: the reference's GEMV decodes other weights than its own
  dequantiser (KQ3) or drops half of every super-block (KQ2): the logits
  are unrelated (relative difference above 0.5).
The device path follows the oracle (tests/test_kquant_gpu.py).
"""
import ctypes

import numpy as np
import pytest

from _paths import oracle, ref, ref_available
import fixtures

pytestmark = pytest.mark.skipif(not ref_available(), reason="reference build unavailable")
f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
TOKS = np.array([1, 5, 900, 77, 4095], np.int32)


def both(name):
    O, R = oracle(), ref()
    p = fixtures.path(name).encode()
    om = O.vxo_model_load(p, 0)
    h = ctypes.c_void_p()
    assert R.vx_model_create(p, ctypes.byref(h)) == 0
    a, b = np.zeros(4096, np.float32), np.zeros(4096, np.float32)
    assert O.vxo_forward(om, f32p(TOKS), len(TOKS), f32p(a)) == 0
    assert R.vx_model_forward(h, f32p(TOKS), len(TOKS), f32p(b)) == 0
    O.vxo_model_free(om)
    R.vx_model_destroy(h)
    assert np.isfinite(a).all() and np.max(np.abs(a)) > 0.1
    return float(np.max(np.abs(a - b)) / np.max(np.abs(a)))


@pytest.mark.parametrize("name", ["tiny_q5k", "tiny_q6k", "tiny_q8k"])
def test_blockwise_types_match_reference(name):
    assert both(name) <= 1e-5


def test_q3k_reference_rounds_activations():
    assert 1e-4 < both("tiny_q3k") < 0.1


@pytest.mark.parametrize("name", ["tiny_q2k", "tiny_q4k"])
def test_q2k_q4k_reference_gemv_disagrees_with_its_dequant(name):
    assert both(name) > 0.5


def test_mixed_q4k_q6k_model_loads_in_the_oracle():
    """The Q4_K/Q6_K mix (value, down and LM head in Q6_K) decodes to finite
    logits; the reference's Q4_K GEMV (KQ2) makes its own differ."""
    assert both("tiny_kqmix") > 0.1
