"""Device forward of K-quant models (vx_model_create on the tiny_q*k and
tiny_kqmix fixtures) against the oracle within 2e-3 x max|logit|, over a
prompt of two chunks, then two decode steps.

Covers the K-quant forward path: K-quant embedding rows, k_gemv_kq_img on
the forward's activation image, and row-stacked matrices of mixed K-quant
types (reference dispatch src/model.c:222-233).
"""
import ctypes
import numpy as np
import pytest
from _paths import oracle
import fixtures

pytestmark = pytest.mark.gpu
f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


@pytest.mark.parametrize("name", ["tiny_q2k", "tiny_q3k", "tiny_q4k", "tiny_q5k", "tiny_q6k", "tiny_q8k", "tiny_kqmix"])
def test_kquant_model_vs_oracle(cuda, name):
    import vxb200
    O = oracle()
    p = fixtures.path(name)
    om = O.vxo_model_load(p.encode(), 0)
    m = vxb200.Model(p)
    toks = np.random.default_rng(3).integers(0, 4096, 70).astype(np.int32)
    for chunk in (toks[:67], toks[67:68], toks[68:]):
        want = np.zeros(4096, np.float32)
        assert O.vxo_forward(om, f32p(chunk), len(chunk), f32p(want)) == 0
        got = m.forward(chunk)
        assert np.max(np.abs(got - want)) <= 2e-3 * np.max(np.abs(want)), name
    m.close()
    O.vxo_model_free(om)
