"""GPU parity of the device forward pass through the public C API
(vx_model_create / vx_model_forward) against the reference goldens and the
CPU oracle.

Tolerance (the benchmark definition): logits within 2e-3 * max|logit|; greedy
tokens identical wherever the reference's top-2 margin exceeds 1e-3.
"""
import ctypes
import os

import numpy as np
import pytest

from _paths import oracle
import fixtures

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LOGIT_TOL = 2e-3
f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


@pytest.mark.parametrize("name", ["tiny_target", "tiny_draft"])
def test_logits_vs_reference_goldens(cuda, name):
    import vxb200
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    m = vxb200.Model(fixtures.path(name))
    prompt = g["prompt"]
    for i in range(g["logits"].shape[0]):
        lg = m.forward(prompt[i:i + 1])
        assert m.cache_len == i + 1
        assert rel_err(lg, g["logits"][i]) <= LOGIT_TOL
    m.close()


@pytest.mark.parametrize("name", ["tiny_target", "tiny_draft"])
def test_greedy_stream_vs_reference(cuda, name):
    import vxb200
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    m = vxb200.Model(fixtures.path(name))
    lg = m.forward(g["prompt"])           # batched prefill of the whole prompt
    out = []
    for i in range(len(g["greedy"])):
        t = int(np.argmax(lg))
        out.append(t)
        if t != g["greedy"][i]:
            assert g["margins"][i] <= 1e-3, (i, t, g["greedy"][i], g["margins"][i])
            break
        lg = m.forward(np.array([t]))
    m.close()


def test_cache_len_is_authoritative(cuda):
    """Callers rewind cache_len directly (src/speculative.c:101, :153);
    re-running the same tokens must reproduce the logits."""
    import vxb200
    m = vxb200.Model(fixtures.path("tiny_target"))
    rng = np.random.default_rng(0)
    toks = rng.integers(0, 4096, 12)
    a = m.forward(toks)
    m.cache_len = 4
    b = m.forward(toks[4:])
    assert m.cache_len == 12
    assert np.array_equal(a, b)
    m.cache_len = 0
    c = m.forward(toks[:5])
    d_all = [m.forward(toks[i:i + 1]) for i in range(5, 12)]
    assert rel_err(d_all[-1], a) <= 1e-5
    m.close()


@pytest.mark.parametrize("name", ["l7b_2layer", "d11b_2layer"])
def test_wide_models_vs_oracle(cuda, name):
    """7B-width Q4_0 target layers and the 1.1B-shape GQA (32/4 heads, hd 64)
    Q8_0 draft, 2 layers each, vocab 32000."""
    import vxb200
    O = oracle()
    path = fixtures.path(name)
    om = O.vxo_model_load(path.encode(), 0)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, 32000, 6).astype(np.int32)
    ref = np.zeros((len(toks), 32000), np.float32)
    assert O.vxo_forward_all(om, f32p(toks), len(toks), f32p(ref)) == 0
    O.vxo_model_free(om)
    m = vxb200.Model(path)
    lg = m.forward(toks[:3])
    assert rel_err(lg, ref[2]) <= LOGIT_TOL
    for i in range(3, len(toks)):
        lg = m.forward(toks[i:i + 1])
        assert rel_err(lg, ref[i]) <= LOGIT_TOL
    m.close()


def test_bad_token_is_an_error(cuda):
    import vxb200
    m = vxb200.Model(fixtures.path("tiny_target"))
    with pytest.raises(vxb200.VxError):
        m.forward(np.array([5000]))
    m.close()
