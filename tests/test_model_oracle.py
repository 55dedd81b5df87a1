"""The oracle's forward pass against the reference's own vx_model_forward
(oracle/_ref, scalar build with the out-of-place attn_o fix), bit for bit, on
the tiny configuration-1 checkpoints written by the library's GGUF writer."""
import ctypes
import hashlib

import numpy as np
import pytest

from _paths import oracle, ref, ref_available
import fixtures

f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


def test_writer_is_deterministic(tmp_path):
    import vxb200
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    for p in (a, b):
        vxb200.write_synth(str(p), 128, 2, 4, 4, 384, 4096, 8, 2)
    assert hashlib.sha256(a.read_bytes()).hexdigest() == hashlib.sha256(b.read_bytes()).hexdigest()


def oracle_logits(name, tokens, all_rows=True):
    O = oracle()
    m = O.vxo_model_load(fixtures.path(name).encode(), 0)
    assert m
    cfg = (ctypes.c_int * 8)()
    O.vxo_model_config(m, cfg)
    V = cfg[6]
    toks = np.asarray(tokens, dtype=np.int32)
    out = np.zeros((len(toks), V), np.float32)
    assert O.vxo_forward_all(m, f32p(toks), len(toks), f32p(out)) == 0
    O.vxo_model_free(m)
    return out


@pytest.mark.skipif(not ref_available(), reason="reference build not available")
@pytest.mark.parametrize("name", ["tiny_target", "tiny_draft"])
def test_forward_bit_exact_vs_reference(name):
    R = ref()
    h = ctypes.c_void_p()
    assert R.vx_model_create(fixtures.path(name).encode(), ctypes.byref(h)) == 0
    cfg = (ctypes.c_int * 8)()
    R.vxref_config(h, cfg)
    assert list(cfg)[:7] == [fixtures.CONFIGS[name][1], fixtures.CONFIGS[name][2], fixtures.CONFIGS[name][3],
                             fixtures.CONFIGS[name][0], fixtures.CONFIGS[name][0] // fixtures.CONFIGS[name][2],
                             fixtures.CONFIGS[name][4], fixtures.CONFIGS[name][5]]
    V = cfg[6]
    rng = np.random.default_rng(12345)
    toks = rng.integers(0, V, 24).astype(np.int32)
    ref_out = np.zeros((len(toks), V), np.float32)
    for i, t in enumerate(toks):
        one = np.array([t], np.int32)
        assert R.vx_model_forward(h, f32p(one), 1, f32p(ref_out[i])) == 0
    assert R.vxref_cache_len(h) == len(toks)
    R.vx_model_destroy(h)
    ora = oracle_logits(name, toks)
    assert np.array_equal(ora.view(np.uint32), ref_out.view(np.uint32))


@pytest.mark.skipif(not ref_available(), reason="reference build not available")
@pytest.mark.parametrize("name,n", [("l7b_2layer", 6), ("d11b_2layer", 12), ("l70b_2layer", 3)])
def test_forward_bit_exact_vs_reference_at_benchmark_widths(name, n):
    """The same pin at the widths the GPU tests compare against the oracle:
    7B width (32 heads of 128), the 1.1B draft shape (GQA 32/4, heads of 64)
    and the 70B width (GQA 64/8, theta 5e5, vocabulary 128256), 2 layers each
    (reference src/model.c:391-628, GQA map :303)."""
    R = ref()
    h = ctypes.c_void_p()
    assert R.vx_model_create(fixtures.path(name).encode(), ctypes.byref(h)) == 0
    cfg = (ctypes.c_int * 8)()
    R.vxref_config(h, cfg)
    e, L, H, KH, F, V = fixtures.CONFIGS[name][:6]
    assert list(cfg)[:7] == [L, H, KH, e, e // H, F, V]
    toks = np.random.default_rng(12345).integers(0, V, n).astype(np.int32)
    ref_out = np.zeros((n, V), np.float32)
    for i, t in enumerate(toks):
        assert R.vx_model_forward(h, f32p(np.array([t], np.int32)), 1, f32p(ref_out[i])) == 0
    R.vx_model_destroy(h)
    ora = oracle_logits(name, toks)
    assert np.array_equal(ora.view(np.uint32), ref_out.view(np.uint32))
