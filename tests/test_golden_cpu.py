"""The oracle reproduces the committed golden vectors of the reference
(tests/golden/make_golden.py) bit for bit: logits and the greedy stream."""
import ctypes
import os

import numpy as np
import pytest

from _paths import oracle
import fixtures

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


@pytest.mark.parametrize("name", ["tiny_target", "tiny_draft"])
def test_oracle_matches_reference_goldens(name):
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    O = oracle()
    m = O.vxo_model_load(fixtures.path(name).encode(), 0)
    V = 4096
    prompt = g["prompt"].astype(np.int32)
    n = g["logits"].shape[0]
    out = np.zeros((n, V), np.float32)
    assert O.vxo_forward_all(m, f32p(prompt), n, f32p(out)) == 0
    assert np.array_equal(out.view(np.uint32), g["logits"].view(np.uint32))
    gen = np.zeros(len(g["greedy"]), np.int32)
    O.vxo_greedy_generate(m, f32p(prompt), len(prompt), f32p(gen), len(gen))
    assert np.array_equal(gen, g["greedy"])
    O.vxo_model_free(m)
