"""Greedy decoding on the device (vx_model_generate_greedy, the loop of the
reference's CLI, src/main.c:283-324, one CUDA-graph replay per token).

- The tiny target's stream equals the reference build's greedy stream
  (tests/golden) wherever the reference's top-2 margin exceeds 1e-3, the
  same rule as test_model_gpu.py.
- At 7B width it emits exactly the tokens of a host loop over
  vx_model_forward with the reference's first-max argmax, and the tokens of
  the CPU oracle's greedy loop (oracle/vxo_fwd.c, the reference's scalar
  forward) wherever the oracle's top-2 margin exceeds 1e-3.
- eos_id stops the loop without emitting it; cache_len counts every
  forwarded token, so a forward of the last emitted token continues the
  stream.
"""
import ctypes
import os

import numpy as np
import pytest

from _paths import oracle
import fixtures

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def host_loop(m, prompt, n):
    """First-max argmax over vx_model_forward's logits (src/main.c:307-311)."""
    lg = m.forward(prompt)
    out = []
    for _ in range(n):
        t = int(np.argmax(lg))
        out.append(t)
        lg = m.forward(np.array([t], np.int32))
    return np.array(out, np.int32)


def oracle_greedy(path, prompt, n, V=32000):
    """The oracle's greedy stream (first-max argmax after every forward) and
    each step's top-2 logit margin."""
    O = oracle()
    f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    om = O.vxo_model_load(path.encode(), 0)
    ref = np.zeros(V, np.float32)
    assert O.vxo_forward(om, f32p(prompt), len(prompt), f32p(ref)) == 0
    toks, margins = [], []
    for _ in range(n):
        top2 = np.partition(ref, -2)[-2:]
        t = int(np.argmax(ref))
        toks.append(t)
        margins.append(float(top2[1] - top2[0]))
        one = np.array([t], np.int32)
        assert O.vxo_forward(om, f32p(one), 1, f32p(ref)) == 0
    O.vxo_model_free(om)
    return toks, margins


def test_greedy_matches_reference_golden(cuda):
    import vxb200
    g = np.load(os.path.join(GOLD, "tiny_target.npz"))
    m = vxb200.Model(fixtures.path("tiny_target"))
    out = m.generate_greedy(g["prompt"], len(g["greedy"]))
    assert len(out) == len(g["greedy"])
    assert m.cache_len == len(g["prompt"]) + len(out) - 1
    for i in range(len(out)):
        if out[i] != g["greedy"][i]:
            assert g["margins"][i] <= 1e-3, (i, out[i], g["greedy"][i], g["margins"][i])
            break
    m.close()


def test_greedy_equals_host_loop_7b_width(cuda):
    import vxb200
    prompt = np.random.default_rng(3).integers(0, 32000, 70).astype(np.int32)   # two prompt chunks
    m = vxb200.Model(fixtures.path("l7b_2layer"))
    want = host_loop(m, prompt, 20)
    m.cache_len = 0
    got = m.generate_greedy(prompt, 20)
    assert np.array_equal(got, want)
    m.close()
    # the reference's arithmetic: equal up to the first near-tie of the oracle's logits
    toks, margins = oracle_greedy(fixtures.path("l7b_2layer"), prompt, 20)
    for i in range(20):
        if int(got[i]) != toks[i]:
            assert margins[i] <= 1e-3, (i, int(got[i]), toks[i], margins[i])
            break


def test_eos_and_continuation(cuda):
    import vxb200
    m = vxb200.Model(fixtures.path("tiny_target"))
    prompt = np.random.default_rng(9).integers(0, 4096, 16).astype(np.int32)
    full = m.generate_greedy(prompt, 24)
    assert len(full) == 24
    # continuing from the cache: forwarding the last emitted token gives the next one
    nxt = int(np.argmax(m.forward(full[-1:])))
    m.cache_len = 0
    longer = m.generate_greedy(prompt, 25)
    assert np.array_equal(longer[:24], full) and longer[24] == nxt
    # eos: the first occurrence of some later token ends the stream before it
    k = 10
    eos = int(full[k])
    first = int(np.argmax(full == eos))
    m.cache_len = 0
    cut = m.generate_greedy(prompt, 24, eos_id=eos)
    assert np.array_equal(cut, full[:first])
    assert m.cache_len == len(prompt) + first
    m.close()
