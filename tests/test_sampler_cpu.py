"""CPU checks of the oracle's sampling pieces (O-spec).

- Philox4x32-10 against the known-answer vectors published with the
  generator (Salmon et al., SC'11; Random123 kat_vectors).
- The canonical exp against math.exp.
- vxo_sample draws follow softmax(l/T).
- O-spec at temperature 0 reproduces target-only greedy decoding exactly,
  and acceptance of identical distributions is certain.
"""
import ctypes
import math

import numpy as np
import pytest

from _paths import oracle
import fixtures

f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


@pytest.mark.parametrize("ctr,key,want", [
    ((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
    ((0xffffffff,) * 4, (0xffffffff,) * 2, (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
    ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
     (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1)),
])
def test_philox_known_answers(ctr, key, want):
    O = oracle()
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    O.vxo_philox4x32_10(c, k, o)
    assert tuple(o) == want
    if ctr[3] == 0:   # the sampler's keyed word is word 0 of the block with counter word 3 = 0
        assert O.vxo_philox_u32(key[0] | (key[1] << 32), ctr[0], ctr[1], ctr[2]) == want[0]


def test_expf_accuracy():
    O = oracle()
    xs = np.concatenate([-np.logspace(-8, math.log10(79.9), 4000), np.linspace(-30, 0, 4001)])
    worst = 0.0
    for x in xs.astype(np.float32):
        got = O.vxo_expf(float(x))
        want = math.exp(float(x))
        worst = max(worst, abs(got - want) / want)
    assert worst < 5e-7          # a few ulp of fp32
    assert O.vxo_expf(-81.0) == 0.0 and O.vxo_expf(0.0) == 1.0


def test_sample_follows_softmax():
    O = oracle()
    rng = np.random.default_rng(3)
    l = rng.standard_normal(8).astype(np.float32) * 2
    T = 0.8
    n = 40000
    counts = np.zeros(8)
    for i in range(n):
        counts[O.vxo_sample(f32p(l), 8, T, O.vxo_philox_u32(7, i, 0, 1))] += 1
    p = np.exp((l - l.max()) / T)
    p /= p.sum()
    assert np.max(np.abs(counts / n - p)) < 0.01
    assert O.vxo_sample(f32p(l), 8, 0.0, 123) == int(np.argmax(l))


def test_accept_identical_distributions_always_accepts():
    O = oracle()
    rng = np.random.default_rng(4)
    k, V = 5, 1000
    P = rng.standard_normal((k + 1, V)).astype(np.float32)
    Q = P[:k].copy()
    d = np.array([O.vxo_sample(f32p(Q[i]), V, 0.8, O.vxo_philox_u32(9, 100 + i, 3, 1)) for i in range(k)], np.int32)
    nxt = ctypes.c_int()
    a = O.vxo_accept(f32p(P), f32p(Q), f32p(d), k, V, 0.8, 9, 3, 100, ctypes.byref(nxt))
    assert a == k and 0 <= nxt.value < V


def test_greedy_spec_equals_greedy_target():
    O = oracle()
    t = O.vxo_model_load(fixtures.path("tiny_target").encode(), 0)
    d = O.vxo_model_load(fixtures.path("tiny_draft").encode(), 0)
    rng = np.random.default_rng(12345)
    prompt = rng.integers(0, 4096, 32).astype(np.int32)
    n = 48
    g = np.zeros(n, np.int32)
    O.vxo_greedy_generate(t, f32p(prompt), len(prompt), f32p(g), n)
    s = np.zeros(n, np.int32)
    rounds = ctypes.c_int()
    got = O.vxo_spec_generate(t, d, f32p(prompt), len(prompt), 4, 0.0, 1, 0, f32p(s), n, ctypes.byref(rounds))
    assert got == n
    assert np.array_equal(g, s)
    assert rounds.value <= n
    O.vxo_model_free(t)
    O.vxo_model_free(d)
