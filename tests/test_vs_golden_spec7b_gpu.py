"""Parity at the full benchmarked model: the spec7b target of bench.py
(Llama-2-7B shape, 32 layers, Q4_0, writer seed 11) on bench.py's sequence-0
prompt (512 ids), against a CPU golden computed by the oracle's scalar forward
(tests/golden/spec7b_seq0.npz, made by tests/golden/make_spec7b_golden.py;
the oracle is pinned bit for bit to the reference's own sources by
test_oracle_pin.py).

- The logits of the last prompt position are within 2e-3 x max|logit| of the
  golden (reference src/model.c:391-628 over 32 layers, prompt pass on the
  tensor-core GEMM).
- The device greedy loop emits the golden's greedy stream up to the first
  step whose CPU top-2 margin is at most 1e-3 (the benchmark definition); at
  temperature 0 this is also the stream speculative decoding emits.
"""
import os

import numpy as np
import pytest

import fixtures

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "spec7b_seq0.npz")
LOGIT_TOL = 2e-3


def test_full_7b_target_vs_cpu_golden(cuda):
    import vxb200
    g = np.load(GOLD)
    prompt, want, margins = g["prompt"], g["greedy"], g["margins"]
    assert np.array_equal(prompt, np.random.default_rng(1000).integers(0, 32000, 512, dtype=np.int32))
    m = vxb200.Model(fixtures.path("llama7b_q4"))
    lg = m.forward(prompt)
    ref = g["last_prompt_logits"]
    assert float(np.max(np.abs(lg - ref))) <= LOGIT_TOL * float(np.max(np.abs(ref)))
    m.cache_len = 0
    got = m.generate_greedy(prompt, len(want))
    assert len(got) == len(want)
    for i in range(len(want)):
        if int(got[i]) != int(want[i]):
            assert margins[i] <= 1e-3, (i, int(got[i]), int(want[i]), float(margins[i]))
            break
    m.close()
