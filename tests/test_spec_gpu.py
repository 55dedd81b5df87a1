"""Configuration 1 end to end on the device: speculative decoding through the
public API (vx_speculative_*), tiny Q8_0 target and draft, 32-token prompt,
k = 4, 128 new tokens.

- Greedy: the output must equal the reference's target-only greedy stream
  (tests/golden, produced by the reference build) wherever the reference's
  top-2 margin exceeds 1e-3 (the benchmark definition).
- Sampled (T = 0.8): the oracle's O-spec run on the same checkpoints with the
  same seed; sampling is bit-exact given identical logits and the logits agree
  to ~1e-6, so the streams are expected to be identical.
- Batch: each sequence of a batch equals its single-sequence run.
"""
import ctypes
import os

import numpy as np
import pytest

from _paths import oracle
import fixtures

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


@pytest.fixture(scope="module")
def models(cuda):
    import vxb200
    t = vxb200.Model(fixtures.path("tiny_target"))
    d = vxb200.Model(fixtures.path("tiny_draft"))
    yield t, d
    t.close()
    d.close()


def test_greedy_equals_reference_greedy(models):
    import vxb200
    t, d = models
    g = np.load(os.path.join(GOLD, "tiny_target.npz"))
    n = len(g["greedy"])                  # the whole configuration-1 workload: 128 new tokens
    assert n == 128
    sp = vxb200.Speculative(d, t, 4, temp=0.0)
    out = sp.generate(g["prompt"], n)
    assert len(out) == n
    ref = g["greedy"]
    for i in range(n):
        if out[i] != ref[i]:
            assert g["margins"][i] <= 1e-3, (i, out[i], ref[i])
            break
    st = sp.stats()
    assert st.emitted == n and st.rounds >= 1 and st.accepted <= st.drafted
    sp.close()


def test_sampled_matches_oracle_spec(models):
    import vxb200
    t, d = models
    O = oracle()
    ot = O.vxo_model_load(fixtures.path("tiny_target").encode(), 0)
    od = O.vxo_model_load(fixtures.path("tiny_draft").encode(), 0)
    rng = np.random.default_rng(12345)
    prompt = rng.integers(0, 4096, 32).astype(np.int32)
    n = 128
    want = np.zeros(n, np.int32)
    rounds = ctypes.c_int()
    O.vxo_spec_generate(ot, od, f32p(prompt), len(prompt), 4, 0.8, 1234, 0, f32p(want), n, ctypes.byref(rounds))
    sp = vxb200.Speculative(d, t, 4, temp=0.8, seed=1234)
    got = sp.generate(prompt, n)
    assert len(got) == n
    agree = int(np.argmax(got != want)) if np.any(got != want) else n
    assert agree == n, f"streams diverge at token {agree}"
    O.vxo_model_free(ot)
    O.vxo_model_free(od)
    sp.close()


def test_batch_equals_single(models):
    import vxb200
    t, d = models
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 4096, n).astype(np.int32) for n in (32, 17, 2)]
    sp = vxb200.Speculative(d, t, 4, temp=0.8, seed=99)
    batch = sp.generate_batch(prompts, 40)
    for i, p in enumerate(prompts):
        single = vxb200.Speculative(d, t, 4, temp=0.8, seed=99, seq_id_base=i)
        one = single.generate(p, 40)
        assert np.array_equal(one, batch[i]), i
        single.close()
    sp.close()


def test_stream_single_token_prompt(models):
    """vx_speculative_generate_stream: a one-token prompt (src/speculative.c:296-300)."""
    import vxb200
    t, d = models
    sp = vxb200.Speculative(d, t, 3, temp=0.0)
    out = np.zeros(20, np.int32)
    n = vxb200.lib().vx_speculative_generate_stream(sp.h, 7, out.ctypes.data, 20)
    assert n == 20
    # greedy speculative == greedy target decoding from the same prompt
    t.cache_len = 0
    lg = t.forward(np.array([7]))
    for i in range(20):
        tok = int(np.argmax(lg))
        assert tok == out[i], i
        lg = t.forward(np.array([tok]))
    sp.close()


_EAGER_SCRIPT = r"""
import sys
sys.path[:0] = [{tests!r}, {pkg!r}]
import numpy as np, vxb200, fixtures
vxb200.check(vxb200.lib().vxc_device_init(0))
t = vxb200.Model(fixtures.path("tiny_target")); d = vxb200.Model(fixtures.path("tiny_draft"))
sp = vxb200.Speculative(d, t, 4, temp=0.8, seed=7)
p = np.random.default_rng(3).integers(0, 4096, 32, dtype=np.int32)
print(" ".join(str(int(x)) for x in sp.generate(p, 48)))
"""


def test_eager_rounds_equal_graph_rounds(models):
    """VX_SPEC_EAGER=1 (plain launches, for profilers) emits the same tokens as the graph loop."""
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    pkg = os.path.join(os.path.dirname(here), "veltrix-engine_b200")
    code = _EAGER_SCRIPT.format(tests=here, pkg=pkg)
    outs = []
    for eager in ("0", "1"):
        env = dict(os.environ, VX_SPEC_EAGER=eager)
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(r.stdout.strip().splitlines()[-1])
    assert outs[0] == outs[1] and len(outs[0].split()) == 48


def test_generation_stops_at_n_ctx(models):
    """The reference loop stops when prompt + generated tokens reach the
    target's n_ctx (src/speculative.c:254, :293): a sequence emits at most
    n_ctx - prompt_len tokens, the same ones an unbounded run starts with, and
    nothing when its prompt already fills the context."""
    import vxb200
    t, d = models
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, 4096, n).astype(np.int32) for n in (40, 20, 64)]
    sp = vxb200.Speculative(d, t, 4, temp=0.8, seed=5)
    free_run = sp.generate_batch(prompts, 30)
    assert [len(o) for o in free_run] == [30, 30, 30]
    saved = t.head.config.n_ctx
    try:
        t.head.config.n_ctx = 48
        capped = sp.generate_batch(prompts, 30)
        assert [len(o) for o in capped] == [8, 28, 0]
        for a, b in zip(capped, free_run):
            assert np.array_equal(a, b[:len(a)])
        one = vxb200.Speculative(d, t, 4, temp=0.8, seed=5, seq_id_base=1)
        one_out = one.generate(prompts[1], 100)
        assert len(one_out) == 28 and np.array_equal(one_out, free_run[1][:28])
        one.close()
    finally:
        t.head.config.n_ctx = saved
    sp.close()
