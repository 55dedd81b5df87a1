"""Generate tests/golden/*.npz from the REFERENCE implementation itself.

Runs the reference's own vx_model_forward (sources compiled in place by
oracle/Makefile into oracle/_ref/libvxref.so: scalar build, out-of-place
attn_o) on the tiny configuration-1 checkpoints that the library's
deterministic GGUF writer produces, and stores:
  - logits of every position of a 24-token prompt (fp32),
  - the target-only greedy continuation of a 32-token prompt (128 tokens, the
    configuration-1 workload) and
    the top-2 logit margin at each step.
Run from the repository root:  python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from _paths import ref  # noqa: E402
import fixtures  # noqa: E402

f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)


def ref_run(name, prompt, n_new):
    R = ref()
    h = ctypes.c_void_p()
    assert R.vx_model_create(fixtures.path(name).encode(), ctypes.byref(h)) == 0
    cfg = (ctypes.c_int * 8)()
    R.vxref_config(h, cfg)
    V = cfg[6]
    logits = np.zeros((len(prompt), V), np.float32)
    for i, t in enumerate(prompt):
        one = np.array([t], np.int32)
        assert R.vx_model_forward(h, f32p(one), 1, f32p(logits[i])) == 0
    gen, margins = [], []
    lg = logits[-1].copy()
    for _ in range(n_new):
        top = np.argsort(-lg, kind="stable")[:2]
        best = int(np.argmax(lg))        # first max, as src/speculative.c:93-98
        gen.append(best)
        margins.append(float(lg[top[0]] - lg[top[1]]))
        one = np.array([best], np.int32)
        assert R.vx_model_forward(h, f32p(one), 1, f32p(lg)) == 0
    R.vx_model_destroy(h)
    return logits, np.array(gen, np.int32), np.array(margins, np.float32)


def main():
    rng = np.random.default_rng(12345)
    prompt = rng.integers(0, 4096, 32).astype(np.int32)
    for name in ("tiny_target", "tiny_draft"):
        logits, gen, marg = ref_run(name, prompt, 128)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), prompt=prompt, logits=logits[:8], greedy=gen,
                            margins=marg)
        print(name, "greedy head", gen[:8], "min margin", marg.min())


if __name__ == "__main__":
    main()
