"""Generate tests/golden/spec7b_seq0.npz: the benchmarked configuration's
first sequence, computed on the CPU.

The model is the spec7b target of bench.py (Llama-2-7B shape, 32 layers,
Q4_0, writer seed 11, RoPE theta 1e4), written by the library's deterministic
GGUF writer; the prompt is bench.py's sequence 0 (512 ids from
numpy default_rng(1000)).  With temperature 0 speculative decoding emits the
target's greedy stream, so the golden is the target-only greedy continuation
(first maximum wins, src/speculative.c:93-98) after the 512-id prompt, with
the top-2 logit margin at each step, and the logits of the last prompt
position.

By default the oracle computes it (oracle/vxo_fwd.c, the reference's scalar
forward restated; tests/test_oracle_pin.py pins it bit for bit to the
reference's own sources): about 20 minutes on 8 host threads.  With
--reference the reference's own vx_model_forward (oracle/_ref/libvxref.so)
computes it instead, about five times slower.
Run from the repository root:  python tests/golden/make_spec7b_golden.py
"""
import argparse
import ctypes
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from _paths import oracle, ref  # noqa: E402

f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)

# bench.py SPEC_TARGET and spec_prompts(0, 1)
TARGET = dict(n_embd=4096, n_layers=32, n_heads=32, n_kv_heads=32, n_ff=11008, n_vocab=32000, wtype=2, seed=11,
              rope_theta=10000.0)
PROMPT_SEED, PROMPT_LEN, N_NEW = 1000, 512, 16


def prompt():
    return np.random.default_rng(PROMPT_SEED).integers(0, TARGET["n_vocab"], PROMPT_LEN, dtype=np.int32)


def model_path():
    """tests/fixtures.py "llama7b_q4": the writer's file for TARGET (bench.py SPEC_TARGET)."""
    import fixtures
    assert fixtures.CONFIGS["llama7b_q4"] == (TARGET["n_embd"], TARGET["n_layers"], TARGET["n_heads"],
                                              TARGET["n_kv_heads"], TARGET["n_ff"], TARGET["n_vocab"],
                                              TARGET["wtype"], TARGET["seed"], TARGET["rope_theta"])
    return fixtures.path("llama7b_q4")


def check_prefix(n):
    """The oracle against the reference's own forward on this model, bit for bit."""
    path = model_path().encode()
    V = TARGET["n_vocab"]
    R = ref()
    R.vx_set_n_threads(os.cpu_count() or 1)
    h = ctypes.c_void_p()
    assert R.vx_model_create(path, ctypes.byref(h)) == 0
    O = oracle()
    om = O.vxo_model_load(path, 1024)
    assert om
    a, b = np.zeros(V, np.float32), np.zeros(V, np.float32)
    for i, t in enumerate(prompt()[:n]):
        one = np.array([t], np.int32)
        assert R.vx_model_forward(h, f32p(one), 1, f32p(a)) == 0
        assert O.vxo_forward(om, f32p(one), 1, f32p(b)) == 0
        if not np.array_equal(a.view(np.uint32), b.view(np.uint32)):
            print(f"position {i}: logits differ, max |diff| {float(np.max(np.abs(a - b)))}")
            return 1
    R.vx_model_destroy(h)
    O.vxo_model_free(om)
    print(f"oracle == reference bit for bit over the first {n} prompt positions")
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", action="store_true")
    ap.add_argument("--out", default=os.path.join(HERE, "spec7b_seq0.npz"))
    ap.add_argument("--check-prefix", type=int, default=0, metavar="N",
                    help="instead: run the first N prompt ids through both the oracle and the reference "
                         "and require bit-identical logits after every one")
    args = ap.parse_args()
    if args.check_prefix:
        return check_prefix(args.check_prefix)
    path = model_path().encode()
    V = TARGET["n_vocab"]
    ids = prompt()
    lg = np.zeros(V, np.float32)
    t0 = time.time()
    if args.reference:
        R = ref()
        R.vx_set_n_threads(os.cpu_count() or 1)
        h = ctypes.c_void_p()
        assert R.vx_model_create(path, ctypes.byref(h)) == 0
        fwd = lambda tok: R.vx_model_forward(h, f32p(np.array([tok], np.int32)), 1, f32p(lg))
        done = lambda: R.vx_model_destroy(h)
        source = "reference vx_model_forward (oracle/_ref/libvxref.so, scalar build)"
    else:
        O = oracle()
        om = O.vxo_model_load(path, 1024)
        assert om
        fwd = lambda tok: O.vxo_forward(om, f32p(np.array([tok], np.int32)), 1, f32p(lg))
        done = lambda: O.vxo_model_free(om)
        source = "oracle vxo_forward (oracle/vxo_fwd.c)"
    for i, t in enumerate(ids):
        assert fwd(int(t)) == 0
        if i % 64 == 63:
            print(f"prompt {i + 1}/{PROMPT_LEN}  {time.time() - t0:.0f} s", flush=True)
    last_prompt_logits = lg.copy()
    gen, margins = [], []
    for _ in range(N_NEW):
        top2 = np.partition(lg, -2)[-2:]
        best = int(np.argmax(lg))
        gen.append(best)
        margins.append(float(top2[1] - top2[0]))
        assert fwd(best) == 0
    done()
    out = args.out
    np.savez_compressed(out, prompt=ids, greedy=np.array(gen, np.int32), margins=np.array(margins, np.float32),
                        last_prompt_logits=last_prompt_logits, source=np.array(source))
    print("greedy", gen, "min margin", min(margins), f"{time.time() - t0:.0f} s ->", out)


if __name__ == "__main__":
    sys.exit(main())
