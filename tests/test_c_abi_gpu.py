"""The drop-in boundary from C: tests/c_abi/_build/ref_driver is compiled
against the reference's own public headers (include/model.h,
include/speculative.h, include/veltrix.h of the reference) and linked against
libveltrix_b200.so (tests/c_abi/Makefile, run by __graft_entry__.build()).
It decodes configuration 1 through vx_model_forward and
vx_speculative_generate; the streams must match the reference's greedy golden
(wherever its top-2 margin exceeds 1e-3), and a cache_len written by the
caller must be honoured."""
import os
import subprocess

import numpy as np
import pytest

import fixtures

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
DRIVER = os.path.join(HERE, "c_abi", "_build", "ref_driver")


def test_reference_header_caller(cuda):
    assert os.path.exists(DRIVER), "tests/c_abi/_build/ref_driver is missing: run __graft_entry__.build()"
    g = np.load(os.path.join(HERE, "golden", "tiny_target.npz"))
    n = len(g["greedy"])
    r = subprocess.run([DRIVER, fixtures.path("tiny_target"), fixtures.path("tiny_draft"), str(n)],
                       input=" ".join(str(int(v)) for v in g["prompt"]), capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = {l.split()[0]: l.split()[1:] for l in r.stdout.strip().splitlines()}
    greedy = np.array([int(v) for v in lines["greedy"]])
    spec = np.array([int(v) for v in lines["spec"]])
    assert len(greedy) == n and len(spec) == n
    ref = g["greedy"]
    for i in range(n):
        if greedy[i] != ref[i]:
            assert g["margins"][i] <= 1e-3, (i, greedy[i], ref[i])
            break
    # greedy speculative decoding is target-only greedy decoding
    assert np.array_equal(spec, greedy)
    assert int(lines["cache_len"][0]) == len(g["prompt"])
