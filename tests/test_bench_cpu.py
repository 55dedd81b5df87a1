"""bench.py checks that need no GPU: every name a function reads is defined
somewhere (a typo in a workload runner would otherwise only show on a GPU
box), and the reference arm of the 70B workload answers with its
`unavailable` line."""
import builtins
import json
import os
import subprocess
import sys
import symtable

from _paths import ROOT


def test_bench_has_no_undefined_names():
    src = open(os.path.join(ROOT, "bench.py")).read()
    top = symtable.symtable(src, "bench.py", "exec")
    glob = set(top.get_identifiers())
    bad = []

    def walk(t, enclosing):
        for sym in t.get_symbols():
            n = sym.get_name()
            if sym.is_referenced() and not (sym.is_local() or sym.is_parameter() or sym.is_imported()):
                if n not in glob and n not in enclosing and not hasattr(builtins, n):
                    bad.append((t.get_name(), n))
        for c in t.get_children():
            walk(c, enclosing | set(t.get_identifiers()))

    walk(top, set())
    assert not bad, bad


def test_spec70b_reference_arm_is_unavailable():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--workload", "spec70b"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def _reference_line(workload):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                        workload, "--steps", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_accept_and_tiny_reference_arms_print_their_lines():
    for workload, unit in (("accept", "GB/s"), ("spec_tiny", "tok/s")):
        line = _reference_line(workload)
        assert line["impl"] == "reference" and line["unit"] == unit and line["value"] > 0
        assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["value"] == line["value"]


def test_roofline_arithmetic_matches_the_configuration_figures():
    """Bytes and flops the bench divides by: 70B target 69.50 G weights and
    39.09 GB of Q4_0 (LM head included, embedding excluded), 3.11e13 flop per
    224-row verify (2 x rows x weights; the exact scheme's MMA work is 3x
    that, three fp16 products per weight x activation, no padding at 224
    rows), 7B target 3.7165 GB, acceptance 90.1 MB."""
    sys.path.insert(0, ROOT)
    import bench
    w70 = bench.target_weights(bench.SPEC70_TARGET)
    assert abs(w70 - 69.50e9) < 0.01e9
    assert abs(bench.model_bytes(bench.SPEC70_TARGET) - 39.09e9) < 0.01e9
    assert abs(2 * 224 * w70 - 3.11e13) < 0.01e13
    assert bench.verify_mma_flops(224, w70) == 3 * 2 * 224 * w70
    assert bench.verify_mma_flops(40, 1) == 6 * 48          # 40 rows pad to N = 48 (GEMV)
    assert bench.verify_mma_flops(300, 1) == 6 * (256 + 48)  # GEMM slabs of 256 rows, each padded
    assert abs(bench.model_bytes(bench.SPEC_TARGET) - 3.7165e9) < 0.001e9
    assert abs(bench.accept_bytes() - 90.1e6) < 0.1e6


def test_first_tokens_check_against_the_committed_golden():
    """The spec7b line's `first_tokens_vs_oracle` field: sequence 0's first
    tokens against tests/golden/spec7b_seq0.npz under the margin rule."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import bench
    g = np.load(bench.GOLDEN_SEQ0)
    assert np.array_equal(g["prompt"], bench.spec_prompts(0, 1)[0])
    want = [int(t) for t in g["greedy"][:8]]
    ok = bench.first_tokens_vs_golden(want)
    assert ok["match"] is True and ok["identical_prefix"] == 8 and ok["compared"] == 8
    # a different token where the CPU margin is clear fails the check
    i = int(np.argmax(g["margins"][:8] > 1e-3))
    bad = list(want)
    bad[i] = (bad[i] + 1) % 32000
    r = bench.first_tokens_vs_golden(bad)
    assert r["match"] is False and r["identical_prefix"] == i
    # other workloads have no golden
    bench.TINY = True
    try:
        assert bench.first_tokens_vs_golden(want) is None
    finally:
        bench.TINY = False
