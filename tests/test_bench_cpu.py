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
