"""C-ABI checks that need no GPU: the library loads, exports every function
declared in include/*.h, and the public struct layout matches the
reference's include/veltrix.h (callers read/write vx_model fields)."""
import ctypes
import os
import re
import subprocess

import pytest

from _paths import ROOT

HEADERS = ["veltrix.h", "model.h", "speculative.h", "veltrix_cuda.h", "veltrix_synth.h"]


def declared_functions():
    names = set()
    for h in HEADERS:
        p = os.path.join(ROOT, "include", h)
        if not os.path.exists(p):
            continue
        src = open(p).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(vx\w+)\s*\(", src, flags=re.M):
            if "typedef" in m.group(0):
                continue
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    import vxb200
    L = vxb200.lib()
    names = declared_functions()
    assert len(names) > 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_binding_prototypes_cover_headers():
    import vxb200
    missing = [n for n in declared_functions() if n not in vxb200.PROTOTYPES]
    assert not missing, missing


def test_vx_model_layout_matches_c(tmp_path):
    """offsetof(vx_model, cache_len/config.n_ctx) in C == the ctypes mirror."""
    import vxb200
    src = tmp_path / "o.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "veltrix.h"\n'
                   'int main(){printf("%zu %zu %zu\\n", offsetof(vx_model, cache_len), '
                   'offsetof(vx_model, config.n_ctx), sizeof(vx_model_config));return 0;}\n')
    exe = tmp_path / "o"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    a, b, c = map(int, subprocess.run([str(exe)], capture_output=True, text=True).stdout.split())
    assert a == vxb200.ModelHead.cache_len.offset
    assert b == vxb200.ModelConfig.n_ctx.offset
    assert c == ctypes.sizeof(vxb200.ModelConfig)


def test_no_device_fails_loudly():
    """Without a CUDA device every entry point fails: no CPU fallback."""
    import vxb200
    L = vxb200.lib()
    if L.vxc_device_count() > 0:
        pytest.skip("a CUDA device is present")
    assert L.vxc_device_init(0) != 0
    assert b"no CUDA device" in L.vxc_error_string()
    h = ctypes.c_void_p()
    assert L.vx_model_create(b"/nonexistent.gguf", ctypes.byref(h)) != 0
    # the additive entry points fail the same way
    cfg = vxb200.SynthConfig(256, 2, 8, 8, 768, 4096, 10000.0, 2)
    assert L.vx_model_create_synth(ctypes.byref(cfg), 1, 0, 1, None, ctypes.byref(h)) != 0
    assert L.vx_model_create_tp(b"/nonexistent.gguf", 0, 2, b"\0" * 128, ctypes.byref(h)) != 0


def test_additive_entry_points_check_arguments():
    """Argument errors are reported before any device work (vx_error codes)."""
    import vxb200
    L = vxb200.lib()
    h = ctypes.c_void_p()
    VX_ERR_PARAM = -4
    cfg = vxb200.SynthConfig(256, 2, 8, 8, 768, 4096, 10000.0, 2)
    assert L.vx_model_create_tp(None, 0, 2, b"\0" * 128, ctypes.byref(h)) == VX_ERR_PARAM
    assert L.vx_model_create_tp(b"x.gguf", 2, 2, b"\0" * 128, ctypes.byref(h)) == VX_ERR_PARAM   # rank >= world
    assert L.vx_model_create_tp(b"x.gguf", 0, 2, None, ctypes.byref(h)) == VX_ERR_PARAM
    assert L.vx_model_create_synth(ctypes.byref(cfg), 1, 0, 2, None, ctypes.byref(h)) == VX_ERR_PARAM  # no id
    assert L.vx_model_create_synth(None, 1, 0, 1, None, ctypes.byref(h)) == VX_ERR_PARAM
    assert L.vx_model_generate_greedy(None, None, 0, None, 1, -1) == VX_ERR_PARAM
    # the writer rejects K-quant widths that are not whole super-blocks
    bad = vxb200.SynthConfig(128, 1, 4, 4, 384, 256, 10000.0, 12)
    assert L.vx_synth_write_gguf(b"/tmp/never_written.gguf", ctypes.byref(bad), 1) == VX_ERR_PARAM


REF_INCLUDE = "/root/reference/include"


@pytest.mark.skipif(not os.path.isdir(REF_INCLUDE), reason="reference headers not present on this machine")
def test_vx_model_layout_matches_reference_header(tmp_path):
    """The same C program compiled against the reference's include/veltrix.h
    and against this repository's prints identical offsets for every field a
    caller of the reference API can read or poke, and identical error codes."""
    src = tmp_path / "lay.c"
    fields = ["config", "config.n_layers", "config.n_vocab", "config.n_ctx", "config.rope_theta",
              "config.has_ffn_bias", "tensors", "n_tensors", "tok_embd", "attn_q", "output_w",
              "k_cache", "v_cache", "cache_len"]
    body = "".join(f'printf("%zu\\n", offsetof(vx_model, {f}));' for f in fields)
    codes = "".join(f'printf("%d\\n", (int){c});' for c in
                    ("VX_OK", "VX_ERR_FILE", "VX_ERR_FORMAT", "VX_ERR_MEMORY", "VX_ERR_PARAM", "VX_ERR_GGUF",
                     "VX_ERR_NOMODEL", "VX_ERR_UNSUPPORTED"))
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "model.h"\n#include "speculative.h"\n'
                   'int main(){' + body + codes + 'printf("%zu\\n", sizeof(vx_model_config));return 0;}\n')
    outs = []
    for inc in (REF_INCLUDE, os.path.join(ROOT, "include")):
        exe = tmp_path / ("lay_" + str(len(outs)))
        subprocess.run(["gcc", "-I", inc, str(src), "-o", str(exe)], check=True)
        outs.append(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split())
    assert outs[0] == outs[1]
