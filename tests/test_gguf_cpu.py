"""The host library's GGUF reader (veltrix-engine_b200/host/vxh_gguf.c) on
valid, truncated and corrupted files, without a GPU.

The reader maps the file and hands pointers into the mapping to the device
upload, so a length or offset that points past the end of the file must be
refused before anything reads there: a truncated download would otherwise
end the caller's process with SIGBUS.  The reference refuses such a file with
VX_ERR_FORMAT (src/gguf.c:257-275: a tensor whose bytes, sized as
src/quantize.c:59-85 sizes them, run past the end of the file), and so must
the reader.  Valid files written by the library's own writer parse with the
hyper-parameters they were written with (src/gguf.c:524-551 keys).
"""
import ctypes
import os
import struct

import numpy as np
import pytest

import _paths  # noqa: F401  (puts the package on sys.path)
import fixtures

VX_ERR_FORMAT = -2


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 128), ("type", ctypes.c_int), ("n_dims", ctypes.c_int),
                ("ne", ctypes.c_int64 * 4), ("data", ctypes.c_void_p)]


class _Gguf(ctypes.Structure):
    """host/vxh_gguf.h vxh_gguf."""
    _fields_ = [("map", ctypes.c_void_p), ("size", ctypes.c_size_t), ("n_tensors", ctypes.c_int),
                ("t", ctypes.POINTER(_Tensor)), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("n_embd", ctypes.c_int), ("n_ff", ctypes.c_int),
                ("n_vocab", ctypes.c_int), ("rope_theta", ctypes.c_float), ("arch", ctypes.c_char * 64)]


@pytest.fixture(scope="module")
def lib():
    import vxb200
    L = vxb200.lib()
    L.vxh_gguf_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Gguf)]
    L.vxh_gguf_open.restype = ctypes.c_int
    L.vxh_gguf_close.argtypes = [ctypes.POINTER(_Gguf)]
    return L


def gguf_open(L, path):
    """(rc, hyper-parameters, [(name, type, ne, data offset)]) of one open."""
    g = _Gguf()
    rc = L.vxh_gguf_open(str(path).encode(), ctypes.byref(g))
    if rc:
        return rc, None, None
    hp = (g.n_layers, g.n_heads, g.n_kv_heads, g.n_embd, g.n_ff, g.n_vocab, g.rope_theta)
    ts = [(g.t[i].name.decode(), g.t[i].type, tuple(g.t[i].ne), g.t[i].data - g.map) for i in range(g.n_tensors)]
    L.vxh_gguf_close(ctypes.byref(g))
    return rc, hp, ts


def layout(buf):
    """Offsets of the fields of a GGUF v3 file: per KV (key-length offset,
    value-type offset, value offset), per tensor info (name-length offset,
    dims offset, type offset, data-offset offset), and where the data
    section starts."""
    nt, nkv = struct.unpack_from("<QQ", buf, 8)
    o, kvs, tis = 24, [], []

    def skip(o, t):
        w = {0: 1, 1: 1, 7: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 10: 8, 11: 8, 12: 8}
        if t in w:
            return o + w[t]
        if t == 8:
            return o + 8 + struct.unpack_from("<Q", buf, o)[0]
        at, n = struct.unpack_from("<IQ", buf, o)
        o += 12
        for _ in range(n):
            o = skip(o, at)
        return o

    for _ in range(nkv):
        k0 = o
        kl = struct.unpack_from("<Q", buf, o)[0]
        o += 8 + kl
        vt = struct.unpack_from("<I", buf, o)[0]
        kvs.append((k0, o, o + 4, vt))
        o = skip(o + 4, vt)
    for _ in range(nt):
        n0 = o
        nl = struct.unpack_from("<Q", buf, o)[0]
        o += 8 + nl
        nd = struct.unpack_from("<I", buf, o)[0]
        d0 = o + 4
        o = d0 + 8 * nd
        tis.append((n0, d0, o, o + 4))
        o += 12
    return kvs, tis, o + (32 - o % 32) % 32


@pytest.fixture(scope="module")
def tiny():
    p = fixtures.path("tiny_draft")
    with open(p, "rb") as f:
        return p, f.read()


def put(tmp_path, name, data):
    p = tmp_path / name
    p.write_bytes(data)
    return p


def test_valid_files_parse_with_their_hyper_parameters(lib):
    for name in ("tiny_target", "tiny_draft", "tiny_q4k", "tiny_kqmix"):
        e, L, h, kv, ff, v, wt, seed, th = fixtures.CONFIGS[name]
        rc, hp, ts = gguf_open(lib, fixtures.path(name))
        assert rc == 0, name
        assert hp == (L, h, kv, e, ff, v, th), name
        assert len(ts) == 3 + 9 * L, name
        # the last tensor ends exactly at the end of the file
        assert max(t[3] for t in ts) < os.path.getsize(fixtures.path(name))


def test_truncated_files_are_refused(lib, tiny, tmp_path):
    path, buf = tiny
    kvs, tis, data0 = layout(buf)
    assert gguf_open(lib, path)[0] == 0
    # every cut inside the header, the KV section and the tensor infos, a
    # sample of cuts inside the data section, and one byte short of the end
    rng = np.random.default_rng(3)
    cuts = list(range(0, data0 + 1)) + sorted(rng.integers(data0 + 1, len(buf), 40).tolist()) + [len(buf) - 1]
    for c in cuts:
        p = put(tmp_path, "cut.gguf", buf[:c])
        rc = gguf_open(lib, p)[0]
        assert rc == VX_ERR_FORMAT, (c, rc)


def test_lengths_and_offsets_outside_the_file_are_refused(lib, tiny, tmp_path):
    path, buf = tiny
    kvs, tis, data0 = layout(buf)
    huge = [2 ** 64 - 1, 2 ** 63, 2 ** 64 - 8, len(buf)]
    cases = []
    for v in huge:
        cases.append(("key length", kvs[0][0], v))
        cases.append(("tensor name length", tis[0][0], v))
        cases.append(("tensor data offset", tis[-1][3], v))
    # a string value (general.architecture is the first KV the writer emits)
    str_kv = [k for k in kvs if k[3] == 8]
    assert str_kv
    for v in huge:
        cases.append(("string length", str_kv[0][2], v))
    # a dimension that no file can hold, and one that makes the tensor end past the file
    cases.append(("dimension", tis[0][1], 2 ** 62))
    cases.append(("dimension", tis[-1][1], 10 ** 9))
    for what, off, v in cases:
        b = bytearray(buf)
        struct.pack_into("<Q", b, off, v)
        rc = gguf_open(lib, put(tmp_path, "bad.gguf", bytes(b)))[0]
        assert rc == VX_ERR_FORMAT, (what, v, rc)
    # a tensor type whose block size is known must fit too: the last tensor
    # in the file, Q8_0 (34 bytes per 32 weights), retyped as F32 (128 bytes)
    rc, _, ts = gguf_open(lib, path)
    last = max(range(len(ts)), key=lambda i: ts[i][3])
    b = bytearray(buf)
    ty_off = tis[last][2]
    assert struct.unpack_from("<I", b, ty_off)[0] == 8
    struct.pack_into("<I", b, ty_off, 0)
    assert gguf_open(lib, put(tmp_path, "bad.gguf", bytes(b)))[0] == VX_ERR_FORMAT


def minimal(kv_value_type, kv_value):
    """A GGUF with one KV pair ("x") and no tensors."""
    return (struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + struct.pack("<Q", 1) + b"x"
            + struct.pack("<I", kv_value_type) + kv_value)


def nested(levels):
    """An array value `levels` arrays deep, one element per level, with one
    u32 in the innermost array."""
    body = struct.pack("<IQ", 4, 1) + struct.pack("<I", 7)
    for _ in range(levels - 1):
        body = struct.pack("<IQ", 9, 1) + body
    return body


def test_nested_arrays(lib, tmp_path):
    # GGUF arrays of arrays parse a few levels deep; a deeper nesting is
    # refused instead of recursing once per level
    assert gguf_open(lib, put(tmp_path, "n2.gguf", minimal(9, nested(2))))[0] == 0
    assert gguf_open(lib, put(tmp_path, "n8.gguf", minimal(9, nested(8))))[0] == 0
    assert gguf_open(lib, put(tmp_path, "n9.gguf", minimal(9, nested(9))))[0] == VX_ERR_FORMAT
    assert gguf_open(lib, put(tmp_path, "deep.gguf", minimal(9, nested(100000))))[0] == VX_ERR_FORMAT
    # an array whose count runs past the end of the file
    big = struct.pack("<IQ", 4, 2 ** 62) + b"\0" * 16
    assert gguf_open(lib, put(tmp_path, "cnt.gguf", minimal(9, big)))[0] == VX_ERR_FORMAT


def test_bad_magic_and_short_files(lib, tiny, tmp_path):
    path, buf = tiny
    assert gguf_open(lib, put(tmp_path, "magic.gguf", b"GGUG" + buf[4:]))[0] == VX_ERR_FORMAT
    assert gguf_open(lib, put(tmp_path, "empty.gguf", b""))[0] == VX_ERR_FORMAT
    assert gguf_open(lib, tmp_path / "missing.gguf")[0] == -1   # VX_ERR_FILE
