"""Shared paths and ctypes loaders for the tests (test infrastructure only)."""
import ctypes
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "veltrix-engine_b200")
ORACLE = os.path.join(ROOT, "oracle")
REF_DIR = os.path.join(ORACLE, "_ref")
if PKG not in sys.path:
    sys.path.insert(0, PKG)

_c_int_p = ctypes.POINTER(ctypes.c_int)
_vp = ctypes.c_void_p


def build_oracle():
    so = os.path.join(ORACLE, "libvxoracle.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", ORACLE], check=True, capture_output=True)
    return so


def oracle():
    L = ctypes.CDLL(build_oracle())
    L.vxo_fp16_to_fp32.restype = ctypes.c_float
    L.vxo_fp16_to_fp32.argtypes = [ctypes.c_uint16]
    L.vxo_fp32_to_fp16_trunc.restype = ctypes.c_uint16
    L.vxo_fp32_to_fp16_trunc.argtypes = [ctypes.c_float]
    for n in ("vxo_quantize_row_q4_0", "vxo_quantize_row_q8_0", "vxo_dequant_q4_0", "vxo_dequant_q8_0"):
        getattr(L, n).argtypes = [_vp, _vp, ctypes.c_int]
    L.vxo_qgemv.argtypes = [ctypes.c_int, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.vxo_rms_norm.argtypes = [_vp, _vp, _vp, ctypes.c_int]
    L.vxo_softmax.argtypes = [_vp, ctypes.c_int]
    L.vxo_rope.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    L.vxo_silu.argtypes = [_vp, ctypes.c_int]
    L.vxo_model_load.restype = _vp
    L.vxo_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.vxo_model_free.argtypes = [_vp]
    L.vxo_model_config.argtypes = [_vp, _c_int_p]
    L.vxo_model_rope_theta.restype = ctypes.c_float
    L.vxo_model_rope_theta.argtypes = [_vp]
    L.vxo_model_cache_len.argtypes = [_vp]
    L.vxo_model_set_cache_len.argtypes = [_vp, ctypes.c_int]
    L.vxo_forward.argtypes = [_vp, _vp, ctypes.c_int, _vp]
    L.vxo_forward_all.argtypes = [_vp, _vp, ctypes.c_int, _vp]
    L.vxo_philox_u32.restype = ctypes.c_uint32
    L.vxo_philox_u32.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
    L.vxo_philox4x32_10.argtypes = [_vp, _vp, _vp]
    L.vxo_expf.restype = ctypes.c_float
    L.vxo_expf.argtypes = [ctypes.c_float]
    L.vxo_argmax.argtypes = [_vp, ctypes.c_int]
    L.vxo_sample.argtypes = [_vp, ctypes.c_int, ctypes.c_float, ctypes.c_uint32]
    L.vxo_accept.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_uint64,
                             ctypes.c_uint32, ctypes.c_uint32, _c_int_p]
    L.vxo_greedy_generate.argtypes = [_vp, _vp, ctypes.c_int, _vp, ctypes.c_int]
    L.vxo_spec_generate.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_uint64,
                                    ctypes.c_uint32, _vp, ctypes.c_int, _c_int_p]
    return L


def ref_available():
    return os.path.exists(os.path.join(REF_DIR, "libvxref.so")) or os.path.isdir("/root/reference/src")


def ref(ship=False):
    """The reference's own sources compiled by oracle/Makefile (scalar or as-shipped)."""
    name = "libvxref_ship.so" if ship else "libvxref.so"
    so = os.path.join(REF_DIR, name)
    if not os.path.exists(so):
        subprocess.run(["make", "-C", ORACLE, "ref"], check=True, capture_output=True)
    L = ctypes.CDLL(so)
    L.vx_fp16_to_fp32.restype = ctypes.c_float
    L.vx_fp16_to_fp32.argtypes = [ctypes.c_uint16]
    L.vx_fp32_to_fp16.restype = ctypes.c_uint16
    L.vx_fp32_to_fp16.argtypes = [ctypes.c_float]
    L.vx_quantize_row_q4_0.argtypes = [_vp, _vp, ctypes.c_int]
    L.vx_dequantize_row_q4_0.argtypes = [_vp, _vp, ctypes.c_int]
    L.vx_dequantize_row_q8_0.argtypes = [_vp, _vp, ctypes.c_int]
    L.vx_gemv_q4_0.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
    L.vx_gemv_f32.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
    L.vx_rms_norm.argtypes = [_vp, _vp, _vp, ctypes.c_int]
    L.vx_softmax.argtypes = [_vp, ctypes.c_int]
    L.vx_rope.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                          ctypes.c_float]
    L.vx_silu.argtypes = [_vp, ctypes.c_int]
    L.vx_model_create.argtypes = [ctypes.c_char_p, ctypes.POINTER(_vp)]
    L.vx_model_destroy.argtypes = [_vp]
    L.vx_model_forward.argtypes = [_vp, _vp, ctypes.c_int, _vp]
    L.vxref_cache_len.argtypes = [_vp]
    L.vxref_set_cache_len.argtypes = [_vp, ctypes.c_int]
    L.vxref_config.argtypes = [_vp, _c_int_p]
    L.vx_set_n_threads.argtypes = [ctypes.c_int]
    if ship:
        L.vx_gemv_q4_0_avx2.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
    return L
