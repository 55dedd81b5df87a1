"""ctypes binding of libveltrix_b200.so (the C-ABI in include/veltrix_cuda.h,
include/model.h and include/speculative.h).

The library is built in-tree by ``make -C veltrix-engine_b200``.  Loading fails
loudly when it is missing: there is no Python or CPU fallback for any kernel.
Device buffers are passed as raw pointers (``int``), e.g. a torch CUDA
tensor's ``data_ptr()``; torch is only used by callers for allocation.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libveltrix_b200.so")

_c_int_p = ctypes.POINTER(ctypes.c_int)
_c_float_p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p

# name -> (restype, argtypes); every symbol declared in include/*.h
PROTOTYPES = {
    # veltrix_cuda.h
    "vxc_device_init": (ctypes.c_int, [ctypes.c_int]),
    "vxc_device_count": (ctypes.c_int, []),
    "vxc_error_string": (ctypes.c_char_p, []),
    "vxc_check_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "vxc_qmat_create": (ctypes.c_int, [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
    "vxc_qmat_destroy": (None, [_vp]),
    "vxc_qmat_shape": (ctypes.c_int, [_vp, _c_int_p, _c_int_p, _c_int_p]),
    "vxc_qgemv_workspace_bytes": (ctypes.c_size_t, [_vp, ctypes.c_int]),
    "vxc_qgemv": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_size_t, _vp]),
    "vxc_qgemv_simt": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_size_t, _vp]),
}

_lib = None


class VxError(RuntimeError):
    pass


def lib():
    """Load (once) and return the library with prototypes applied."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise VxError(f"{LIB_PATH} is missing: build it with `make -C veltrix-engine_b200`")
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc, what=""):
    if rc != 0:
        msg = lib().vxc_error_string()
        raise VxError(f"{what} failed with {rc}: {msg.decode() if msg else ''}")


class QMat:
    """A quantised weight matrix resident on the current CUDA device."""

    def __init__(self, qtype, blocks, rows, cols):
        import numpy as np
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        h = _vp()
        check(lib().vxc_qmat_create(qtype, blocks.ctypes.data, rows, cols, ctypes.byref(h)), "vxc_qmat_create")
        self.h = h
        self.qtype, self.rows, self.cols = qtype, rows, cols

    def workspace_bytes(self, M):
        return lib().vxc_qgemv_workspace_bytes(self.h, M)

    def gemv(self, x_ptr, M, y_ptr, ws_ptr, ws_bytes, stream=0, simt=False):
        fn = lib().vxc_qgemv_simt if simt else lib().vxc_qgemv
        check(fn(self.h, x_ptr, M, y_ptr, ws_ptr, ws_bytes, stream), "vxc_qgemv")

    def close(self):
        if self.h:
            lib().vxc_qmat_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
