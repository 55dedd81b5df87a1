"""K-quant matrices on the device (vxc_kquant.cu) against the K-quant
oracle (oracle/vxo_kquant.c, itself pinned bit for bit to the reference
build by test_kquant_cpu.py), for Q2_K, Q3_K, Q4_K, Q5_K, Q6_K and Q8_K:

- vxc_kquant_dequant: the decoded weights equal the reference's bit for bit;
- vxc_qgemv: y = decoded(W) . x within 1e-5 x max|y| of the oracle's
  blockwise GEMV (fp32, only the order of the sum differs), at 1 and 11
  activation rows (more than one 8-row pass) and a row count that leaves
  a partial CTA.
"""
import ctypes

import numpy as np
import pytest

from _paths import oracle
from kqgen import TYPES, random_blocks

pytestmark = pytest.mark.gpu
vp = lambda a: a.ctypes.data_as(ctypes.c_void_p)


@pytest.mark.parametrize("t", sorted(TYPES))
def test_kquant_dequant_and_gemv(cuda, t):
    torch = cuda
    import vxb200
    O = oracle()
    O.vxo_dequant_kquant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    O.vxo_gemv_kquant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                  ctypes.c_int]
    rng = np.random.default_rng(500 + t)
    rows, cols = 300, 2048
    blk = random_blocks(t, rows * cols // 256, rng)
    W = vxb200.QMat(t, blk, rows, cols)
    assert W.workspace_bytes(11) == 0
    # decoded weights
    want_w = np.zeros(rows * cols, np.float32)
    assert O.vxo_dequant_kquant(t, vp(blk), vp(want_w), rows * cols) == 0
    dw = torch.full((rows * cols,), float("nan"), device="cuda")
    vxb200.check(vxb200.lib().vxc_kquant_dequant(W.h, ctypes.c_void_p(dw.data_ptr()), None), "vxc_kquant_dequant")
    torch.cuda.synchronize()
    assert np.array_equal(dw.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    # GEMV
    for M in (1, 11):
        x = rng.standard_normal((M, cols)).astype(np.float32)
        want = np.zeros((M, rows), np.float32)
        for m in range(M):
            assert O.vxo_gemv_kquant(t, vp(blk), vp(x[m]), vp(want[m]), rows, cols) == 0
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((M, rows), float("nan"), device="cuda")
        W.gemv(xd.data_ptr(), M, yd.data_ptr(), None, 0)
        torch.cuda.synchronize()
        got = yd.cpu().numpy()
        assert np.max(np.abs(got - want)) <= 1e-5 * np.max(np.abs(want)), (t, M)
    code = ctypes.c_uint(0)
    assert vxb200.lib().vxc_check_device_error(ctypes.byref(code)) == 0
    W.close()
