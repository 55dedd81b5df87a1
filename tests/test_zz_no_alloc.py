"""vxc_qgemv_noalloc: the GEMV entry point for callers that cannot allocate
device memory (an application that owns the device memory budget, or code
that cannot afford cudaMalloc's device synchronisation).  Its scratch is a
static device array inside the library.

Checked through the C-ABI: two calls in a row give the same result as
vxc_qgemv with a caller-provided workspace, and both agree with the CPU
oracle's GEMV (oracle/vxo_fwd.c vxo_qgemv, the reference's scalar
src/quantize.c:728-750 arithmetic) within 2e-5 x max|y| as in
test_gemv_gpu.py; no device memory is taken between the two calls, and a
shape whose scratch exceeds the static limit is rejected with an error.
This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from _paths import oracle
from qgen import q4_0_blocks, q8_0_blocks

pytestmark = pytest.mark.gpu
TOL = 2e-5


@pytest.mark.parametrize("qt,rows,cols,M", [(2, 4096, 4096, 5), (8, 11008, 4096, 8), (2, 4096, 11008, 1)])
def test_noalloc_matches_qgemv_twice(cuda, qt, rows, cols, M):
    torch = cuda
    import vxb200
    L = vxb200.lib()
    rng = np.random.default_rng(rows + M)
    blk = (q4_0_blocks if qt == 2 else q8_0_blocks)(rows, cols, rng)
    W = vxb200.QMat(qt, blk, rows, cols)
    x = torch.from_numpy(rng.standard_normal((M, cols)).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    # the existing entry point, with its own workspace
    wsb = max(W.workspace_bytes(M), 4)
    assert wsb <= 8 << 20      # VXC_QGEMV_NOALLOC_BYTES
    ws = torch.empty(wsb // 4 + 1, device="cuda")
    y_ref = torch.full((M, rows), float("nan"), device="cuda")
    W.gemv(x.data_ptr(), M, y_ref.data_ptr(), ws.data_ptr(), wsb, stream)
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    mx = float(np.max(np.abs(ref)))
    # the existing entry point against the oracle
    xh = x.cpu().numpy()
    yo = np.zeros((M, rows), np.float32)
    oracle().vxo_qgemv(qt, blk.ctypes.data, xh.ctypes.data, yo.ctypes.data, M, rows, cols)
    assert float(np.max(np.abs(ref - yo))) <= TOL * float(np.max(np.abs(yo)))
    free_after = []
    for _ in range(2):
        y = torch.full((M, rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        rc = L.vxc_qgemv_noalloc(W.h, ctypes.c_void_p(x.data_ptr()), M, ctypes.c_void_p(y.data_ptr()),
                                 ctypes.c_void_p(stream))
        assert rc == 0, L.vxc_error_string()
        torch.cuda.synchronize()
        code = ctypes.c_uint(0)
        assert L.vxc_check_device_error(ctypes.byref(code)) == 0, code.value
        free_after.append(torch.cuda.mem_get_info()[0])
        got = y.cpu().numpy()
        err = float(np.max(np.abs(got - ref)))
        assert err <= TOL * mx, (err, mx)
        assert float(np.max(np.abs(got - yo))) <= TOL * float(np.max(np.abs(yo)))
    # the second call allocates nothing on the device
    assert free_after[1] == free_after[0]
    W.close()


def test_noalloc_rejects_oversized(cuda):
    torch = cuda
    import vxb200
    L = vxb200.lib()
    rows, cols, M = 4096, 4096, 1024       # the GEMM's activation image alone is 16 MiB
    rng = np.random.default_rng(5)
    W = vxb200.QMat(2, q4_0_blocks(rows, cols, rng), rows, cols)
    assert W.workspace_bytes(M) > 8 << 20
    x = torch.zeros((M, cols), device="cuda")
    y = torch.zeros((M, rows), device="cuda")
    rc = L.vxc_qgemv_noalloc(W.h, ctypes.c_void_p(x.data_ptr()), M, ctypes.c_void_p(y.data_ptr()), None)
    assert rc != 0
    assert b"static limit" in L.vxc_error_string()
    W.close()
