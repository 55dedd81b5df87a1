"""GPU parity: quantised GEMV against the CPU oracle, through the C-ABI.
vxc_qgemv runs the streaming CUDA-core kernel for M <= 2, the tcgen05 GEMV
up to 63 rows and the tcgen05 GEMM (weights converted once per 256-row
slab) from 64 rows on; vxc_qgemv_simt is the plain CUDA-core cross-check.

Tolerance: the kernels accumulate in fp32 from exact integer weights and a
22-bit activation split (tensor-core path) or fp32 activations (CUDA-core
paths); they differ from the reference only in summation order, so
max|y_gpu - y_oracle| <= 2e-5 * max|y_oracle| (K <= 11008).
"""
import ctypes

import numpy as np
import pytest

from _paths import oracle
from qgen import q4_0_blocks, q8_0_blocks

pytestmark = pytest.mark.gpu
TOL = 2e-5


def run_case(torch, qt, rows, cols, M, simt, seed=0):
    import vxb200
    rng = np.random.default_rng(seed)
    blk = (q4_0_blocks if qt == 2 else q8_0_blocks)(rows, cols, rng)
    x = rng.standard_normal((M, cols)).astype(np.float32)
    O = oracle()
    yo = np.zeros((M, rows), np.float32)
    O.vxo_qgemv(qt, blk.ctypes.data, x.ctypes.data, yo.ctypes.data, M, rows, cols)
    W = vxb200.QMat(qt, blk, rows, cols)
    xd = torch.from_numpy(x).cuda()
    yd = torch.full((M, rows), float("nan"), device="cuda")
    wsb = max(W.workspace_bytes(M), 4)
    ws = torch.empty(wsb // 4 + 1, device="cuda")
    W.gemv(xd.data_ptr(), M, yd.data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream, simt=simt)
    torch.cuda.synchronize()
    code = ctypes.c_uint(0)
    assert vxb200.lib().vxc_check_device_error(ctypes.byref(code)) == 0, code.value
    y = yd.cpu().numpy()
    W.close()
    err = np.max(np.abs(y - yo))
    return err, np.max(np.abs(yo))


@pytest.mark.parametrize("simt", [False, True])
@pytest.mark.parametrize("qt", [2, 8])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (11008, 4096)])
@pytest.mark.parametrize("M", [1, 2, 5, 8])
def test_config2_shapes(cuda, qt, rows, cols, M, simt):
    err, mx = run_case(cuda, qt, rows, cols, M, simt)
    assert err <= TOL * mx, (err, mx)


@pytest.mark.parametrize("qt", [2, 8])
@pytest.mark.parametrize("rows,cols,M", [(100, 256, 3), (130, 64, 1), (4096, 11008, 5), (257, 2048, 17),
                                         (384, 4096, 40), (512, 1024, 64), (640, 512, 100), (32000, 256, 5)])
def test_edge_shapes(cuda, qt, rows, cols, M):
    """Ragged row tiles, the smallest K, M beyond one N tile and beyond 64."""
    err, mx = run_case(cuda, qt, rows, cols, M, simt=False, seed=rows + M)
    assert err <= TOL * mx, (err, mx)


def test_zero_and_large_activations(cuda):
    """All-zero rows must give exact zeros; rows spanning 1e-30..1e30 exercise
    the per-row power-of-two prescale of the activation split."""
    import vxb200
    torch = cuda
    rng = np.random.default_rng(9)
    rows, cols, M = 256, 512, 4
    blk = q4_0_blocks(rows, cols, rng)
    x = rng.standard_normal((M, cols)).astype(np.float32)
    x[0] = 0
    x[1] *= 1e30
    x[2] *= 1e-30
    O = oracle()
    yo = np.zeros((M, rows), np.float32)
    O.vxo_qgemv(2, blk.ctypes.data, x.ctypes.data, yo.ctypes.data, M, rows, cols)
    W = vxb200.QMat(2, blk, rows, cols)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((M, rows), device="cuda")
    wsb = max(W.workspace_bytes(M), 4)
    ws = torch.empty(wsb // 4 + 1, device="cuda")
    W.gemv(xd.data_ptr(), M, yd.data_ptr(), ws.data_ptr(), wsb)
    y = yd.cpu().numpy()
    assert np.all(y[0] == 0)
    for m in (1, 2, 3):
        assert np.max(np.abs(y[m] - yo[m])) <= TOL * np.max(np.abs(yo[m]))


def test_skinny_rows_do_not_depend_on_m(cuda):
    """One and two activation rows share one accumulation order: row 0 of a
    two-row call equals the one-row call bit for bit."""
    import vxb200
    torch = cuda
    rng = np.random.default_rng(21)
    for qt, rows, cols in ((2, 4096, 4096), (8, 2560, 2048)):
        blk = (q4_0_blocks if qt == 2 else q8_0_blocks)(rows, cols, rng)
        W = vxb200.QMat(qt, blk, rows, cols)
        x = torch.from_numpy(rng.standard_normal((2, cols)).astype(np.float32)).cuda()
        ys = []
        for M in (1, 2):
            wsb = max(W.workspace_bytes(M), 4)
            ws = torch.empty(wsb // 4 + 1, device="cuda")
            y = torch.empty((M, rows), device="cuda")
            W.gemv(x.data_ptr(), M, y.data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            ys.append(y.cpu().numpy())
        W.close()
        assert np.array_equal(ys[0][0], ys[1][0]), qt


@pytest.mark.parametrize("qt,rows,cols,M", [(2, 4096, 4096, 96), (8, 2560, 2048, 300), (2, 384, 11008, 64),
                                            (8, 300, 2048, 520), (2, 32000, 256, 65), (8, 130, 4096, 257),
                                            (2, 1000, 1024, 1111)])
def test_gemm_shapes(cuda, qt, rows, cols, M):
    """The GEMM path: full and ragged 256-row slabs, a single weight tile in
    the last pair (odd tile counts), ragged weight rows, K up to 11008."""
    err, mx = run_case(cuda, qt, rows, cols, M, simt=False, seed=3 * rows + M)
    assert err <= TOL * mx, (err, mx)


def test_gemm_rows_do_not_depend_on_m(cuda):
    """A row's GEMM result depends on that row only: the same rows give the
    same bits whether the call has 64, 300 or 600 rows (other slabs, another
    slab position, other rows beside them)."""
    import vxb200
    torch = cuda
    rng = np.random.default_rng(33)
    for qt, rows, cols in ((2, 4096, 4096), (8, 2560, 2048)):
        blk = (q4_0_blocks if qt == 2 else q8_0_blocks)(rows, cols, rng)
        W = vxb200.QMat(qt, blk, rows, cols)
        x = torch.from_numpy(rng.standard_normal((600, cols)).astype(np.float32)).cuda()
        ys = {}
        for M in (64, 300, 600):
            wsb = max(W.workspace_bytes(M), 4)
            ws = torch.empty(wsb // 4 + 1, device="cuda")
            y = torch.empty((M, rows), device="cuda")
            W.gemv(x.data_ptr(), M, y.data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            ys[M] = y.cpu().numpy()
        # a call whose first row is row 100 of x: every row sits at another place in its slab
        wsb = max(W.workspace_bytes(300), 4)
        ws = torch.empty(wsb // 4 + 1, device="cuda")
        y = torch.empty((300, rows), device="cuda")
        W.gemv(x[100:400].data_ptr(), 300, y.data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        shifted = y.cpu().numpy()
        W.close()
        assert np.array_equal(ys[64], ys[300][:64]), qt
        assert np.array_equal(ys[300], ys[600][:300]), qt
        assert np.array_equal(ys[600][100:400], shifted), qt
