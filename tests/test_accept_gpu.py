"""Configuration 3: the fused acceptance kernel (vxc_accept) and the row
sampler (vxc_sample_rows) against the CPU oracle, bit-exact: same accepted
lengths, same correction/bonus tokens, same sampled tokens.

Inputs follow benchmark configuration 3: 64 sequences, k = 5, V = 32000, target
logits ~ N(0, 2^2) (k+1 rows, the last one for the bonus token), draft
logits = target + N(0, 0.5^2), temperature 0.8, draft tokens drawn from q
with the same Philox stream (purpose DRAFT)."""
import ctypes

import numpy as np
import pytest

from _paths import oracle

pytestmark = pytest.mark.gpu
f32p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
DRAFT, ACCEPT, RESAMPLE = 1, 2, 3


def config3(seed=0, S=64, k=5, V=32000, T=0.8):
    O = oracle()
    rng = np.random.default_rng(seed)
    P = (rng.standard_normal((S, k + 1, V)) * 2.0).astype(np.float32)
    Q = (P[:, :k] + rng.standard_normal((S, k, V)) * 0.5).astype(np.float32)
    pos0 = (100 + np.arange(S)).astype(np.int32)
    ids = np.arange(S, dtype=np.int32)
    d = np.zeros((S, k), np.int32)
    for s in range(S):
        for i in range(k):
            d[s, i] = O.vxo_sample(f32p(Q[s, i]), V, T, O.vxo_philox_u32(77, int(pos0[s]) + i, int(ids[s]), DRAFT))
    return P, Q, d, pos0, ids


def run_gpu_accept(torch, P, Q, d, pos0, ids, T, seed):
    import vxb200
    L = vxb200.lib()
    S, k1, V = P.shape
    k = k1 - 1
    Pd, Qd = torch.from_numpy(P).cuda(), torch.from_numpy(Q).cuda()
    dd, pd_, idd = (torch.from_numpy(a).cuda() for a in (d, pos0, ids))
    na = torch.zeros(S, dtype=torch.int32, device="cuda")
    nx = torch.zeros(S, dtype=torch.int32, device="cuda")
    wsb = L.vxc_accept_workspace_bytes(S, k)
    ws = torch.zeros(wsb // 4 + 1, dtype=torch.int32, device="cuda")
    for _ in range(2):   # a repeated launch gives the same result (no state kept between launches)
        vxb200.check(L.vxc_accept(Pd.data_ptr(), k1 * V, V, Qd.data_ptr(), k * V, V, dd.data_ptr(), S, k, V, T, seed,
                                  idd.data_ptr(), pd_.data_ptr(), na.data_ptr(), nx.data_ptr(), ws.data_ptr(), wsb, None),
                     "vxc_accept")
    torch.cuda.synchronize()
    return na.cpu().numpy(), nx.cpu().numpy()


@pytest.mark.parametrize("T", [0.8, 0.0])
def test_accept_bit_exact(cuda, T):
    O = oracle()
    P, Q, d, pos0, ids = config3(seed=1, T=T if T > 0 else 0.8)
    S, k1, V = P.shape
    k = k1 - 1
    na, nx = run_gpu_accept(cuda, P, Q, d, pos0, ids, T, 77)
    for s in range(S):
        nxt = ctypes.c_int()
        a = O.vxo_accept(f32p(P[s]), f32p(Q[s]), f32p(d[s]), k, V, T, 77, int(ids[s]), int(pos0[s]), ctypes.byref(nxt))
        assert (a, nxt.value) == (na[s], nx[s]), s
    if T > 0:
        assert 0 < na.mean() < k   # config 3 draft is close to the target: partial acceptance


def test_accept_edge_cases(cuda):
    """q == p (must accept all, then bonus), and a draft whose tokens the
    target rules out (rejects at once)."""
    O = oracle()
    S, k, V = 4, 3, 777
    rng = np.random.default_rng(2)
    P = (rng.standard_normal((S, k + 1, V)) * 3).astype(np.float32)
    Q = P[:, :k].copy()
    Q[2:] = -P[2:, :k]            # sequences 2,3: draft prefers what the target dislikes
    pos0 = np.array([5, 6, 7, 8], np.int32)
    ids = np.arange(S, dtype=np.int32)
    d = np.zeros((S, k), np.int32)
    for s in range(S):
        for i in range(k):
            d[s, i] = O.vxo_sample(f32p(Q[s, i]), V, 1.0, O.vxo_philox_u32(5, int(pos0[s]) + i, s, DRAFT))
    na, nx = run_gpu_accept(cuda, P, Q, d, pos0, ids, 1.0, 5)
    assert na[0] == k and na[1] == k
    for s in range(S):
        nxt = ctypes.c_int()
        a = O.vxo_accept(f32p(P[s]), f32p(Q[s]), f32p(d[s]), k, V, 1.0, 5, s, int(pos0[s]), ctypes.byref(nxt))
        assert (a, nxt.value) == (na[s], nx[s])


def test_accept_large_vocab(cuda):
    """Configuration 5's vocabulary (128256): 2048-element draw sub-blocks."""
    P, Q, d, pos0, ids = config3(seed=4, S=6, k=6, V=128256)
    S, k1, V = P.shape
    k = k1 - 1
    na, nx = run_gpu_accept(cuda, P, Q, d, pos0, ids, 0.8, 77)
    O = oracle()
    for s in range(S):
        nxt = ctypes.c_int()
        a = O.vxo_accept(f32p(P[s]), f32p(Q[s]), f32p(d[s]), k, V, 0.8, 77, int(ids[s]), int(pos0[s]), ctypes.byref(nxt))
        assert (a, nxt.value) == (na[s], nx[s]), s


def test_accept_rejects_long_drafts(cuda):
    import vxb200
    L = vxb200.lib()
    torch = cuda
    buf = torch.zeros(4 * 65 * 100, device="cuda")
    ib = torch.zeros(130, dtype=torch.int32, device="cuda")
    rc = L.vxc_accept(buf.data_ptr(), 65 * 100, 100, buf.data_ptr(), 65 * 100, 100, ib.data_ptr(), 1, 65, 100, 0.8,
                      1, ib.data_ptr(), ib.data_ptr(), ib.data_ptr(), ib.data_ptr(), None, 0, None)
    assert rc != 0 and b"at most 64" in L.vxc_error_string()


@pytest.mark.parametrize("T,V", [(0.8, 32000), (1.5, 32000), (0.0, 32000), (0.8, 1001), (0.0, 1001), (0.7, 100)])
def test_sample_rows_bit_exact(cuda, T, V):
    """V = 1001: rows not 16-byte aligned (element loads); V = 100: one
    CTA of the cluster holds the whole row, the other seven nothing."""
    import vxb200
    torch = cuda
    O = oracle()
    rng = np.random.default_rng(3)
    R = 96
    l = (rng.standard_normal((R, V)) * 3).astype(np.float32)
    l[5, 10] = l[5, 20] = l[5].max() + 1       # tie: first maximum wins
    pos = rng.integers(0, 5000, R).astype(np.int32)
    seq = rng.integers(0, 64, R).astype(np.int32)
    ld, pd_, sd = torch.from_numpy(l).cuda(), torch.from_numpy(pos).cuda(), torch.from_numpy(seq).cuda()
    out = torch.zeros(R, dtype=torch.int32, device="cuda")
    vxb200.check(vxb200.lib().vxc_sample_rows(ld.data_ptr(), R, V, T, 99, pd_.data_ptr(), sd.data_ptr(), DRAFT,
                                              out.data_ptr(), None), "vxc_sample_rows")
    got = out.cpu().numpy()
    want = [O.vxo_sample(f32p(l[r]), V, T, O.vxo_philox_u32(99, int(pos[r]), int(seq[r]), DRAFT)) for r in range(R)]
    assert np.array_equal(got, np.array(want))
    if T == 0.0:
        assert got[5] == 10
