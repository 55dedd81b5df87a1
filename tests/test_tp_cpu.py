"""The tensor-parallel split on CPU.  Two gloo ranks take the slices that
vxc_tp_shard_ranges gives them (the function vxc_net_create_tp uses to cut
the weights).  Each runs one llama block and the LM head in float64 on its
slices, with the device forward's exchanges: an all-reduce after the output
projection and after the down projection, and an all-gather of the
vocabulary-split logits.  The result must be the unsplit forward (to
float64 rounding), and the slices must cover every weight exactly once."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
E, H, KH, F, V, T = 256, 8, 4, 768, 512, 5
HD = E // H


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    rng = np.random.default_rng(77)
    w = lambda r, c: rng.standard_normal((r, c)) * 0.05
    return dict(x=rng.standard_normal((T, E)), wq=w(E, E), wk=w(KH * HD, E), wv=w(KH * HD, E), wo=w(E, E),
                wg=w(F, E), wu=w(F, E), wd=w(E, F), wout=w(V, E))


def _rms(x):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-5)


def _attention(q, k, v, n_heads, n_kv):
    """Causal attention over T positions; query head h reads kv head h // (n_heads / n_kv)."""
    G = n_heads // n_kv
    out = np.zeros((T, n_heads * HD))
    for h in range(n_heads):
        kh = h // G
        qh, kk, vv = q[:, h * HD:(h + 1) * HD], k[:, kh * HD:(kh + 1) * HD], v[:, kh * HD:(kh + 1) * HD]
        s = qh @ kk.T / np.sqrt(HD)
        s = np.where(np.tril(np.ones((T, T))) > 0, s, -np.inf)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h * HD:(h + 1) * HD] = (p / p.sum(axis=1, keepdims=True)) @ vv
    return out


def _forward(W, sl=None, allreduce=None, allgather=None):
    """One block + LM head; sl = this rank's slices (None: the whole model)."""
    take = (lambda m, i: m) if sl is None else \
        (lambda m, i: m[sl[i][0]:sl[i][0] + sl[i][1], sl[i][2]:sl[i][2] + sl[i][3]])
    x = W["x"].copy()
    h = _rms(x)
    q, k, v = h @ take(W["wq"], 0).T, h @ take(W["wk"], 1).T, h @ take(W["wv"], 2).T
    a = _attention(q, k, v, q.shape[1] // HD, k.shape[1] // HD)
    o = a @ take(W["wo"], 3).T
    x = x + (allreduce(o) if allreduce else o)
    h = _rms(x)
    g, u = h @ take(W["wg"], 4).T, h @ take(W["wu"], 5).T
    d = (g / (1 + np.exp(-g)) * u) @ take(W["wd"], 6).T
    x = x + (allreduce(d) if allreduce else d)
    lg = _rms(x) @ take(W["wout"], 7).T
    return allgather(lg) if allgather else lg


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, os.path.join(ROOT, "veltrix-engine_b200"))
    import datetime
    import torch
    import torch.distributed as dist
    import vxb200
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    sl = vxb200.tp_shard_ranges(E, H, KH, F, V, rank, world)

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        dist.all_reduce(t)
        return t.numpy()

    def allgather(a):
        parts = [torch.empty(a.shape, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(a)))
        return np.concatenate([p.numpy() for p in parts], axis=1)

    lg = _forward(_weights(), sl, allreduce, allgather)
    q.put((rank, sl, lg))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_split_equals_unsplit_forward():
    world = 2
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((qu.get(timeout=120) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _forward(_weights())
    for rank, sl, lg in res:
        assert np.allclose(lg, full, rtol=1e-12, atol=1e-12), rank
    # every weight of every matrix belongs to exactly one rank
    shapes = [(E, E), (KH * HD, E), (KH * HD, E), (E, E), (F, E), (F, E), (E, F), (V, E)]
    for i, (r, c) in enumerate(shapes):
        cover = np.zeros((r, c), np.int32)
        for _, sl, _ in res:
            r0, nr, c0, nc = sl[i]
            cover[r0:r0 + nr, c0:c0 + nc] += 1
        assert (cover == 1).all(), i


def test_uneven_split_is_rejected():
    sys.path.insert(0, os.path.join(ROOT, "veltrix-engine_b200"))
    import vxb200
    with pytest.raises(vxb200.VxError):
        vxb200.tp_shard_ranges(E, H, KH, F, V, 0, 3)      # 8 heads over 3 GPUs
