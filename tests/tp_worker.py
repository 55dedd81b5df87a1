"""One rank of the tensor-parallel GPU test (tests/test_tp_gpu.py), run as
its own process on GPU `rank`:

    python tests/tp_worker.py RANK WORLD OUT_DIR

It loads this rank's shard of the 70B-width 2-layer fixture and of the tiny
target (the draft stays whole on every GPU), runs the same calls as every
other rank and saves logits and token streams to OUT_DIR/rank<RANK>.npz.
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "veltrix-engine_b200"))

import fixtures  # noqa: E402
import vxb200  # noqa: E402

PROMPT70 = np.array([1, 17, 4242, 99, 128000, 31337], np.int32)
NEXT70 = np.array([777], np.int32)
# 70 ids: one 64-row chunk on the tensor-core GEMM, then 6 rows on the GEMV
PROMPT70_LONG = np.random.default_rng(70).integers(0, 128256, 70).astype(np.int32)
PROMPT_TINY = np.random.default_rng(2024).integers(0, 4096, 32).astype(np.int32)


def unique_ids(rank, out, n=2, wait_s=120.0):
    """NCCL ids made by rank 0 (the same libnccl as every rank) and handed
    to the others through a file."""
    path = os.path.join(out, "nccl_ids")
    if rank == 0:
        ids = b"".join(vxb200.tp_unique_id() for _ in range(n))
        with open(path + ".tmp", "wb") as f:
            f.write(ids)
        os.replace(path + ".tmp", path)
    t0 = time.time()
    while not os.path.exists(path):
        if time.time() - t0 > wait_s:
            raise RuntimeError("rank 0 wrote no NCCL ids")
        time.sleep(0.05)
    ids = open(path, "rb").read()
    return [ids[128 * i:128 * (i + 1)] for i in range(n)]


def main():
    rank, world, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    vxb200.check(vxb200.lib().vxc_device_init(rank), "vxc_device_init")
    uid70, uidt, uids = unique_ids(rank, out, n=3)
    res = {}
    m = vxb200.Model(fixtures.path("l70b_2layer"), tp=(rank, world, uid70))
    res["l70_prefill"] = m.forward(PROMPT70)
    res["l70_decode"] = m.forward(NEXT70)
    m.cache_len = 0
    res["l70_long_prefill"] = m.forward(PROMPT70_LONG)
    m.close()
    # the same shard generated on the device instead of read from the file
    m = vxb200.Model(None, tp=(rank, world, uids), synth=fixtures.CONFIGS["l70b_2layer"])
    res["l70_synth_prefill"] = m.forward(PROMPT70)
    m.close()
    t = vxb200.Model(fixtures.path("tiny_target"), tp=(rank, world, uidt))
    d = vxb200.Model(fixtures.path("tiny_draft"))
    sp = vxb200.Speculative(d, t, 4, temp=0.0)
    res["tiny_greedy"] = np.asarray(sp.generate(PROMPT_TINY, 64), np.int32)
    sp.close()
    sp = vxb200.Speculative(d, t, 4, temp=0.8, seed=1234)
    res["tiny_sampled"] = np.asarray(sp.generate(PROMPT_TINY, 96), np.int32)
    sp.close()
    t.close()
    d.close()
    np.savez(os.path.join(out, f"rank{rank}.npz"), **res)


if __name__ == "__main__":
    main()
