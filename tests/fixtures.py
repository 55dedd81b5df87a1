"""Synthetic checkpoints of the benchmark configurations, written by the
library's own GGUF writer (vx_synth_write_gguf) into a cache directory."""
import os
import tempfile

import vxb200

CACHE = os.environ.get("VX_FIXTURE_DIR", os.path.join(tempfile.gettempdir(), "vx_fixtures"))

# name: (n_embd, n_layers, n_heads, n_kv_heads, n_ff, n_vocab, wtype, seed, rope_theta)
CONFIGS = {
    # config 1: tiny Llama target / draft, all Q8_0
    "tiny_target": (256, 4, 8, 8, 768, 4096, 8, 1, 10000.0),
    "tiny_draft": (128, 2, 4, 4, 384, 4096, 8, 2, 10000.0),
    # K-quant models at the tiny target's shape (every 2-D tensor of one type; widths % 256 == 0)
    "tiny_q2k": (256, 2, 8, 8, 768, 4096, 10, 40, 10000.0),
    "tiny_q3k": (256, 2, 8, 8, 768, 4096, 11, 41, 10000.0),
    "tiny_q4k": (256, 2, 8, 8, 768, 4096, 12, 42, 10000.0),
    "tiny_q5k": (256, 2, 8, 8, 768, 4096, 13, 43, 10000.0),
    "tiny_q6k": (256, 2, 8, 8, 768, 4096, 14, 44, 10000.0),
    "tiny_q8k": (256, 2, 8, 8, 768, 4096, 15, 45, 10000.0),
    # Q4_K with Q6_K value, down and LM-head tensors (VX_SYNTH_KQ_MIX)
    "tiny_kqmix": (256, 2, 8, 8, 768, 4096, 100, 46, 10000.0),
    # config 4 shapes, fewer layers (parity at 7B width)
    "l7b_2layer": (4096, 2, 32, 32, 11008, 32000, 2, 3, 10000.0),
    "d11b_2layer": (2048, 2, 32, 4, 5632, 32000, 8, 4, 10000.0),
    # config 5 target width (Llama-3-70B: 64/8 heads of 128, FFN 28672, vocab 128256), 2 layers
    "l70b_2layer": (8192, 2, 64, 8, 28672, 128256, 2, 5, 500000.0),
    # config 4 full models
    "llama7b_q4": (4096, 32, 32, 32, 11008, 32000, 2, 11, 10000.0),
    "draft11b_q8": (2048, 22, 32, 4, 5632, 32000, 8, 12, 10000.0),
}


def path(name):
    os.makedirs(CACHE, exist_ok=True)
    p = os.path.join(CACHE, name + ".gguf")
    if not os.path.exists(p):
        e, L, h, kv, ff, v, wt, seed, th = CONFIGS[name]
        tmp = p + ".tmp%d" % os.getpid()
        vxb200.write_synth(tmp, e, L, h, kv, ff, v, wt, seed, th)
        os.replace(tmp, p)
    return p
