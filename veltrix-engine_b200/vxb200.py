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
    "vxc_qgemv_noalloc": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, _vp]),
    "vxc_kquant_dequant": (ctypes.c_int, [_vp, _vp, _vp]),
    "vxc_device_current": (ctypes.c_int, []),
    "vxc_launch_count": (ctypes.c_longlong, []),
    "vxc_profile_enable": (None, [ctypes.c_int]),
    "vxc_profile_read": (ctypes.c_int, [_vp, ctypes.c_int]),
    "vxc_net_create": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, ctypes.POINTER(_vp)]),
    "vxc_net_create_tp": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(_vp)]),
    "vxc_net_create_synth": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_uint64, _vp, ctypes.POINTER(_vp)]),
    "vx_model_create_synth": (ctypes.c_int, [_vp, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, _vp,
                                             ctypes.POINTER(_vp)]),
    "vxc_tp_unique_id": (ctypes.c_int, [_vp]),
    "vxc_tp_shard_ranges": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    "vxc_tp_create": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
    "vxc_tp_destroy": (None, [_vp]),
    "vxc_net_destroy": (None, [_vp]),
    "vxc_net_config_get": (ctypes.c_int, [_vp, _vp]),
    "vxc_net_weight_bytes": (ctypes.c_size_t, [_vp]),
    "vxc_seqs_create": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
    "vxc_seqs_destroy": (None, [_vp]),
    "vxc_forward": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp]),
    "vxc_forward_host": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp]),
    # model.h / veltrix.h
    "vx_model_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "vx_model_create_tp": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _vp, ctypes.POINTER(_vp)]),
    "vx_model_destroy": (None, [_vp]),
    "vx_model_forward": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    "vx_model_generate_greedy": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int]),
    "vxc_greedy_generate": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int,
                                           ctypes.c_int, _c_int_p, _c_int_p]),
    "vx_model_kv_truncate": (None, [_vp, ctypes.c_int]),
    "vx_set_compute_level": (None, [ctypes.c_int]),
    "vx_enable_metalearn": (None, [ctypes.c_bool]),
    "vx_set_n_threads": (None, [ctypes.c_int]),
    "vx_set_forward_timing_enabled": (None, [ctypes.c_int]),
    "vx_print_forward_timing": (None, []),
    "vxc_sample_rows": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_uint64, _vp, _vp,
                                        ctypes.c_uint, _vp, _vp]),
    "vxc_accept_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    "vxc_accept": (ctypes.c_int, [_vp, ctypes.c_longlong, ctypes.c_longlong, _vp, ctypes.c_longlong,
                                  ctypes.c_longlong, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                  ctypes.c_uint64, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "vxc_spec_create": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
    "vxc_spec_destroy": (None, [_vp]),
    "vxc_spec_probe": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    "vxc_spec_generate": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_uint64, _vp, _vp, _vp]),
    # speculative.h
    "vx_speculative_create": (_vp, [_vp, _vp, ctypes.c_int]),
    "vx_speculative_destroy": (None, [_vp]),
    "vx_speculative_set_temp": (None, [_vp, ctypes.c_float, ctypes.c_float]),
    "vx_speculative_generate": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, ctypes.c_int]),
    "vx_speculative_generate_stream": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int]),
    "vx_speculative_set_seed": (None, [_vp, ctypes.c_uint64]),
    "vx_speculative_set_seq_id_base": (None, [_vp, ctypes.c_int]),
    "vx_speculative_generate_batch": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp]),
    "vx_speculative_get_stats": (ctypes.c_int, [_vp, _vp]),
    "vx_speculative_probe": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    # veltrix_synth.h
    "vx_synth_write_gguf": (ctypes.c_int, [ctypes.c_char_p, _vp, ctypes.c_uint64]),
}


class SynthConfig(ctypes.Structure):
    _fields_ = [("n_embd", ctypes.c_int), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("n_ff", ctypes.c_int), ("n_vocab", ctypes.c_int),
                ("rope_theta", ctypes.c_float), ("wtype", ctypes.c_int)]


class NetConfig(ctypes.Structure):
    """vxc_net_config (include/veltrix_cuda.h)."""
    _fields_ = [("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
                ("n_embd", ctypes.c_int), ("n_head_dim", ctypes.c_int), ("n_ff", ctypes.c_int),
                ("n_vocab", ctypes.c_int), ("max_pos", ctypes.c_int), ("rope_theta", ctypes.c_float)]


def tp_shard_ranges(n_embd, n_heads, n_kv_heads, n_ff, n_vocab, rank, world):
    """[(first row, rows, first col, cols)] of Wq, Wk, Wv, Wo, W_gate, W_up, W_down, LM head
    that rank `rank` of `world` keeps (the split vxc_net_create_tp applies)."""
    c = NetConfig(1, n_heads, n_kv_heads, n_embd, n_embd // n_heads, n_ff, n_vocab, 4096, 10000.0)
    out = (ctypes.c_int * 32)()
    check(lib().vxc_tp_shard_ranges(ctypes.byref(c), rank, world, out), "vxc_tp_shard_ranges")
    return [tuple(out[4 * i:4 * i + 4]) for i in range(8)]


class ModelConfig(ctypes.Structure):
    """vx_model_config (include/veltrix.h)."""
    _fields_ = [("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
                ("n_embd", ctypes.c_int), ("n_head_dim", ctypes.c_int), ("n_ff", ctypes.c_int),
                ("n_vocab", ctypes.c_int), ("n_ctx", ctypes.c_int), ("rope_theta", ctypes.c_float),
                ("rope_freq_base", ctypes.c_float), ("n_threads", ctypes.c_int), ("arch", ctypes.c_int),
                ("mlp_type", ctypes.c_int), ("norm_type", ctypes.c_int), ("rope_partial_dims", ctypes.c_int),
                ("has_q_bias", ctypes.c_bool), ("has_k_bias", ctypes.c_bool), ("has_v_bias", ctypes.c_bool),
                ("has_post_attn_norm", ctypes.c_bool), ("has_post_ffn_norm", ctypes.c_bool),
                ("has_ffn_bias", ctypes.c_bool)]


class ModelHead(ctypes.Structure):
    """Leading fields of struct vx_model up to cache_len (include/veltrix.h)."""
    _fields_ = [("config", ModelConfig), ("tensors", ctypes.c_void_p), ("n_tensors", ctypes.c_int)] + \
               [("p%d" % i, ctypes.c_void_p) for i in range(27)] + [("cache_len", ctypes.c_int)]


def write_synth(path, n_embd, n_layers, n_heads, n_kv_heads, n_ff, n_vocab, wtype, seed, rope_theta=10000.0):
    c = SynthConfig(n_embd, n_layers, n_heads, n_kv_heads, n_ff, n_vocab, rope_theta, wtype)
    check(lib().vx_synth_write_gguf(path.encode(), ctypes.byref(c), seed), "vx_synth_write_gguf")


class SpecStats(ctypes.Structure):
    _fields_ = [("rounds", ctypes.c_longlong), ("drafted", ctypes.c_longlong), ("accepted", ctypes.c_longlong),
                ("emitted", ctypes.c_longlong), ("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double)]


class Speculative:
    """vx_speculative_state (include/speculative.h) over two Model handles."""

    def __init__(self, draft, target, k, temp=0.0, top_p=1.0, seed=1, seq_id_base=0):
        self.h = lib().vx_speculative_create(draft.h, target.h, k)
        if not self.h:
            raise VxError("vx_speculative_create failed")
        lib().vx_speculative_set_temp(self.h, temp, top_p)
        lib().vx_speculative_set_seed(self.h, seed)
        lib().vx_speculative_set_seq_id_base(self.h, seq_id_base)

    def generate(self, prompt, max_tokens):
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_tokens, np.int32)
        n = lib().vx_speculative_generate(self.h, p.ctypes.data, p.size, out.ctypes.data, max_tokens)
        return out[:n]

    def generate_batch(self, prompts, max_tokens):
        import numpy as np
        ps = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        outs = [np.zeros(max_tokens, np.int32) for _ in ps]
        pa = (_vp * len(ps))(*[p.ctypes.data for p in ps])
        oa = (_vp * len(ps))(*[o.ctypes.data for o in outs])
        lens = np.array([p.size for p in ps], np.int32)
        cnt = np.zeros(len(ps), np.int32)
        lib().vx_speculative_generate_batch(self.h, pa, lens.ctypes.data, len(ps), oa, max_tokens, cnt.ctypes.data)
        return [o[:c] for o, c in zip(outs, cnt)]

    def stats(self):
        s = SpecStats()
        check(lib().vx_speculative_get_stats(self.h, ctypes.byref(s)), "vx_speculative_get_stats")
        return s

    def probe(self, which, reps=5):
        """(ms, kv_bytes) of one piece of the last round: 0 verify, 1 draft step, 2 acceptance."""
        ms, kvb = ctypes.c_double(0), ctypes.c_double(0)
        check(lib().vx_speculative_probe(self.h, which, reps, ctypes.byref(ms), ctypes.byref(kvb)),
              "vx_speculative_probe")
        return ms.value, kvb.value

    def close(self):
        if self.h:
            lib().vx_speculative_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id():
    """NCCL unique id (128 bytes) for vx_model_create_tp, made on rank 0."""
    buf = ctypes.create_string_buffer(128)
    check(lib().vxc_tp_unique_id(buf), "vxc_tp_unique_id")
    return buf.raw


class Model:
    """vx_model handle of the B200 back end (include/model.h)."""

    def __init__(self, path, tp=None, synth=None):
        """tp = (rank, world, nccl_id bytes) loads this rank's tensor-parallel shard.
        synth = (n_embd, n_layers, n_heads, n_kv_heads, n_ff, n_vocab, wtype, seed, rope_theta)
        generates the weights on the device instead of reading `path` (None)."""
        h = _vp()
        if synth is not None:
            e, L, hh, kv, ff, v, wt, seed, th = synth
            c = SynthConfig(e, L, hh, kv, ff, v, th, wt)
            rank, world, uid = tp if tp is not None else (0, 1, None)
            idbuf = ctypes.create_string_buffer(bytes(uid), 128) if uid is not None else None
            rc = lib().vx_model_create_synth(ctypes.byref(c), seed, rank, world, idbuf, ctypes.byref(h))
            path = "<synthetic>"
        elif tp is None:
            rc = lib().vx_model_create(path.encode(), ctypes.byref(h))
        else:
            rank, world, uid = tp
            idbuf = ctypes.create_string_buffer(bytes(uid), 128)
            rc = lib().vx_model_create_tp(path.encode(), rank, world, idbuf, ctypes.byref(h))
        if rc != 0:
            raise VxError(f"vx_model_create({path}) = {rc}: {lib().vxc_error_string()}")
        self.h = h
        self.head = ctypes.cast(h, ctypes.POINTER(ModelHead)).contents

    @property
    def n_vocab(self):
        return self.head.config.n_vocab

    @property
    def cache_len(self):
        return self.head.cache_len

    @cache_len.setter
    def cache_len(self, v):
        self.head.cache_len = v

    def forward(self, tokens):
        import numpy as np
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.n_vocab, np.float32)
        rc = lib().vx_model_forward(self.h, toks.ctypes.data, toks.size, out.ctypes.data)
        if rc != 0:
            raise VxError(f"vx_model_forward = {rc}: {lib().vxc_error_string()}")
        return out

    def generate_greedy(self, prompt, max_tokens, eos_id=-1):
        """vx_model_generate_greedy: the emitted tokens (int32 array)."""
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_tokens, np.int32)
        n = lib().vx_model_generate_greedy(self.h, p.ctypes.data, p.size, out.ctypes.data, max_tokens, eos_id)
        if n < 0:
            raise VxError(f"vx_model_generate_greedy = {n}: {lib().vxc_error_string()}")
        return out[:n]

    def close(self):
        if self.h:
            lib().vx_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

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
