"""Python host-side binding of libiq.so (the C ABI in include/iq.h) -- TEST AND
BENCH TOOLING, not the product: the product is the C ABI (include/iq.h,
libiq.so), which C hosts such as llama_int.c call directly. This module is how
the tests and bench.py reach that ABI from Python; torch appears here only to
hand over device memory and streams.

This is a thin ctypes mirror of the reference's operator surface: ``matmul_vec``
(llama_int.c:1014) with its argument order ``(out, weight, in, M, N)``, where M
is the number of output rows and N the input length. Host arrays are numpy
int64; device arrays are anything exposing ``data_ptr()`` (torch tensors are
used only as device-memory plumbing). Every call raises ``IQError`` on a
non-zero status; there is no CPU fallback: if libiq.so is missing or no B200
is present, calls fail loudly.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("IQ_LIB") or os.path.join(HERE, "libiq.so")  # IQ_LIB: another build

IQ_FN = dict(mul=0, div=1, sqrt=2, sqrt_fast=3, inv_sqrt=4, exp=5, log=6, cos=7, sin=8,
             sigmoid=9, silu=10, safe_exp=11, exp_dyadic=12)

# every symbol include/iq.h declares, with (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
SIGNATURES = {
    "iq_status_str": (ctypes.c_char_p, [_I]),
    "iq_last_cuda_error": (_I, []),
    "iq_version": (_I, []),
    "iq_set_device": (_I, [_I]),
    "iq_matmul_vec": (_I, [_P, _P, _P, _I, _I]),
    "iq_weight_register": (_I, [_P, _I, _I]),
    "iq_weight_unregister": (_I, [_P]),
    "iq_weight_cache_clear": (_I, []),
    "iq_weight_check_mode": (_I, [_I]),
    "iq_weight_cache_limit": (_I, [_I64]),
    "iq_weight_cache_stats": (_I, [_P, _P]),
    "iq_matvec_dev": (_I, [_P, _P, _P, _I, _I, _P]),
    "iq_gemm_dev": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "iq_pack_weights_dev": (_I, [_P, _I, _I, _P, _P]),
    "iq_pack_weights_fmt_dev": (_I, [_P, _I, _I, _I, _P, _P]),
    "iq_packed_free": (_I, [_P]),
    "iq_packed_info": (_I, [_P, _P, _P, _P]),
    "iq_matvec_packed_dev": (_I, [_P, _P, _P, _P]),
    "iq_matvec_packed_noalloc_dev": (_I, [_P, _P, _P, _P]),
    "iq_packed_bytes": (_I, [_P, _P]),
    "iq_packed_format": (_I, [_P, _P]),
    "iq_pack_weights_tc_dev": (_I, [_P, _I, _I, _P, _P]),
    "iq_packed_tc_free": (_I, [_P]),
    "iq_packed_tc_info": (_I, [_P, _P, _P, _P]),
    "iq_gemm_tc_dev": (_I, [_P, _P, _P, _I, _P]),
    "iq_device_status": (_I, []),
    "iq_wait_selftest": (_I, [_I64]),
    "iq_bench_i8_peak": (_I, [_I, _P, _P]),
    "iq_fp_dev": (_I, [_I, _P, _P, _P, _I64, _P]),
    "iq_rmsnorm_dev": (_I, [_P, _P, _P, _I, _I, _P]),
    "iq_softmax_dev": (_I, [_P, _I, _I, _P]),
    "iq_model_create": (_I, [_P, _I, _I, _P]),
    "iq_nccl_unique_id": (_I, [_P]),
    "iq_tp_shard_info": (_I, [_P, _I, _I, _P]),
    "iq_model_create_tp": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "iq_model_destroy": (_I, [_P]),
    "iq_model_load_globals": (_I, [_P, _P, _P, _P]),
    "iq_model_load_layer": (_I, [_P, _I, _P]),
    "iq_model_synth": (_I, [_P, _I, _I]),
    "iq_model_config": (_I, [_P, _P]),
    "iq_mgw_read_config": (_I, [ctypes.c_char_p, _P, _P]),
    "iq_model_load_mgw": (_I, [_P, ctypes.c_char_p]),
    "iq_model_reset": (_I, [_P]),
    "iq_forward": (_I, [_P, _I, _I, _P, _P]),
    "iq_generate": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "iq_generate_batch": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "iq_generate_sampled": (_I, [_P, _P, _I, _I, _I64, _I, _I64, ctypes.c_uint64, _P, _P, _P]),
    "iq_sample_dev": (_I, [_P, _I, _I, _I64, _I, _I64, _P, _P]),
    "iq_rng_seed": (_I, [ctypes.c_uint64, _P]),
    "iq_decode_steps_timed": (_I, [_P, _I, _I, _P]),
    "iq_model_set_attention": (_I, [_P, _I]),
    "iq_model_weight_bytes": (_I, [_P, _P, _P]),
    "iq_model_set_decode": (_I, [_P, _I]),
    "iq_model_set_timeout": (_I, [_P, _I64]),
    "iq_model_set_peer_check": (_I, [_P, _P, _P]),
    "iq_model_set_kv_packed": (_I, [_P, _I, _I]),
    "iq_selftest_watchdog": (_I, [_I, _P, _P]),
    "iq_model_decode_info": (_I, [_P, _P, _P]),
    "iq_bench_grid_sync": (_I, [_I, _I, _I, _P]),
    "iq_model_decode_stamps": (_I, [_P, _P, _I]),
    "iq_tensor_seed": (ctypes.c_uint64, [_I, ctypes.c_char_p]),
    "iq_synth_weights": (_I, [ctypes.c_uint64, _P, _I64]),
    "iq_synth_acts": (_I, [ctypes.c_uint64, _P, _I64]),
    "iq_synth_tokens": (_I, [ctypes.c_uint64, _P, _I, _I]),
    "iq_bf16_to_q1648": (_I64, [ctypes.c_uint16]),
    "iq_q1648_to_bf16": (ctypes.c_uint16, [_I64]),
}


class IQError(RuntimeError):
    def __init__(self, fn, status, lib):
        self.status = status
        msg = lib.iq_status_str(status).decode()
        cuda = lib.iq_last_cuda_error()
        super().__init__(f"{fn} failed: {msg} (status {status}, last cudaError {cuda})")


_lib = None


def lib():
    """Load libiq.so (built in-tree by the package Makefile)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libiq.so not built at {LIB_PATH}; run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _call(name, *args):
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != 0:
        raise IQError(name, rc, L)
    return rc


def _hp(a):
    assert isinstance(a, np.ndarray) and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


def _dp(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


_CUDA_STREAM_LEGACY = 0x1


def _sp(stream):
    """Stream argument: an explicit stream, else torch's current stream when torch
    has initialised CUDA (so device calls order with the tensors' producers),
    else NULL = the library's own stream."""
    if stream is None:
        import sys
        t = sys.modules.get("torch")
        if t is not None and t.cuda.is_initialized():
            h = t.cuda.current_stream().cuda_stream
            # torch's default stream has handle 0, which the library would read as
            # "its own stream": name the legacy default stream (cudaStreamLegacy) instead
            return ctypes.c_void_p(h if h else _CUDA_STREAM_LEGACY)
        return None
    return ctypes.c_void_p(getattr(stream, "cuda_stream", stream))


# ---------------------------------------------------------------- host API

def matmul_vec(out, weight, inp, M, N):
    """Drop-in for matmul_vec(out, weight, in, M, N) on host int64 arrays."""
    assert out.dtype == weight.dtype == inp.dtype == np.int64
    assert out.size >= M and inp.size >= N and weight.size >= M * N
    _call("iq_matmul_vec", _hp(out), _hp(weight), _hp(inp), M, N)


def weight_register(weight, M, N):
    _call("iq_weight_register", _hp(weight), M, N)


def weight_unregister(weight):
    _call("iq_weight_unregister", _hp(weight))


def weight_cache_clear():
    _call("iq_weight_cache_clear")


WCHECK = dict(none=0, sampled=1, full=2)


def weight_check_mode(mode):
    _call("iq_weight_check_mode", WCHECK[mode] if isinstance(mode, str) else mode)


def weight_cache_limit(nbytes):
    _call("iq_weight_cache_limit", nbytes)


def weight_cache_stats():
    """(entries, device bytes) of the drop-in's weight cache."""
    e, b = ctypes.c_int(), ctypes.c_int64()
    _call("iq_weight_cache_stats", ctypes.byref(e), ctypes.byref(b))
    return e.value, b.value


def nccl_unique_id():
    """128-byte NCCL id for iq_model_create_tp (made on one rank, shared with all)."""
    buf = ctypes.create_string_buffer(128)
    _call("iq_nccl_unique_id", buf)
    return buf.raw


def tp_shard_info(cfg, tp_size, tp_rank):
    """Row ownership of a tensor-parallel rank (see iq_tp_shard_info)."""
    c = cfg if isinstance(cfg, Config) else Config.from_dict(cfg)
    info = (ctypes.c_int * 8)()
    _call("iq_tp_shard_info", ctypes.byref(c), tp_size, tp_rank, info)
    keys = ("q_lo", "nh", "kv_lo", "nkv", "d_lo", "d_n", "it_lo", "it_n")
    return dict(zip(keys, list(info)))


def mgw_config(path):
    """(config dict, lm_head_tied) of an int-llm .mgw file."""
    c = Config()
    tied = ctypes.c_int(0)
    _call("iq_mgw_read_config", os.fsencode(path), ctypes.byref(c), ctypes.byref(tied))
    return dict(dim=c.hidden_dim, n_heads=c.num_heads, n_kv_heads=c.num_kv_heads, head_dim=c.head_dim,
                n_layers=c.num_layers, inter=c.intermediate_dim, vocab=c.vocab_size, max_seq=c.max_seq_len,
                rope_theta=c.rope_theta), bool(tied.value)


def set_device(d):
    _call("iq_set_device", d)


# -------------------------------------------------------------- device API

def matvec_dev(out, w, x, M, N, stream=None):
    _call("iq_matvec_dev", _dp(out), _dp(w), _dp(x), M, N, _sp(stream))


class Packed:
    """Byte-plane packed weights on the device (iq_pack_weights_dev)."""

    def __init__(self, d_w, M, N, stream=None, fmt=None):
        """fmt: None = the library's choice, 'planes' or 'bf16'."""
        self.h = ctypes.c_void_p()
        self.M, self.N = M, N
        f = {None: -1, "planes": 0, "bf16": 1}[fmt]
        _call("iq_pack_weights_fmt_dev", _dp(d_w), M, N, f, _sp(stream), ctypes.byref(self.h))

    def info(self):
        """(np, p0, residual_entries): stored planes p0 .. p0+np-1 and the sparse residual size."""
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _call("iq_packed_info", self.h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def fmt(self):
        """'planes' (byte-plane window) or 'bf16' (2 bytes per weight)."""
        f = ctypes.c_int()
        _call("iq_packed_format", self.h, ctypes.byref(f))
        return ("planes", "bf16")[f.value]

    def nbytes(self):
        """Bytes of the stored form one matvec launch reads (iq_packed_bytes)."""
        b = ctypes.c_int64()
        _call("iq_packed_bytes", self.h, ctypes.byref(b))
        return b.value

    def free(self):
        if self.h:
            _call("iq_packed_free", self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def matvec_packed_dev(out, packed, x, stream=None):
    _call("iq_matvec_packed_dev", _dp(out), packed.h, _dp(x), _sp(stream))


class PackedTC:
    """Weights packed for the tcgen05 GEMM (iq_pack_weights_tc_dev)."""

    def __init__(self, d_w, M, N, stream=None):
        self.h = ctypes.c_void_p()
        _call("iq_pack_weights_tc_dev", _dp(d_w), M, N, _sp(stream), ctypes.byref(self.h))

    def info(self):
        """(np, p0, residual_entries) of the GEMM form."""
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _call("iq_packed_tc_info", self.h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def free(self):
        if self.h:
            _call("iq_packed_tc_free", self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def gemm_tc_dev(out, packed, X, rows, stream=None):
    _call("iq_gemm_tc_dev", _dp(out), packed.h, _dp(X), rows, _sp(stream))


def sample_dev(d_logits, rows, V, temperature, top_k, top_p, rng):
    """sample_token per row on the device; rng: uint64 [rows][2], advanced in place."""
    out = np.zeros(rows, dtype=np.int32)
    assert rng.dtype == np.uint64 and rng.flags.c_contiguous
    _call("iq_sample_dev", _dp(d_logits), rows, V, temperature, top_k, top_p, _hp(rng), _hp(out))
    return out


def device_status():
    """IQ_OK, or the timeout status a kernel's bounded wait recorded (then cleared)."""
    return lib().iq_device_status()


def bench_i8_peak(iters=20000):
    """(int8 TOP/s, ms) of the tcgen05 kind::i8 peak kernel on the current device."""
    t, ms = ctypes.c_double(), ctypes.c_float()
    _call("iq_bench_i8_peak", iters, ctypes.byref(t), ctypes.byref(ms))
    return t.value, ms.value


def gemm_dev(out, w, X, rows, M, N, stream=None):
    _call("iq_gemm_dev", _dp(out), _dp(w), _dp(X), rows, M, N, _sp(stream))


def fp_dev(fn, x, y, out, n, stream=None):
    code = IQ_FN[fn] if isinstance(fn, str) else fn
    _call("iq_fp_dev", code, _dp(x), _dp(y), _dp(out), n, _sp(stream))


def rmsnorm_dev(out, x, w, rows, dim, stream=None):
    _call("iq_rmsnorm_dev", _dp(out), _dp(x), _dp(w), rows, dim, _sp(stream))


def softmax_dev(x, rows, n, stream=None):
    _call("iq_softmax_dev", _dp(x), rows, n, _sp(stream))


# --------------------------------------------------------- synthetic inputs

def synth_weights(cfg, name, shape):
    a = np.empty(shape, dtype=np.int64)
    _call("iq_synth_weights", lib().iq_tensor_seed(cfg, name.encode()), _hp(a), a.size)
    return a


def synth_acts(cfg, name, shape):
    a = np.empty(shape, dtype=np.int64)
    _call("iq_synth_acts", lib().iq_tensor_seed(cfg, name.encode()), _hp(a), a.size)
    return a


def synth_tokens(cfg, name, n, vocab):
    a = np.empty(n, dtype=np.int32)
    _call("iq_synth_tokens", lib().iq_tensor_seed(cfg, name.encode()), _hp(a), n, vocab)
    return a


# ------------------------------------------------------------------- model

class Config(ctypes.Structure):
    """iq_config (llama_config_t, llama_int.c:788-798)."""
    _fields_ = [(n, ctypes.c_int) for n in ("hidden_dim", "num_heads", "num_kv_heads", "head_dim",
                                             "num_layers", "intermediate_dim", "vocab_size",
                                             "max_seq_len", "rope_theta")]

    @classmethod
    def from_dict(cls, c):
        return cls(c["dim"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["n_layers"], c["inter"],
                   c["vocab"], c["max_seq"], c["rope_theta"])


class Model:
    """Device-resident integer Llama (iq_model_*): forward / generate with the
    reference's semantics (llama_forward, generate in llama_int.c)."""

    def __init__(self, cfg, max_batch=1, device=0, tp_rank=0, tp_size=1, nccl_id=None):
        self.cfg = cfg if isinstance(cfg, Config) else Config.from_dict(cfg)
        self.max_batch = max_batch
        self.h = ctypes.c_void_p()
        if tp_size == 1:
            _call("iq_model_create", ctypes.byref(self.cfg), max_batch, device, ctypes.byref(self.h))
        else:
            idbuf = ctypes.create_string_buffer(bytes(nccl_id), 128)
            _call("iq_model_create_tp", ctypes.byref(self.cfg), max_batch, device, tp_rank, tp_size,
                  idbuf, ctypes.byref(self.h))

    def close(self):
        if self.h:
            h, self.h = self.h, ctypes.c_void_p()   # the handle is gone even when destroy reports an error
            _call("iq_model_destroy", h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, w):
        """w: dict(embed, final_norm, lm_head, layers=[9 arrays per layer])."""
        _call("iq_model_load_globals", self.h, _hp(w["embed"]), _hp(w["final_norm"]), _hp(w["lm_head"]))
        for l, lay in enumerate(w["layers"]):
            arr = (ctypes.c_void_p * 9)(*[a.ctypes.data for a in lay])
            _call("iq_model_load_layer", self.h, l, arr)

    def load_mgw(self, path):
        """Every tensor from an int-llm .mgw file (iq_model_load_mgw)."""
        _call("iq_model_load_mgw", self.h, os.fsencode(path))

    def synth(self, config_index, threads=None):
        _call("iq_model_synth", self.h, config_index, threads or os.cpu_count() or 1)

    def reset(self):
        _call("iq_model_reset", self.h)

    def forward(self, token, pos, want_logits=True):
        lg = np.empty(self.cfg.vocab_size, dtype=np.int64) if want_logits else None
        a = ctypes.c_int(-1)
        _call("iq_forward", self.h, token, pos, _hp(lg) if want_logits else None, ctypes.byref(a))
        return a.value, lg

    def generate(self, prompt, max_new, logit_hash=False):
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(len(pr) + max_new, dtype=np.int32)
        n = ctypes.c_int(0)
        h = ctypes.c_uint64(0)
        _call("iq_generate", self.h, _hp(pr), len(pr), max_new, _hp(out), ctypes.byref(n),
              ctypes.byref(h) if logit_hash else None)
        return out[:n.value].tolist(), (h.value if logit_hash else None)

    def generate_sampled(self, prompt, max_new, temperature, top_k, top_p, seed, logit_hash=False):
        """generate() with sample_token (temperature / top_p in Q16.48)."""
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(len(pr) + max_new, dtype=np.int32)
        n = ctypes.c_int(0)
        h = ctypes.c_uint64(0)
        _call("iq_generate_sampled", self.h, _hp(pr), len(pr), max_new, temperature, top_k, top_p, seed, _hp(out),
              ctypes.byref(n), ctypes.byref(h) if logit_hash else None)
        return out[:n.value].tolist(), (h.value if logit_hash else None)

    def generate_batch(self, prompts, max_new, logit_hash=False):
        """Tokens per sequence; with logit_hash=True also the per-sequence hashes."""
        pr = np.ascontiguousarray(prompts, dtype=np.int32)
        B, L = pr.shape
        assert B == self.max_batch
        out = np.zeros((B, L + max_new), dtype=np.int32)
        n = np.zeros(B, dtype=np.int32)
        hs = np.zeros(B, dtype=np.uint64)
        _call("iq_generate_batch", self.h, _hp(pr), L, max_new, _hp(out), _hp(n), _hp(hs) if logit_hash else None)
        toks = [out[b, :n[b]].tolist() for b in range(B)]
        return (toks, [int(h) for h in hs]) if logit_hash else toks

    def set_attention(self, short_max):
        """Contexts up to short_max use the single-kernel attention (0 = phased only)."""
        _call("iq_model_set_attention", self.h, short_max)

    PEER_CHECK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)

    def set_peer_check(self, fn):
        """fn() -> bool, True when another tensor-parallel rank has left; checked
        before every call that launches work (iq_model_set_peer_check)."""
        self._peer_cb = self.PEER_CHECK(lambda _ctx: 1 if fn() else 0) if fn else None
        _call("iq_model_set_peer_check", self.h,
              ctypes.cast(self._peer_cb, ctypes.c_void_p) if fn else None, None)

    def set_timeout(self, ms):
        _call("iq_model_set_timeout", self.h, int(ms))

    def set_kv_packed(self, k_bits, v_bits):
        """The reference's --kv-packed KbVb cache (0, 0 = exact)."""
        _call("iq_model_set_kv_packed", self.h, k_bits, v_bits)

    def set_decode(self, mode):
        """1 = persistent decode kernel where it applies (default), 0 = one kernel per op."""
        _call("iq_model_set_decode", self.h, mode)

    def decode_info(self):
        """(persistent kernel in use, its grid size)."""
        a, b = ctypes.c_int(), ctypes.c_int()
        _call("iq_model_decode_info", self.h, ctypes.byref(a), ctypes.byref(b))
        return bool(a.value), b.value

    def weight_bytes(self):
        """(decode bytes per token, GEMM-form bytes) of this rank's stored weights."""
        d, g = ctypes.c_int64(), ctypes.c_int64()
        _call("iq_model_weight_bytes", self.h, ctypes.byref(d), ctypes.byref(g))
        return d.value, g.value

    def decode_steps_timed(self, pos0, steps):
        ms = ctypes.c_float(0)
        _call("iq_decode_steps_timed", self.h, pos0, steps, ctypes.byref(ms))
        return ms.value
