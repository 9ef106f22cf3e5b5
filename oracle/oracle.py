"""ctypes loader for the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. It exposes:
  * ``O``   -- libiqoracle.so, the C restatement of the reference path
               (iq_oracle.c), always available once built;
  * ``ref()`` -- oracle/_ref/libllamaref.so, the reference llama_int.c compiled
               from source (ref_harness.c), or None where it was not built;
  * ``ref(shim=True)`` -- oracle/_ref/libllamaref_iq.so, the same reference
               with its matmul_vec replaced by the libiq.so drop-in
               (include/iq_matvec_shim.h): the integration check of that shim.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libiqoracle.so")
REF_SO = os.path.join(HERE, "_ref", "libllamaref.so")
REF_IQ_SO = os.path.join(HERE, "_ref", "libllamaref_iq.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64


def build():
    subprocess.check_call(["make", "-s", "-C", HERE], stdout=subprocess.DEVNULL)


def _load_oracle():
    if not os.path.exists(ORACLE_SO):
        build()
    L = ctypes.CDLL(ORACLE_SO)
    sig = {
        "iqo_fp": (_I64, [_I, _I64, _I64]),
        "iqo_fp_vec": (None, [_I, _P, _P, _P, _I64]),
        "iqo_det_hash": (_U64, [_P]),
        "iqo_matmul_vec": (None, [_P, _P, _P, _I, _I]),
        "iqo_matmul_rows": (None, [_P, _P, _P, _I, _I, _I]),
        "iqo_rmsnorm": (None, [_P, _P, _P, _I]),
        "iqo_softmax": (None, [_P, _I]),
        "iqo_rope_tables": (None, [_I, _I, _I, _P, _P]),
        "iqo_bf16_to_q1648": (_I64, [ctypes.c_uint16]),
        "iqo_q1648_to_bf16_rne": (ctypes.c_uint16, [_I64]),
        "iqo_fnv1a64": (_U64, [ctypes.c_char_p]),
        "iqo_fnv_mix_i64": (_U64, [_U64, _I64]),
        "iqo_fnv_array": (_U64, [_U64, _P, _I64]),
        "iqo_tensor_seed": (_U64, [_I, ctypes.c_char_p]),
        "iqo_synth_weights": (None, [_U64, _P, _I64]),
        "iqo_synth_acts": (None, [_U64, _P, _I64]),
        "iqo_synth_tokens": (None, [_U64, _P, _I, _I]),
        "iqo_model_create": (_P, [_P, _P, _P, _P, _P]),
        "iqo_model_reset": (None, [_P]),
        "iqo_model_forward": (_I, [_P, _I, _I, _P]),
        "iqo_model_generate": (_I, [_P, _P, _I, _I, _P, _P]),
        "iqo_model_free": (None, [_P]),
        "iqo_sample_token": (_I, [_P, _I, _I64, _I, _I64, _P]),
        "iqo_rng_seed": (None, [_U64, _P]),
        "iqo_model_generate_sampled": (_I, [_P, _P, _I, _I, _I64, _I, _I64, _U64, _P, _P]),
    }
    for k, (r, a) in sig.items():
        f = getattr(L, k)
        f.restype = r
        f.argtypes = a
    return L


O = _load_oracle()
_REF = None


_REF_IQ = None
_REF_SIG = {
    "ref_matmul_vec": (None, [_P, _P, _P, _I, _I]),
    "ref_matmul_vec_mt": (None, [_P, _P, _P, _I, _I, _I]),
    "ref_rmsnorm": (None, [_P, _P, _P, _I]),
    "ref_softmax": (None, [_P, _I]),
    "ref_bf16_to_q1648": (_I64, [ctypes.c_uint16]),
    "ref_fp": (_I64, [_I, _I64, _I64]),
    "ref_rope_tables": (None, [_I, _I, _I, _P, _P]),
    "ref_model_create": (_P, [_P, _P, _P, _P, _P]),
    "ref_model_reset": (None, [_P]),
    "ref_model_forward": (_I, [_P, _I, _I, _P]),
    "ref_model_generate": (_I, [_P, _P, _I, _I, _P]),
    "ref_model_free": (None, [_P]),
    "ref_model_open_mgw": (_P, [ctypes.c_char_p, _I]),
    "ref_model_close_mgw": (None, [_P]),
    "ref_sample_token": (_I, [_P, _I, _I64, _I, _I64, _P]),
    "ref_rng_seed": (None, [_U64, _P]),
    "ref_model_generate_sampled": (_I, [_P, _P, _I, _I, _I64, _I, _I64, _U64, _P]),
    "ref_set_kv_packed": (None, [_I, _I]),
}


def ref(shim=False):
    """The reference compiled from source (or, shim=True, its drop-in build
    linked to libiq.so), or None when oracle/_ref does not hold it."""
    global _REF, _REF_IQ
    path = REF_IQ_SO if shim else REF_SO
    cur = _REF_IQ if shim else _REF
    if cur is None and os.path.exists(path):
        L = ctypes.CDLL(path)
        for k, (r, a) in _REF_SIG.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        cur = L
        if shim:
            _REF_IQ = L
        else:
            _REF = L
    return cur


def p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------ conveniences

def seed(cfg, name):
    return O.iqo_tensor_seed(cfg, name.encode())


def synth_weights(cfg, name, shape):
    a = np.empty(shape, dtype=np.int64)
    O.iqo_synth_weights(seed(cfg, name), p(a), a.size)
    return a


def synth_acts(cfg, name, shape):
    a = np.empty(shape, dtype=np.int64)
    O.iqo_synth_acts(seed(cfg, name), p(a), a.size)
    return a


def synth_tokens(cfg, name, n, vocab):
    a = np.empty(n, dtype=np.int32)
    O.iqo_synth_tokens(seed(cfg, name), p(a), n, vocab)
    return a


def matmul_vec(w, x):
    M, N = w.shape
    out = np.empty(M, dtype=np.int64)
    O.iqo_matmul_vec(p(out), p(np.ascontiguousarray(w)), p(np.ascontiguousarray(x)), M, N)
    return out


def matmul_rows(w, X):
    M, N = w.shape
    rows = X.shape[0]
    out = np.empty((rows, M), dtype=np.int64)
    O.iqo_matmul_rows(p(out), p(np.ascontiguousarray(w)), p(np.ascontiguousarray(X)), rows, M, N)
    return out


def fp_vec(fn, x, y=None):
    out = np.empty_like(x)
    O.iqo_fp_vec(fn, p(x), p(y) if y is not None else None, p(out), x.size)
    return out


def fnv_hash(arr, h=1469598103934665603):
    """FNV-1a 64 over little-endian int64 values (fp_determinism.c:43-56)."""
    a = np.ascontiguousarray(arr, dtype=np.int64).ravel()
    return O.iqo_fnv_array(h, p(a), a.size)
