"""CPU tests of the C-ABI boundary: libiq.so builds, loads without a GPU and
exports every symbol include/iq.h declares; argument validation needs no GPU."""
import ctypes
import os
import re
import subprocess

import numpy as np

import iq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            syms |= set(re.findall(r"IQ_API\s+[\w\s\*]+?\b(iq_\w+)\s*\(", txt))
    return syms


def test_library_exports_every_declared_symbol():
    L = iq.lib()
    syms = declared_symbols()
    assert len(syms) >= 10
    out = subprocess.check_output(["nm", "-D", "--defined-only", iq.LIB_PATH]).decode()
    exported = set(re.findall(r" T (iq_\w+)", out))
    missing = syms - exported
    assert not missing, missing
    for s in syms:
        getattr(L, s)
    # the python mirror binds every declared symbol
    assert syms <= set(iq.SIGNATURES), syms - set(iq.SIGNATURES)


def test_library_is_self_contained():
    out = subprocess.check_output(["ldd", iq.LIB_PATH]).decode()
    assert "libcudart" not in out  # runtime linked statically
    assert "oracle" not in out


def test_status_strings_and_arg_checks():
    L = iq.lib()
    assert L.iq_status_str(0) == b"ok"
    assert L.iq_status_str(-6) == b"out of range"
    assert L.iq_version() >= 100
    # argument errors are reported before any device work
    assert L.iq_matmul_vec(None, None, None, 4, 4) == -1
    a = np.zeros(4, dtype=np.int64)
    pa = a.ctypes.data_as(ctypes.c_void_p)
    assert L.iq_matmul_vec(pa, pa, pa, 0, 4) == -1
    assert L.iq_matmul_vec(pa, pa, pa, 4, -1) == -1
    assert L.iq_matvec_dev(pa, pa, pa, 4, 4, None) == -1   # out aliases in
    assert L.iq_fp_dev(99, pa, None, pa, 4, None) == -1
    assert L.iq_fp_dev(0, pa, None, pa, 4, None) == -1     # fp_mul needs y


def test_synth_generator_matches_oracle():
    import oracle as orc
    for cfg, name, shape in ((1, "w:2048x256", (256, 64)), (0, "lm_head.weight", (3000,))):
        assert (iq.synth_weights(cfg, name, shape) == orc.synth_weights(cfg, name, shape)).all()
    assert (iq.synth_acts(1, "x:2048x256", (2048,)) == orc.synth_acts(1, "x:2048x256", (2048,))).all()
    assert (iq.synth_tokens(0, "prompt:0", 64, 32000) == orc.synth_tokens(0, "prompt:0", 64, 32000)).all()
    L = iq.lib()
    for b in range(0, 65536, 5):
        assert L.iq_bf16_to_q1648(b) == orc.O.iqo_bf16_to_q1648(b)


def test_watchdog_logic_without_gpu():
    """The bounded wait of tensor-parallel steps (iq_selftest_watchdog runs the
    library's own wait loop on scripted events): completion returns IQ_OK
    without abort; a communicator error returns IQ_ERR_NCCL and aborts; a step
    that never completes times out (IQ_ERR_TIMEOUT) and aborts; a failed stream
    query is a CUDA error."""
    L = iq.lib()
    ab, polls = ctypes.c_int(), ctypes.c_int()
    assert L.iq_selftest_watchdog(0, ctypes.byref(ab), ctypes.byref(polls)) == 0
    assert ab.value == 0 and polls.value == 3
    assert L.iq_selftest_watchdog(1, ctypes.byref(ab), ctypes.byref(polls)) == -4
    assert ab.value == 1 and polls.value == 2
    assert L.iq_selftest_watchdog(2, ctypes.byref(ab), ctypes.byref(polls)) == -5
    assert ab.value == 1 and polls.value == 11   # 10 ms per poll, limit 100 ms
    assert L.iq_selftest_watchdog(3, ctypes.byref(ab), ctypes.byref(polls)) == -2
    assert ab.value == 0
