"""int-llm's own entry points over this library: the .mgw weight container
(llama_int.c:386-454, 2344-2803) and the source-level drop-in of matmul_vec
(include/iq_matvec_shim.h force-included into a copy of llama_int.c whose
line-1014 definition is renamed; built by `make -C oracle shim` into
oracle/_ref/libllamaref_iq.so)."""
import ctypes
import os

import numpy as np
import pytest

import configs
import helpers
import iq
import oracle as orc

needs_ref = pytest.mark.skipif(not os.path.exists(orc.REF_SO), reason="oracle/_ref not built")
needs_shim = pytest.mark.skipif(not os.path.exists(orc.REF_IQ_SO), reason="oracle/_ref/libllamaref_iq.so not built")


def _ref_generate(L, path, streaming, prompt, max_new):
    h = L.ref_model_open_mgw(os.fsencode(path), streaming)
    assert h, path
    pr = np.ascontiguousarray(prompt, dtype=np.int32)
    out = np.zeros(len(pr) + max_new, np.int32)
    n = L.ref_model_generate(h, orc.p(pr), len(pr), max_new, orc.p(out))
    L.ref_model_close_mgw(h)
    return out[:n].tolist()


@pytest.fixture(scope="module")
def tiny_mgw(tmp_path_factory):
    c = dict(configs.TINY_TEST)
    w = helpers.model_weights(9, c)
    d = tmp_path_factory.mktemp("mgw")
    paths = {}
    for tied in (False, True):
        paths[tied] = str(d / f"tiny_{int(tied)}.mgw")
        helpers.write_mgw(paths[tied], c, w, tied=tied)
    return c, w, paths


# ------------------------------------------------------------------ CPU

def test_mgw_config_roundtrip_and_rejects_malformed(tiny_mgw, tmp_path):
    c, w, paths = tiny_mgw
    got, tied = iq.mgw_config(paths[True])
    assert got == c and tied
    assert iq.mgw_config(paths[False]) == (c, False)
    bad = tmp_path / "bad.mgw"
    raw = bytearray(open(paths[False], "rb").read())
    raw[0:4] = b"XGW\0"                       # magic (llama_int.c:2369)
    bad.write_bytes(bytes(raw))
    with pytest.raises(iq.IQError):
        iq.mgw_config(str(bad))
    bad.write_bytes(bytes(raw[:100]))         # shorter than header + config
    with pytest.raises(iq.IQError):
        iq.mgw_config(str(bad))
    with pytest.raises(iq.IQError):
        iq.mgw_config(str(tmp_path / "missing.mgw"))


@needs_ref
def test_reference_loads_written_mgw_in_both_modes(tiny_mgw):
    """The test writer's files are ones the reference itself accepts: its mmap
    (mgw_load) and streaming (mgw_load_streaming) loaders give the same tokens
    as its generate() over the in-memory weights."""
    c, w, paths = tiny_mgw
    prompt = orc.synth_tokens(9, "prompt:mgw", 8, c["vocab"])
    R = orc.ref()
    m = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    want, _ = m.generate(prompt, 16)
    m.close()
    for tied in (False,):
        for streaming in (0, 1):
            assert _ref_generate(R, paths[tied], streaming, prompt, 16) == want


# ------------------------------------------------------------------ GPU

@pytest.mark.gpu
@needs_ref
def test_model_load_mgw_matches_reference(tiny_mgw):
    """iq_model_load_mgw on untied and tied files: tokens equal the reference's
    generate() on the same file, every logit hash equals its llama_forward's."""
    c, w, paths = tiny_mgw
    prompt = orc.synth_tokens(9, "prompt:mgw", 8, c["vocab"])
    R = orc.ref()
    for tied in (False, True):
        cfg, t = iq.mgw_config(paths[tied])
        m = iq.Model(cfg)
        m.load_mgw(paths[tied])
        toks, lh = m.generate(prompt, 16, logit_hash=True)
        m.close()
        wt = dict(w, lm_head=w["embed"]) if tied else w
        o = helpers.OracleModel(c, wt, lib=R, prefix="ref_")
        want, _ = o.generate(prompt, 16)
        o.close()
        assert toks == want == _ref_generate(R, paths[tied], 0, prompt, 16), tied
        oi = helpers.OracleModel(c, wt)
        _, lh_o = oi.generate(prompt, 16)
        oi.close()
        assert lh == lh_o, tied


@pytest.mark.gpu
@needs_shim
def test_dropin_shim_in_reference_generate_cached_and_streaming(tiny_mgw):
    """The reference's own generate() with every matmul_vec call served by
    iq_matmul_vec: the mmap'd (layers cached) path and the streaming path, which
    mallocs each layer afresh and frees it after use (llama_int.c:2840-2872),
    give the unpatched reference's tokens, under the default sampled check and
    under the full-hash check."""
    c, w, paths = tiny_mgw
    prompt = orc.synth_tokens(9, "prompt:mgw", 8, c["vocab"])
    R, S = orc.ref(), orc.ref(shim=True)
    want = _ref_generate(R, paths[False], 1, prompt, 20)
    try:
        for mode in ("sampled", "full"):
            iq.weight_check_mode(mode)
            for streaming in (0, 1):
                iq.weight_cache_clear()
                got = _ref_generate(S, paths[False], streaming, prompt, 20)
                assert got == want, (mode, streaming)
                entries, nbytes = iq.weight_cache_stats()
                assert entries > 0 and nbytes > 0   # the drop-in really ran
    finally:
        iq.weight_check_mode("sampled")
        iq.weight_cache_clear()
