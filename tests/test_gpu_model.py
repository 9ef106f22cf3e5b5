"""GPU parity of the device forward / generate against the oracle and the
reference goldens (every logit, token ids, logit hash)."""
import json
import os

import numpy as np
import pytest

import configs
import helpers
import iq
import oracle as orc

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def gold(n):
    return json.load(open(os.path.join(GOLD, n)))


@pytest.fixture(scope="module")
def tiny():
    g = gold("tiny_model.json")
    c = g["config"]
    w = helpers.model_weights(g["cfg_index"], c)
    m = iq.Model(c)
    m.load(w)
    yield g, c, w, m
    m.close()


def test_tiny_generate_matches_reference_golden(tiny):
    g, c, w, m = tiny
    toks, lh = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
    assert toks == g["tokens"]
    assert lh == g["logit_hash"]
    toks2, _ = m.generate(np.array(g["prompt"]), g["max_new"])   # graph path, no per-step sync
    assert toks2 == g["tokens"]


@pytest.mark.parametrize("short_max", [0, 9, 1 << 20])
def test_attention_kernel_choice_is_bit_identical(tiny, short_max):
    """Phased attention only (0), a switch from single-kernel to phased in the
    middle of decoding (9), single-kernel only: same tokens and logit hash."""
    g, c, w, m = tiny
    m.set_attention(short_max)
    try:
        toks, lh = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
        toks2, _ = m.generate(np.array(g["prompt"]), g["max_new"])
    finally:
        m.set_attention(384)
    assert toks == toks2 == g["tokens"]
    assert lh == g["logit_hash"]


def test_tiny_forward_every_logit_vs_oracle(tiny):
    g, c, w, m = tiny
    o = helpers.OracleModel(c, w)
    m.reset()
    toks = orc.synth_tokens(9, "prompt:fwd", 40, c["vocab"])
    for pos, t in enumerate(toks):
        a1, l1 = m.forward(int(t), pos)
        a2, l2 = o.forward(int(t), pos)
        assert (l1 == l2).all(), pos
        assert a1 == a2
    o.close()


def test_forward_range_errors(tiny):
    g, c, w, m = tiny
    for tok, pos in ((c["vocab"], 0), (-1, 0), (0, c["max_seq"]), (0, -1)):
        with pytest.raises(iq.IQError) as e:
            m.forward(tok, pos)
        assert e.value.status == -6


def test_generate_stops_at_max_seq():
    c = dict(configs.TINY_TEST, max_seq=12, n_layers=1)
    w = helpers.model_weights(9, c)
    m = iq.Model(c)
    m.load(w)
    o = helpers.OracleModel(c, w)
    pr = orc.synth_tokens(9, "prompt:short", 8, c["vocab"])
    t1, h1 = m.generate(pr, 30, logit_hash=True)
    t2, h2 = o.generate(pr, 30)
    t3, _ = m.generate(pr, 30)
    assert t1 == t2 == t3 and h1 == h2
    m.close(); o.close()


def test_batched_generate_equals_independent_sequences():
    c = dict(configs.TINY_TEST, max_seq=48)
    w = helpers.model_weights(9, c)
    B = 5
    m = iq.Model(c, max_batch=B)
    m.load(w)
    o = helpers.OracleModel(c, w)
    prompts = np.stack([orc.synth_tokens(9, f"prompt:b{b}", 6, c["vocab"]) for b in range(B)])
    got = m.generate_batch(prompts, 20)
    for b in range(B):
        want, _ = o.generate(prompts[b], 20)
        assert got[b] == want, b
    m.close(); o.close()


def test_cfg0_tinyllama_greedy_decode_golden():
    """Config 0: TinyLlama-shape model, seeded weights, 8-token prompt, 32 greedy
    tokens; token ids and the FNV hash of every logit equal the reference's."""
    g = gold("cfg0_tinyllama.json")
    m = iq.Model(configs.TINYLLAMA)
    m.synth(0)
    m.reset()
    a, lg = m.forward(g["prompt"][0], 0)
    assert orc.fnv_hash(lg) == g["first_step_logit_hash"]
    toks, lh = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
    assert toks == g["tokens"]
    assert orc.fnv_hash(np.array(toks)) == g["token_hash"]
    assert lh == g["logit_hash"]
    toks2, _ = m.generate(np.array(g["prompt"]), g["max_new"])
    assert toks2 == g["tokens"]
    m.set_attention(0)  # phased attention kernels on the same golden
    toks3, lh3 = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
    assert toks3 == g["tokens"] and lh3 == g["logit_hash"]
    m.close()


def test_long_prompt_chunked_prefill_matches_sequential_oracle():
    """A prompt longer than one prefill chunk (1024 rows): batched prefill with
    per-row causal attention equals the reference's position-by-position loop,
    every logit included (hash), then greedy decode continues identically."""
    c = dict(configs.TINY_TEST, n_layers=1, max_seq=1100)
    w = helpers.model_weights(9, c)
    m = iq.Model(c)
    m.load(w)
    o = helpers.OracleModel(c, w)
    pr = orc.synth_tokens(9, "prompt:long", 1030, c["vocab"])
    t1, h1 = m.generate(pr, 12, logit_hash=True)
    t2, h2 = o.generate(pr, 12)
    t3, _ = m.generate(pr, 12)
    assert t1 == t2 == t3 and h1 == h2
    m.close(); o.close()


def _load_model(g, max_batch=1):
    c = g["config"]
    w = helpers.model_weights(g["cfg_index"], c)
    m = iq.Model(c, max_batch=max_batch)
    m.load(w)
    return c, w, m


def test_geom7b_hd128_mha_matches_reference_golden():
    """Llama-2-7B geometry at reduced width (head_dim 128, n_kv = n_heads, FFN
    ratio 11008/4096): a 370-token prompt and 29 decode steps that cross from the
    single-kernel attention (context <= 384) to the phased kernels. Tokens and
    the hash of every logit of all 399 forwards equal the reference's."""
    g = gold("geom7b_model.json")
    c, w, m = _load_model(g)
    prompt = orc.synth_tokens(g["cfg_index"], g["prompt_name"], g["prompt_len"], c["vocab"])
    for short_max in (384, 0):   # default switch-over, then phased attention only
        m.set_attention(short_max)
        toks, lh = m.generate(prompt, g["max_new"], logit_hash=True)
        assert toks[g["prompt_len"]:] == g["tokens"], short_max
        assert lh == g["logit_hash"], short_max
        toks2, _ = m.generate(prompt, g["max_new"])   # graph path, no per-step sync
        assert toks2[g["prompt_len"]:] == g["tokens"], short_max
    m.close()


def test_eos_stops_generation_like_the_reference():
    """A model whose LM-head row 2 ties the row of a token greedy decoding emits
    mid-generation: the first-max rule then samples EOS (2) and generate() stops
    (llama_int.c:3110). Tokens, the returned length and the logit hash (which
    covers the forward that sampled EOS) equal the reference's; the batched path
    stops each sequence the same way."""
    g = gold("eos_model.json")
    c = g["config"]
    w = helpers.model_weights(g["cfg_index"], c)
    w["lm_head"][2] = w["lm_head"][g["lm_head_row2_from"]]
    m = iq.Model(c)
    m.load(w)
    toks, lh = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
    assert toks == g["tokens"] and len(toks) == g["n_out"] < len(g["prompt"]) + g["max_new"]
    assert lh == g["logit_hash"]
    toks2, _ = m.generate(np.array(g["prompt"]), g["max_new"])
    assert toks2 == g["tokens"]
    m.close()
    mb = iq.Model(c, max_batch=3)
    mb.load(w)
    other = orc.synth_tokens(g["cfg_index"], "prompt:other", 8, c["vocab"])
    prompts = np.stack([np.array(g["prompt"]), other, np.array(g["prompt"])])
    got, hs = mb.generate_batch(prompts, g["max_new"], logit_hash=True)
    assert got[0] == got[2] == g["tokens"] and hs[0] == hs[2] == g["logit_hash"]
    o = helpers.OracleModel(c, w)
    want1, lh1 = o.generate(other, g["max_new"])
    assert got[1] == want1 and hs[1] == lh1
    o.close()
    mb.close()


def test_cfg3_geometry_batched_decode_matches_reference_golden():
    """Config-3 geometry (TinyLlama width, GQA 8:1, 2 layers, max_seq 2176):
    8 sequences with 2080-token prompts prefilled, then 23 batched decode steps
    at context 2081..2103. Every sequence's tokens and every-logit hash equal
    the reference's generate() run on that sequence alone."""
    g = gold("cfg3_model.json")
    c, w, m = _load_model(g, max_batch=g["batch"])
    prompts = np.stack([orc.synth_tokens(g["cfg_index"], n, g["prompt_len"], c["vocab"])
                        for n in g["prompt_names"]])
    got, hs = m.generate_batch(prompts, g["max_new"], logit_hash=True)
    for b in range(g["batch"]):
        assert got[b][g["prompt_len"]:] == g["tokens"][b], b
        assert hs[b] == g["logit_hashes"][b], b
    got2 = m.generate_batch(prompts, g["max_new"])
    assert [t[g["prompt_len"]:] for t in got2] == g["tokens"]
    m.close()


# ------------------------------------------------- persistent decode kernel

def test_persistent_decode_kernel_matches_goldens():
    """Decode mode 1 (one cooperative kernel per step, grid barriers between
    phases) gives the reference's tokens and every-logit hash: the tiny model
    (short-context attention, one CTA per head) and the 7B-geometry model from
    position 370 on (contexts above 256: attention split over 64-position
    tiles in three barrier-separated steps)."""
    g = gold("tiny_model.json")
    c, w, m = _load_model(g)
    m.set_decode(1)
    assert m.decode_info()[0]
    toks, lh = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
    assert toks == g["tokens"] and lh == g["logit_hash"]
    toks2, _ = m.generate(np.array(g["prompt"]), g["max_new"])
    assert toks2 == g["tokens"]
    assert iq.device_status() == 0
    m.close()
    g = gold("geom7b_model.json")
    c, w, m = _load_model(g)
    m.set_decode(1)
    assert m.decode_info()[0]
    prompt = orc.synth_tokens(g["cfg_index"], g["prompt_name"], g["prompt_len"], c["vocab"])
    toks, lh = m.generate(prompt, g["max_new"], logit_hash=True)
    assert toks[g["prompt_len"]:] == g["tokens"] and lh == g["logit_hash"]
    assert iq.device_status() == 0
    m.close()


def test_persistent_decode_crosses_into_tiled_attention():
    """A decode that starts below and ends above the 256-position switch of the
    persistent kernel's attention equals the oracle, every logit hashed; and
    mode 0 gives the same."""
    c = dict(configs.TINY_TEST, n_layers=1, max_seq=300)
    w = helpers.model_weights(9, c)
    m = iq.Model(c)
    m.load(w)
    o = helpers.OracleModel(c, w)
    pr = orc.synth_tokens(9, "prompt:cross", 240, c["vocab"])
    want, wlh = o.generate(pr, 40)
    for mode in (1, 0):
        m.set_decode(mode)
        assert m.decode_info()[0] == (mode == 1)
        t1, h1 = m.generate(pr, 40, logit_hash=True)
        t2, _ = m.generate(pr, 40)
        assert t1 == t2 == want and h1 == wlh, mode
    m.close(); o.close()


# ------------------------------------------------------------------ sampling

ONE = 1 << 48
SAMPLE_PARAMS = [(0, 0, ONE), (ONE // 200, 0, ONE), (ONE // 100, 0, ONE), (ONE, 0, ONE), (ONE // 2, 5, ONE),
                 (ONE * 3 // 2, 40, ONE * 9 // 10), (ONE, 0, ONE // 2), (ONE * 2, 1, ONE), (ONE, 0, 1),
                 (ONE // 3, 100, ONE * 3 // 4), (ONE, 31999, ONE * 99 // 100)]


def test_sample_token_device_vs_oracle():
    """k_sample equals the oracle's sample_token (itself pinned to the
    reference's) on random logits: vocabulary sizes 1..32000, ties planted at
    the maximum and at the top-k / top-p boundaries, every parameter regime,
    three consecutive draws per generator state."""
    import torch
    rng = np.random.default_rng(17)
    for trial, V in enumerate([1, 7, 600, 5000, 32000]):
        rows = 3
        lg = rng.integers(-(8 << 48), 8 << 48, (rows, V)).astype(np.int64)
        if V > 20:
            lg[0, rng.integers(0, V, 9)] = lg[0].max()
            lg[1, rng.integers(0, V, 40)] = np.sort(lg[1])[-30]     # ties inside the top k
            lg[2] = lg[2] >> 20                                     # narrow spread: flat softmax
        d = torch.from_numpy(lg).cuda()
        for temp, k, p in SAMPLE_PARAMS:
            st = np.zeros((rows, 2), np.uint64)
            for r in range(rows):
                orc.O.iqo_rng_seed(trial * 100 + r + k, orc.p(st[r]))
            ost = st.copy()
            for draw in range(3):
                got = iq.sample_dev(d, rows, V, temp, k, p, st)
                for r in range(rows):
                    s2 = np.ascontiguousarray(ost[r])
                    want = orc.O.iqo_sample_token(orc.p(np.ascontiguousarray(lg[r])), V, temp, k, p, orc.p(s2))
                    ost[r] = s2
                    assert got[r] == want, (V, temp, k, p, draw, r)
                assert (st == ost).all()


def test_generate_sampled_matches_oracle_and_reference_golden():
    """generate() with sampling: the tiny model against the oracle (tokens and
    every-logit hash) for several parameter sets, and the config-0 model
    against the reference's own sampled generate (golden)."""
    c = dict(configs.TINY_TEST, max_seq=64)
    w = helpers.model_weights(9, c)
    m = iq.Model(c)
    m.load(w)
    o = helpers.OracleModel(c, w)
    pr = np.ascontiguousarray(orc.synth_tokens(9, "prompt:sample", 8, c["vocab"]), dtype=np.int32)
    for temp, k, p in SAMPLE_PARAMS[:8]:
        toks, lh = m.generate_sampled(pr, 24, temp, k, p, 99, logit_hash=True)
        out = np.zeros(8 + 24, np.int32)
        import ctypes
        h = ctypes.c_uint64()
        n = orc.O.iqo_model_generate_sampled(o.h, orc.p(pr), 8, 24, temp, k, p, 99, orc.p(out), ctypes.byref(h))
        assert toks == out[:n].tolist() and lh == h.value, (temp, k, p)
        toks2, _ = m.generate_sampled(pr, 24, temp, k, p, 99)
        assert toks2 == toks
    g, _ = m.generate(pr, 24)   # greedy again afterwards
    assert g == o.generate(pr, 24)[0]
    m.close(); o.close()
    gs = gold("cfg0_sampled.json")
    m = iq.Model(configs.TINYLLAMA)
    m.synth(0)
    for run in gs["runs"]:
        toks, _ = m.generate_sampled(np.array(gs["prompt"]), gs["max_new"], run["temperature"], run["top_k"],
                                     run["top_p"], run["seed"])
        assert toks == run["tokens"], run["seed"]
    m.close()


# ------------------------------------------------------------- packed KV cache

@pytest.mark.skipif(orc.ref() is None, reason="oracle/_ref not built")
@pytest.mark.parametrize("kb,vb", [(8, 10), (4, 16), (1, 1)])
def test_packed_kv_cache_matches_reference(kb, vb):
    """--kv-packed KbVb (per-vector L-inf magnitude + b-bit codes, llama_int.c:
    1197-1235, 1392-1501): tokens equal the reference's own generate() with
    the same switch, every logit hash equals its llama_forward's, for a prompt
    prefilled in batched rows and decode past several 64-position tiles; the
    exact cache again afterwards gives the exact goldens."""
    c = dict(configs.TINY_TEST, max_seq=200)
    w = helpers.model_weights(9, c)
    R = orc.ref()
    pr = orc.synth_tokens(9, "prompt:packed", 90, c["vocab"])
    R.ref_set_kv_packed(kb, vb)
    try:
        mr = helpers.OracleModel(c, w, lib=R, prefix="ref_")
        want, _ = mr.generate(pr, 60)
        mr.reset()
        lh = 1469598103934665603
        toks = [int(t) for t in pr]
        for pos in range(len(toks) + 59):
            a, lg = mr.forward(toks[pos], pos)
            lh = orc.O.iqo_fnv_array(lh, orc.p(lg), lg.size)
            if pos >= len(pr) - 1:
                if pos > len(pr) - 1 and a == 2:
                    break
                toks.append(a)
        mr.close()
    finally:
        R.ref_set_kv_packed(0, 0)
    m = iq.Model(c)
    m.load(w)
    m.set_kv_packed(kb, vb)
    got, glh = m.generate(pr, 60, logit_hash=True)
    got2, _ = m.generate(pr, 60)
    assert got == got2 == want
    assert glh == lh
    m.set_kv_packed(0, 0)
    o = helpers.OracleModel(c, w)
    assert m.generate(pr, 30)[0] == o.generate(pr, 30)[0]
    o.close()
    m.close()
