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
