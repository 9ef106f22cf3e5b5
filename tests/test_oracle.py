"""CPU tests: pin the C restatement oracle against the reference's golden
vectors and against the reference compiled from source (when present)."""
import json
import os

import numpy as np
import pytest

import configs
import helpers
import oracle as orc

GOLD = os.path.join(os.path.dirname(__file__), "golden")
ONE = 1 << 48
FN_NAMES = ["fp_mul", "fp_div", "fp_sqrt", "fp_sqrt_fast", "fp_inv_sqrt", "fp_exp", "fp_log",
            "fp_sincos_cos", "fp_sincos_sin", "fp_sigmoid", "fp_silu", "fp_rng"]


def gold(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def test_determinism_golden():
    """fp_determinism.c grid hash: the reference's committed golden c0d933ea340452ec
    (tests/determinism_golden.txt) and every per-function sub-hash."""
    import ctypes
    subs = (ctypes.c_uint64 * 12)()
    comb = orc.O.iqo_det_hash(subs)
    g = gold("determinism.json")
    assert g["DETERMINISM_HASH"] == "c0d933ea340452ec"
    assert f"{comb:016x}" == g["DETERMINISM_HASH"]
    for i, n in enumerate(FN_NAMES):
        assert f"{subs[i]:016x}" == g["sub:" + n], n


def test_bf16_conversion_kats():
    """fp_test.c:1181-1233 bf16 known answers (exact values here)."""
    f = orc.O.iqo_bf16_to_q1648
    assert f(0x0000) == 0
    assert f(0x3F80) == ONE
    assert f(0xBF80) == -ONE
    assert f(0x4000) == 2 * ONE
    assert f(0x3F00) == ONE // 2
    assert f(0x7F80) == 32000 * ONE      # exponent 255 clamps
    assert f(0x0001) == 0                # subnormal -> 0


def test_bf16_rne_roundtrip():
    f, g = orc.O.iqo_bf16_to_q1648, orc.O.iqo_q1648_to_bf16_rne
    for b in list(range(0x3000, 0x4700, 7)) + list(range(0xB000, 0xC700, 11)):
        v = f(b)
        assert g(v) == b, hex(b)
    # round to nearest even: halfway between 1.0 and 1.0078125 rounds to 1.0
    assert g(ONE + (ONE >> 8)) == 0x3F80
    assert g(ONE + 3 * (ONE >> 8)) == 0x3F82


def test_synth_weights_bf16_exact():
    w = orc.synth_weights(1, "w:test", (1000,))
    back = np.array([orc.O.iqo_bf16_to_q1648(orc.O.iqo_q1648_to_bf16_rne(int(v))) for v in w])
    assert (back == w).all()
    assert np.abs(w).max() < (1 << 47)
    # N(0, 0.02): sample std within 10%
    s = np.std(w.astype(np.float64) / ONE)
    assert 0.018 < s < 0.022


def test_synth_acts_range():
    x = orc.synth_acts(1, "x:test", (4096,))
    assert x.min() >= -(8 * ONE) and x.max() < 8 * ONE


def test_matvec_cfg1_golden():
    """Config-1 shapes: the restatement reproduces the reference outputs (hash of all rows)."""
    for g in gold("matvec_cfg1.json"):
        K, N = g["K"], g["N"]
        w = orc.synth_weights(1, g["weight"], (N, K))
        x = orc.synth_acts(1, g["act"], (K,))
        assert orc.fnv_hash(w) == g["w_hash"]
        assert orc.fnv_hash(x) == g["x_hash"]
        out = orc.matmul_vec(w, x)
        assert [int(v) for v in out[:8]] == g["out_head"]
        assert orc.fnv_hash(out) == g["out_hash"]


def test_tiny_model_golden():
    g = gold("tiny_model.json")
    c = g["config"]
    w = helpers.model_weights(g["cfg_index"], c)
    m = helpers.OracleModel(c, w)
    toks, lh = m.generate(np.array(g["prompt"]), g["max_new"])
    m.close()
    assert toks == g["tokens"]
    assert lh == g["logit_hash"]


# ---------------- against the reference compiled from source (this container only)

needs_ref = pytest.mark.skipif(orc.ref() is None, reason="oracle/_ref not built")


@needs_ref
def test_fp_functions_vs_reference():
    R = orc.ref()
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.integers(-(1 << 62), 1 << 62, 2000),
                         rng.integers(-40 * ONE, 40 * ONE, 2000),
                         np.array([0, 1, -1, ONE, -ONE, 2 ** 63 - 1, -2 ** 63 + 1])]).astype(np.int64)
    ys = np.roll(xs, 17)
    for fn in range(12):
        for x, y in zip(xs[::3], ys[::3]):
            x, y = int(x), int(y)
            if fn == 1 and y == 0:
                continue
            assert orc.O.iqo_fp(fn, x, y) == R.ref_fp(fn, x, y), (fn, x, y)


@needs_ref
@pytest.mark.parametrize("M,N", [(1, 1), (3, 17), (5, 64), (7, 65), (64, 1000), (33, 2048)])
def test_matvec_vs_reference_edges(M, N):
    R = orc.ref()
    rng = np.random.default_rng(M * 1000 + N)
    for dist in ("full", "cfg"):
        if dist == "full":   # full-range int64: exercises the mod 2^128 wrap
            w = rng.integers(-2 ** 63, 2 ** 63 - 1, (M, N), dtype=np.int64)
            x = rng.integers(-2 ** 63, 2 ** 63 - 1, N, dtype=np.int64)
        else:
            w = orc.synth_weights(1, f"w:{M}x{N}", (M, N))
            x = orc.synth_acts(1, f"x:{M}x{N}", (N,))
        ref = np.empty(M, dtype=np.int64)
        R.ref_matmul_vec(orc.p(ref), orc.p(w), orc.p(x), M, N)
        assert (orc.matmul_vec(w, x) == ref).all()


@needs_ref
def test_rmsnorm_softmax_rope_vs_reference():
    R = orc.ref()
    rng = np.random.default_rng(3)
    for dim in (1, 7, 256, 2048):
        x = rng.integers(-8 * ONE, 8 * ONE, dim, dtype=np.int64)
        w = rng.integers(-2 * ONE, 2 * ONE, dim, dtype=np.int64)
        a, b = np.empty_like(x), np.empty_like(x)
        R.ref_rmsnorm(orc.p(a), orc.p(x), orc.p(w), dim)
        orc.O.iqo_rmsnorm(orc.p(b), orc.p(x), orc.p(w), dim)
        assert (a == b).all()
        s1 = rng.integers(-30 * ONE, 30 * ONE, dim, dtype=np.int64)
        s2 = s1.copy()
        R.ref_softmax(orc.p(s1), dim)
        orc.O.iqo_softmax(orc.p(s2), dim)
        assert (s1 == s2).all()
    for hd, T in ((64, 300), (128, 100)):
        c1, s1 = np.empty(T * hd // 2, np.int64), np.empty(T * hd // 2, np.int64)
        c2, s2 = np.empty_like(c1), np.empty_like(s1)
        R.ref_rope_tables(hd, T, 10000, orc.p(c1), orc.p(s1))
        orc.O.iqo_rope_tables(hd, T, 10000, orc.p(c2), orc.p(s2))
        assert (c1 == c2).all() and (s1 == s2).all()


@needs_ref
def test_bf16_all_vs_reference():
    R = orc.ref()
    for b in range(0, 65536, 3):
        assert orc.O.iqo_bf16_to_q1648(b) == R.ref_bf16_to_q1648(b)


@needs_ref
def test_tiny_model_logits_vs_reference():
    c = dict(configs.TINY_TEST, n_layers=1, max_seq=40)
    w = helpers.model_weights(9, c)
    a = helpers.OracleModel(c, w)
    b = helpers.OracleModel(c, w, lib=orc.ref(), prefix="ref_")
    toks = orc.synth_tokens(9, "prompt:x", 20, c["vocab"])
    for pos, t in enumerate(toks):
        ia, la = a.forward(int(t), pos)
        ib, lb = b.forward(int(t), pos)
        assert ia == ib and (la == lb).all(), pos
    # rejected token / position: both refuse (llama_int.c:2813-2820)
    assert a.forward(c["vocab"], 0)[0] == -1 and b.forward(c["vocab"], 0)[0] == -1
    assert a.forward(0, c["max_seq"])[0] == -1 and b.forward(0, c["max_seq"])[0] == -1
    a.close(); b.close()


# ------------------------------------------------------------------ sampling

def _params():
    ONE_ = 1 << 48
    return [(0, 0, ONE_), (ONE_ // 200, 0, ONE_), (ONE_ // 100, 0, ONE_), (ONE_, 0, ONE_),
            (ONE_ // 2, 5, ONE_), (ONE_ * 3 // 2, 40, ONE_ * 9 // 10), (ONE_, 0, ONE_ // 2),
            (ONE_ * 2, 1, ONE_), (ONE_, 0, 1), (ONE_ // 3, 100, ONE_ * 3 // 4)]


@pytest.mark.skipif(orc.ref() is None, reason="oracle/_ref not built")
def test_sample_token_restatement_vs_reference():
    """The oracle's sample_token restatement equals the reference's own
    (llama_int.c:2958-3039) on random logits, with ties planted, over
    temperature (below/at the 0.01 floor), top-k, top-p, and consecutive draws
    from one generator state."""
    import ctypes
    R = orc.ref()
    rng = np.random.default_rng(5)
    for trial in range(30):
        V = int(rng.integers(1, 600))
        lg = (rng.integers(-(8 << 48), 8 << 48, V)).astype(np.int64)
        if V > 10:
            lg[rng.integers(0, V, 5)] = lg.max()    # ties at the maximum
        for temp, k, p in _params():
            s1 = np.zeros(2, np.uint64)
            orc.O.iqo_rng_seed(trial * 7 + k, orc.p(s1))
            s2 = s1.copy()
            for draw in range(3):
                a = orc.O.iqo_sample_token(orc.p(lg), V, temp, k, p, orc.p(s1))
                b = R.ref_sample_token(orc.p(lg), V, temp, k, p, orc.p(s2))
                assert a == b, (trial, temp, k, p, draw)
                assert (s1 == s2).all()


@pytest.mark.skipif(orc.ref() is None, reason="oracle/_ref not built")
def test_generate_sampled_restatement_vs_reference():
    c = dict(configs.TINY_TEST, n_layers=1, max_seq=64)
    w = helpers.model_weights(9, c)
    pr = np.ascontiguousarray(orc.synth_tokens(9, "prompt:sample", 8, c["vocab"]), dtype=np.int32)
    R = orc.ref()
    mo = helpers.OracleModel(c, w)
    mr = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    for temp, k, p in _params()[:7]:
        o1 = np.zeros(8 + 20, np.int32)
        o2 = np.zeros(8 + 20, np.int32)
        n1 = orc.O.iqo_model_generate_sampled(mo.h, orc.p(pr), 8, 20, temp, k, p, 1234, orc.p(o1), None)
        n2 = R.ref_model_generate_sampled(mr.h, orc.p(pr), 8, 20, temp, k, p, 1234, orc.p(o2))
        assert n1 == n2 and (o1[:n1] == o2[:n2]).all(), (temp, k, p)
    mo.close(); mr.close()
