"""Generates the committed golden fixtures from the REFERENCE itself.

Run in a container where the reference checkout exists and oracle/_ref is built
(`make -C oracle`). Every value here comes from the reference's own code
compiled from source (oracle/_ref/libllamaref.so, oracle/_ref/fp_determinism);
the C restatement (oracle/libiqoracle.so) is only used for the synthetic
inputs, whose generator is cross-checked against the reference's bf16 decoder.

  python tests/golden/make_golden.py            # fast fixtures (or --fast with other flags)
  python tests/golden/make_golden.py --cfg0     # TinyLlama greedy decode: tokens + every-logit hash (minutes)
  python tests/golden/make_golden.py --cfg2     # M=512 GEMM hashes
  python tests/golden/make_golden.py --geom7b   # head_dim-128 MHA model, 400 positions
  python tests/golden/make_golden.py --cfg3     # config-3 geometry, 8 sequences at T~2100 (minutes, 8 processes)
  python tests/golden/make_golden.py --eos      # a model made to emit EOS (token 2) mid-generation
  python tests/golden/make_golden.py --sampled  # config-0 generate() with sampling, 3 parameter sets (minutes)
"""
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "int-llm_b200"),
                os.path.join(ROOT, "tests")]
import configs  # noqa: E402
import helpers  # noqa: E402
import oracle as orc  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def save(name, obj):
    with open(os.path.join(OUT, name), "w") as f:
        json.dump(obj, f, indent=1, sort_keys=True)
    print("wrote", name)


def determinism():
    exe = os.path.join(ROOT, "oracle", "_ref", "fp_determinism")
    txt = subprocess.check_output([exe]).decode()
    d = {}
    for line in txt.splitlines():
        if "=" in line:
            k, v = line.split("=", 1)
            d[k.strip()] = v.strip()
    save("determinism.json", d)


def matvec_cfg1(R):
    res = []
    for K, N in configs.CFG1_SHAPES:
        wn, xn = configs.matvec_names(K, N)
        w = orc.synth_weights(1, wn, (N, K))
        x = orc.synth_acts(1, xn, (K,))
        out = np.empty(N, dtype=np.int64)
        R.ref_matmul_vec(orc.p(out), orc.p(w), orc.p(x), N, K)
        res.append(dict(K=K, N=N, weight=wn, act=xn, w_hash=orc.fnv_hash(w), x_hash=orc.fnv_hash(x),
                        out_hash=orc.fnv_hash(out), out_head=[int(v) for v in out[:8]]))
    save("matvec_cfg1.json", res)


def tiny_model(R):
    c = configs.TINY_TEST
    w = helpers.model_weights(9, c)
    m = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    prompt = orc.synth_tokens(9, "prompt:0", 8, c["vocab"])
    # logits of every step, via llama_forward in generate's call order
    m.reset()
    toks = list(int(t) for t in prompt)
    lh = 1469598103934665603
    per_step = []
    for pos in range(len(prompt)):
        a, lg = m.forward(toks[pos], pos)
        lh = orc.O.iqo_fnv_array(lh, orc.p(lg), lg.size)
        per_step.append(orc.fnv_hash(lg))
    toks.append(a)
    max_new = 24
    for i in range(1, max_new):
        pos = len(prompt) + i - 1
        a, lg = m.forward(toks[pos], pos)
        lh = orc.O.iqo_fnv_array(lh, orc.p(lg), lg.size)
        per_step.append(orc.fnv_hash(lg))
        if a == 2:
            break
        toks.append(a)
    gen, _ = m.generate(prompt, max_new)
    assert gen == toks, (gen, toks)
    m.close()
    save("tiny_model.json", dict(config=c, cfg_index=9, prompt=[int(t) for t in prompt], max_new=max_new,
                                 tokens=toks, token_hash=orc.fnv_hash(np.array(toks)),
                                 logit_hash=lh, step_logit_hashes=per_step))


def ref_generate_hashed(m, prompt, max_new):
    """The reference's generate() loop (llama_int.c:3067-3135) run through its
    own llama_forward, hashing every forward's logits in call order."""
    m.reset()
    toks = [int(t) for t in prompt]
    lh = 1469598103934665603
    for pos in range(len(prompt)):
        a, lg = m.forward(toks[pos], pos)
        lh = orc.O.iqo_fnv_array(lh, orc.p(lg), lg.size)
    toks.append(a)
    for i in range(1, max_new):
        pos = len(prompt) + i - 1
        if pos >= m.c["max_seq"]:
            break
        a, lg = m.forward(toks[pos], pos)
        lh = orc.O.iqo_fnv_array(lh, orc.p(lg), lg.size)
        if a == 2:
            break
        toks.append(a)
    return toks, lh


def geom7b(R):
    c, ci = configs.GEOM7B_TEST, 10
    w = helpers.model_weights(ci, c)
    m = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    prompt = orc.synth_tokens(ci, "prompt:0", 370, c["vocab"])
    toks, lh = ref_generate_hashed(m, prompt, 30)
    gen, _ = m.generate(prompt, 30)
    assert gen == toks
    m.close()
    save("geom7b_model.json", dict(config=c, cfg_index=ci, prompt_len=370, prompt_name="prompt:0", max_new=30,
                                   tokens=toks[370:], logit_hash=lh,
                                   note="reference llama_forward, every logit of all 399 forwards hashed"))


_C3 = {}


def _cfg3_seq(b):
    R = orc.ref()
    c, ci = configs.CFG3_TEST, 11
    m = helpers.OracleModel(c, _C3["w"], lib=R, prefix="ref_")
    prompt = orc.synth_tokens(ci, f"prompt:{b}", _C3["plen"], c["vocab"])
    toks, lh = ref_generate_hashed(m, prompt, _C3["max_new"])
    m.close()
    return toks[_C3["plen"]:], lh


def cfg3(R):
    import multiprocessing as mp
    c, ci = configs.CFG3_TEST, 11
    _C3.update(w=helpers.model_weights(ci, c), plen=2080, max_new=24)
    B = 8
    t0 = time.time()
    with mp.get_context("fork").Pool(min(B, os.cpu_count() or 1)) as pool:
        res = pool.map(_cfg3_seq, range(B))
    print("cfg3 reference", time.time() - t0)
    save("cfg3_model.json", dict(config=c, cfg_index=ci, batch=B, prompt_len=2080, max_new=24,
                                 prompt_names=[f"prompt:{b}" for b in range(B)],
                                 tokens=[r[0] for r in res], logit_hashes=[r[1] for r in res],
                                 note="per sequence: the reference's llama_forward over the prompt and 23 "
                                      "decode steps (positions up to 2102), every logit hashed"))


def eos_weights():
    """TINY_TEST with one layer whose LM-head row 2 is set equal to the row of
    the token greedy decoding first emits at decode step 6 (t* > 2): from that
    step on, logits 2 and t* tie and the first-max rule picks 2 = EOS."""
    c, ci = dict(configs.TINY_TEST, n_layers=1), 12
    w = helpers.model_weights(ci, c)
    prompt = orc.synth_tokens(ci, "prompt:eos", 8, c["vocab"])
    return c, ci, w, prompt


def eos(R):
    c, ci, w, prompt = eos_weights()
    m = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    toks, _ = m.generate(prompt, 24)
    m.close()
    gen = toks[8:]
    k = next(i for i in range(6, len(gen)) if gen[i] > 2 and gen[i] not in gen[:i])
    w["lm_head"][2] = w["lm_head"][gen[k]]
    m = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    toks2, lh = ref_generate_hashed(m, prompt, 24)
    rt, _ = m.generate(prompt, 24)
    m.close()
    assert rt == toks2 and toks2 == toks[:8 + k], (rt, toks2, toks)
    save("eos_model.json", dict(config=c, cfg_index=ci, prompt=[int(t) for t in prompt], max_new=24,
                                lm_head_row2_from=int(gen[k]), tokens=toks2, n_out=len(toks2), logit_hash=lh,
                                note="reference generate() stops at EOS (llama_int.c:3110); the logit hash "
                                     "covers every forward up to and including the one that sampled 2"))


def cfg0_logits(R):
    """Config-0 logit hash from the reference's own forwards (31 decode + 8 prefill)."""
    c = configs.TINYLLAMA
    w = helpers.model_weights(0, c)
    mr = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    prompt = orc.synth_tokens(0, "prompt:0", 8, c["vocab"])
    t0 = time.time()
    toks, lh = ref_generate_hashed(mr, prompt, 32)
    print("reference forwards", time.time() - t0)
    mr.reset()
    a, lg = mr.forward(int(prompt[0]), 0)
    mr.close()
    old = json.load(open(os.path.join(OUT, "cfg0_tinyllama.json")))
    assert old["tokens"] == toks
    save("cfg0_tinyllama.json", dict(prompt=[int(t) for t in prompt], max_new=32, tokens=toks,
                                     token_hash=orc.fnv_hash(np.array(toks)), logit_hash=lh,
                                     first_step_logit_hash=orc.fnv_hash(lg),
                                     note="tokens and every-logit hash from the reference's own "
                                          "llama_forward, called in generate()'s order"))


SAMPLED = [dict(temperature=(1 << 48) * 4 // 5, top_k=40, top_p=(1 << 48) * 9 // 10, seed=42),
           dict(temperature=(1 << 48) * 3 // 2, top_k=0, top_p=(1 << 48) // 2, seed=7),
           dict(temperature=(1 << 48), top_k=5, top_p=1 << 48, seed=2026)]


def cfg0_sampled(R):
    """Config-0 model, 8-token prompt, 32 tokens drawn by the reference's own
    generate() with sampling parameters (sample_token, llama_int.c:2958-3039)."""
    c = configs.TINYLLAMA
    w = helpers.model_weights(0, c)
    mr = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    prompt = np.ascontiguousarray(orc.synth_tokens(0, "prompt:0", 8, c["vocab"]), dtype=np.int32)
    runs = []
    for sp in SAMPLED:
        t0 = time.time()
        out = np.zeros(8 + 32, np.int32)
        n = R.ref_model_generate_sampled(mr.h, orc.p(prompt), 8, 32, sp["temperature"], sp["top_k"], sp["top_p"],
                                         sp["seed"], orc.p(out))
        runs.append(dict(sp, tokens=[int(t) for t in out[:n]]))
        print("sampled run", time.time() - t0)
    mr.close()
    save("cfg0_sampled.json", dict(prompt=[int(t) for t in prompt], max_new=32, runs=runs,
                                   note="temperature / top_p in Q16.48; tokens from the reference's generate(sp)"))


def cfg2(R):
    res = []
    rows = configs.CFG2_ROWS
    for tag, K, N in configs.CFG2_SHAPES:
        wn, xn = configs.gemm_names(tag, K, N, rows)
        w = orc.synth_weights(2, wn, (N, K))
        X = orc.synth_acts(2, xn, (rows, K))
        out = np.empty((rows, N), dtype=np.int64)
        for r in range(rows):
            R.ref_matmul_vec_mt(orc.p(out[r]), orc.p(w), orc.p(X[r]), N, K, os.cpu_count())
        res.append(dict(tag=tag, K=K, N=N, rows=rows, weight=wn, act=xn, out_hash=orc.fnv_hash(out),
                        row_hashes=[orc.fnv_hash(out[r]) for r in range(0, rows, 64)]))
    save("gemm_cfg2.json", res)


if __name__ == "__main__":
    R = orc.ref()
    assert R is not None, "oracle/_ref not built (needs the reference checkout)"
    if "--fast" in sys.argv or not any(a.startswith("--") for a in sys.argv[1:]):
        determinism()
        matvec_cfg1(R)
        tiny_model(R)
    if "--cfg2" in sys.argv:
        cfg2(R)
    if "--cfg0" in sys.argv:
        cfg0_logits(R)
    if "--sampled" in sys.argv:
        cfg0_sampled(R)
    if "--geom7b" in sys.argv:
        geom7b(R)
    if "--eos" in sys.argv:
        eos(R)
    if "--cfg3" in sys.argv:
        cfg3(R)
