"""Generates the committed golden fixtures from the REFERENCE itself.

Run in a container where the reference checkout exists and oracle/_ref is built
(`make -C oracle`). Every value here comes from the reference's own code
compiled from source (oracle/_ref/libllamaref.so, oracle/_ref/fp_determinism);
the C restatement (oracle/libiqoracle.so) is only used for the synthetic
inputs, whose generator is cross-checked against the reference's bf16 decoder.

  python tests/golden/make_golden.py            # fast fixtures
  python tests/golden/make_golden.py --cfg0     # + TinyLlama greedy decode (minutes)
  python tests/golden/make_golden.py --cfg2     # + M=512 GEMM hashes
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


def cfg0(R):
    c = configs.TINYLLAMA
    t0 = time.time()
    w = helpers.model_weights(0, c)
    print("weights", time.time() - t0)
    m = helpers.OracleModel(c, w, lib=orc.O, prefix="iqo_")  # restatement: threaded
    prompt = orc.synth_tokens(0, "prompt:0", 8, c["vocab"])
    toks, lh = m.generate(prompt, 32)
    print("restatement generate", time.time() - t0)
    m.close()
    mr = helpers.OracleModel(c, w, lib=R, prefix="ref_")
    rtoks, _ = mr.generate(prompt, 32)
    print("reference generate", time.time() - t0)
    assert rtoks == toks, (rtoks, toks)
    # one reference forward's full logits pin the logit hash of the first step
    mr.reset()
    a, lg = mr.forward(int(prompt[0]), 0)
    mr.close()
    save("cfg0_tinyllama.json", dict(prompt=[int(t) for t in prompt], max_new=32, tokens=toks,
                                     token_hash=orc.fnv_hash(np.array(toks)), logit_hash=lh,
                                     first_step_logit_hash=orc.fnv_hash(lg),
                                     note="tokens from the reference generate(); logit_hash from the "
                                          "restatement, whose tokens and first-step logits equal the reference's"))


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
    determinism()
    matvec_cfg1(R)
    tiny_model(R)
    if "--cfg2" in sys.argv:
        cfg2(R)
    if "--cfg0" in sys.argv:
        cfg0(R)
