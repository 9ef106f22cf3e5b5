"""Tensor-parallel host logic on CPU: two gloo ranks each compute the output
rows they own (iq_tp_shard_info) of every projection with the oracle, all-gather
them, and must reproduce the unsharded result bit for bit; the row ownership
must partition every projection exactly."""
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import configs
import iq
import oracle as orc


def _ranges(c, P, r):
    s = iq.tp_shard_info(c, P, r)
    hd = c["head_dim"]
    return {
        "q": (s["q_lo"] * hd, s["nh"] * hd), "k": (s["kv_lo"] * hd, s["nkv"] * hd),
        "o": (s["d_lo"], s["d_n"]), "gate": (s["it_lo"], s["it_n"]), "down": (s["d_lo"], s["d_n"]),
        "lm": (r * c["vocab"] // P, c["vocab"] // P),
    }


@pytest.mark.parametrize("P", [1, 2, 4, 8])
@pytest.mark.parametrize("cfg", ["TINYLLAMA", "LLAMA7B"])
def test_row_ownership_partitions(P, cfg):
    c = getattr(configs, cfg)
    hd, grp = c["head_dim"], c["n_heads"] // c["n_kv_heads"]
    seen = {k: [] for k in ("q", "o", "gate", "lm")}
    for r in range(P):
        rg = _ranges(c, P, r)
        for k in seen:
            seen[k].append(rg[k])
        # every local q head's kv head is local
        s = iq.tp_shard_info(c, P, r)
        for h in range(s["q_lo"], s["q_lo"] + s["nh"]):
            assert s["kv_lo"] <= h // grp < s["kv_lo"] + s["nkv"]
    totals = {"q": c["dim"], "o": c["dim"], "gate": c["inter"], "lm": c["vocab"]}
    for k, parts in seen.items():
        pos = 0
        for lo, n in parts:
            assert lo == pos
            pos += n
        assert pos == totals[k]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = dict(configs.TINY_TEST)
    d = c["dim"]
    rng = np.random.default_rng(5)
    x = rng.integers(-8 << 48, 8 << 48, d).astype(np.int64)
    ok = True
    for name, rows in (("q", d), ("o", d), ("gate", c["inter"]), ("lm", c["vocab"])):
        W = orc.synth_weights(9, f"w:tp:{name}", (rows, d))
        full = orc.matmul_vec(W, x)
        lo, n = _ranges(c, world, rank)[name]
        mine = torch.from_numpy(orc.matmul_vec(np.ascontiguousarray(W[lo:lo + n]), x))
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        ok &= bool((torch.cat(parts).numpy() == full).all())
    # global first-max argmax from per-rank (value, index) pairs
    lg = orc.synth_acts(9, "x:tp:logits", (c["vocab"],))
    lg[[7, 300]] = lg.max() + 5            # a tie across ranks: the lower index wins
    lo, n = _ranges(c, world, rank)["lm"]
    loc = lg[lo:lo + n]
    pair = torch.tensor([int(loc.max()), lo + int(np.argmax(loc))], dtype=torch.int64)
    pairs = [torch.empty_like(pair) for _ in range(world)]
    dist.all_gather(pairs, pair)
    best = max(pairs, key=lambda t: (int(t[0]), -int(t[1])))
    ok &= int(best[1]) == int(np.argmax(lg)) == 7
    q.put((rank, ok))
    dist.destroy_process_group()


def test_gloo_two_ranks_reassemble_projections():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
