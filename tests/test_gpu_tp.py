"""Tensor-parallel model on 2 GPUs (one process per GPU, NCCL): tokens and the
hash of every logit equal the single-GPU reference goldens, and batched decode
equals the unsharded model. Skipped when fewer than 2 GPUs are visible."""
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


def _rank(rank, world, ids, q):
    import faulthandler
    faulthandler.enable()                                # a crash prints its stack too
    faulthandler.dump_traceback_later(150, exit=False)   # names the call if anything blocks
    import torch
    torch.cuda.set_device(rank)
    try:
        g = json.load(open(os.path.join(GOLD, "tiny_model.json")))
        c = g["config"]
        w = helpers.model_weights(g["cfg_index"], c)
        m = iq.Model(c, device=rank, tp_rank=rank, tp_size=world, nccl_id=ids[0])
        m.load(w)
        toks, lh = m.generate(np.array(g["prompt"]), g["max_new"], logit_hash=True)
        toks2, _ = m.generate(np.array(g["prompt"]), g["max_new"])   # graph replays, no host sync
        a, lg = m.forward(int(g["prompt"][0]), 0)
        ok = toks == g["tokens"] and lh == g["logit_hash"] and toks2 == g["tokens"]
        ok = ok and orc.fnv_hash(lg) == g["step_logit_hashes"][0]
        m.close()
        # batched decode (B = 3): every sequence equals the unsharded model's
        cb = dict(c, max_seq=48)
        mb = iq.Model(cb, max_batch=3, device=rank, tp_rank=rank, tp_size=world, nccl_id=ids[1])
        mb.load(w)
        prompts = np.stack([orc.synth_tokens(9, f"prompt:tp{b}", 6, c["vocab"]) for b in range(3)])
        got = mb.generate_batch(prompts, 20)
        mb.close()
        m1 = iq.Model(cb, device=rank)
        m1.load(w)
        for b in range(3):
            want, _ = m1.generate(prompts[b], 20)
            ok = ok and got[b] == want
        m1.close()
        q.put((rank, bool(ok), None))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, repr(e)))


def test_tp2_generate_matches_goldens():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ids = [iq.nccl_unique_id(), iq.nccl_unique_id()]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, ids, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, ok, err = q.get(timeout=240)
            res[r] = (ok, err)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert res == {0: (True, None), 1: (True, None)}, res


def _rank_leave(rank, world, nid, q, gone):
    """Rank 1 finishes one generate and leaves between steps (no collective in
    flight) after marking itself gone in a host-side store (an Event); rank 0
    learns of it from its peer check before its next launch, so its generate
    returns IQ_ERR_NCCL having posted no collective, and the model then refuses
    work (IQ_ERR_STATE)."""
    import faulthandler
    faulthandler.enable()                                # a crash prints its stack too
    faulthandler.dump_traceback_later(200, exit=False)   # names the call if anything blocks
    import sys
    import time
    import torch
    torch.cuda.set_device(rank)
    t0 = time.time()

    def note(what):
        print(f"[rank {rank} +{time.time() - t0:.1f}s] {what}", file=sys.stderr, flush=True)
    try:
        g = json.load(open(os.path.join(GOLD, "tiny_model.json")))
        c = g["config"]
        w = helpers.model_weights(g["cfg_index"], c)
        m = iq.Model(c, device=rank, tp_rank=rank, tp_size=world, nccl_id=nid)
        m.load(w)
        toks, _ = m.generate(np.array(g["prompt"]), 8)
        if rank == 1:
            q.put((rank, toks == g["tokens"][:len(toks)], "left"))
            q.close()
            q.join_thread()   # the message is in the pipe and the queue's lock released before _exit
            gone.set()
            os._exit(0)   # leaves without destroying its communicator
        m.set_timeout(3000)
        m.set_peer_check(gone.is_set)
        gone.wait(60)
        note("peer gone; generate")
        try:
            m.generate(np.array(g["prompt"]), 8)
            status = 0
        except iq.IQError as e:
            status = e.status
        note(f"generate returned {status}")
        try:
            m.generate(np.array(g["prompt"]), 8)
            after = 0
        except iq.IQError as e:
            after = e.status
        note(f"second generate returned {after}")
        q.put((rank, status == -4 and after == -7, (status, after)))   # IQ_ERR_NCCL, IQ_ERR_STATE
        try:   # a failed model's destroy is bounded too (IQ_ERR_TIMEOUT if the stream never drains)
            m.close()
        except iq.IQError as e:
            note(f"close returned {e.status}")
        note("closed")
    except Exception as e:
        q.put((rank, False, repr(e)))


def test_tp2_peer_leaving_between_steps_fails_cleanly():
    """Failure detection without a GPU fault: a rank leaves between steps, the
    surviving rank learns of it on the host before its next launch (the peer
    check), its call returns IQ_ERR_NCCL without posting a collective, and the
    model refuses further work (IQ_ERR_STATE). NVLS is off in both ranks."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    nid = iq.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    gone = ctx.Event()
    procs = [ctx.Process(target=_rank_leave, args=(r, 2, nid, q, gone)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, ok, info = q.get(timeout=240)
            res[r] = (ok, info)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert res[1][0] and res[0][0], res
