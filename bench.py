"""Benchmark: Q16.48 matvec microbench (config 1) on B200 through libiq.so.

A step = one pass of matmul_vec over the five config-1 shapes
(K x N = 2048x2048, 2048x256, 2048x5632, 5632x2048, 2048x32000), weights and
activations already resident in HBM (712 MiB of int64 weights per step: the
working set exceeds the 126 MB L2, so each shape is read cold from HBM).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: every rank runs the whole workload on its own GPU
(independent matvecs, no data-path collective: weak scaling); time is the max
over ranks. The same line carries two extra workloads: `cfg0_decode`
(TinyLlama greedy decode, output-row tensor parallel over the N ranks with
NCCL all-gathers) and, at N = 1, `cfg2_gemm` (the M=512 prefill GEMM), each
with its own roofline and CPU baseline. `--impl reference` times the reference's own CPU matmul_vec
(oracle/_ref, llama_int.c:1014) on the host cores, rows split across threads.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "int-llm_b200")]
import configs  # noqa: E402

METRIC = "Q16.48 matvec throughput, config 1 (M=1, 5 TinyLlama shapes), bit-exact"
UNIT = "GMAC/s"
SHAPES = configs.CFG1_SHAPES
MACS_PER_STEP = sum(K * N for K, N in SHAPES)
BYTES_PER_STEP = sum(8 * (K * N + K + N) for K, N in SHAPES)


def env_int(k, d):
    return int(os.environ.get(k, d))


def workload_config():
    return {"workload": "config1_matvec_M1",
            "shapes_KxN": [f"{K}x{N}" for K, N in SHAPES],
            "weights": "bf16-representable N(0,0.02) in Q16.48 (seeded)",
            "activations": "uniform [-8,8) Q16.48 (seeded)",
            "l2": "inputs larger than L2: every step streams all five packed matrices (283 MB at 3 "
                  "planes, 747 MB as int64) through the 126 MB L2",
            "parallelism": "independent replicas per GPU (weak scaling)"}


def synth_inputs(gen=None):
    """Seeded config-1 inputs. Our arm uses the library's own generator
    (iq_synth_*); the reference arm passes the oracle's C generator, which makes
    identical values (tests/test_abi.py) without loading libiq.so."""
    if gen is None:
        import iq as gen
    return [(gen.synth_weights(1, configs.matvec_names(K, N)[0], (N, K)),
             gen.synth_acts(1, configs.matvec_names(K, N)[1], (K,))) for K, N in SHAPES]


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    return orc


class Clocks:
    """nvidia-smi sampler running during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q,
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic():
    """ncu dram bytes (read + write) of one LM-head launch, from the committed
    summary of the profiled bench command (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get("lm_head_launch_bytes")
    except Exception:
        return None


# ------------------------------------------------------------------ CPU legs

def cpu_reference_lib():
    """The reference's own matmul_vec compiled from source (oracle/_ref), else
    the oracle's C restatement. Returns (callable(out,w,x,M,N,threads), kind)."""
    orc = _oracle()
    R = orc.ref()
    if R is not None:
        return (lambda o, w, x, M, N, t: R.ref_matmul_vec_mt(orc.p(o), orc.p(w), orc.p(x), M, N, t)), "reference"
    return (lambda o, w, x, M, N, t: orc.O.iqo_matmul_vec(orc.p(o), orc.p(w), orc.p(x), M, N)), "port"


def cpu_step(fn, ins, outs, threads):
    for (w, x), o, (K, N) in zip(ins, outs, SHAPES):
        fn(o, w, x, N, K, threads)


def cpu_baseline(ins, budget_s=10.0):
    """Single-thread reference matmul_vec over whole config-1 steps, ~budget_s."""
    fn, kind = cpu_reference_lib()
    outs = [np.empty(N, np.int64) for K, N in SHAPES]
    cpu_step(fn, ins, outs, 1)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        cpu_step(fn, ins, outs, 1)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": MACS_PER_STEP * n / dt / 1e9, "unit": UNIT, "cores": 1, "kind": kind,
            "sample": f"{n} whole config-1 steps ({MACS_PER_STEP} MAC each), single thread, "
                      f"{dt:.1f} s; host {os.cpu_count()} cpus"}


def run_reference(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    ins = synth_inputs(_oracle())
    fn, kind = cpu_reference_lib()
    threads = os.cpu_count() or 1
    outs = [np.empty(N, np.int64) for K, N in SHAPES]
    for _ in range(args.warmup):
        cpu_step(fn, ins, outs, threads)
    t0 = time.perf_counter()
    done = 0
    for _ in range(args.steps):   # bounded: stops early after 60 s of CPU work
        cpu_step(fn, ins, outs, threads)
        done += 1
        if time.perf_counter() - t0 > 60.0:
            break
    dt = time.perf_counter() - t0
    v = MACS_PER_STEP * done / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": done, "warmup": args.warmup, "ms_per_step": dt / done * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic", "config": workload_config(),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{args.steps} whole config-1 steps, rows split over {threads} threads"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ------------------------------------------------------------------ GPU leg

def _events(n):
    import torch
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def cfg1_leg(args, rank, world, local, dist):
    """Config 1 headline: one step = the five config-1 matvecs (one CUDA-graph
    replay), packed weights resident in HBM, every rank its own replica."""
    import torch
    import iq
    ins = synth_inputs()
    dev = [(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()) for w, x in ins]
    outs = [torch.empty(N, dtype=torch.int64, device="cuda") for K, N in SHAPES]
    s = torch.cuda.Stream()
    L = iq.lib()
    sp = ctypes.c_void_p(s.cuda_stream)
    # weights resident in HBM in the library's packed byte-plane form (a window
    # of byte planes, packed once before timing); IQ_BENCH_RAW=1 times the
    # CUDA-core kernel on the plain int64 matrices instead
    raw = os.environ.get("IQ_BENCH_RAW") == "1"
    packed = [iq.Packed(w, N, K) for (w, x), (K, N) in zip(dev, SHAPES)]
    torch.cuda.synchronize()
    ptrs = [(ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()), pk.h)
            for o, (w, x), pk in zip(outs, dev, packed)]
    # bytes one launch of each shape reads: the stored form, x and out
    shape_bytes = [(8 * K * N if raw else pk.nbytes()) + 8 * (K + N) for pk, (K, N) in zip(packed, SHAPES)]
    step_bytes = sum(shape_bytes)

    def launch(i):
        po, pw, px, pk = ptrs[i]
        K, N = SHAPES[i]
        rc = L.iq_matvec_dev(po, pw, px, N, K, sp) if raw else L.iq_matvec_packed_dev(po, pk, px, sp)
        if rc:
            raise iq.IQError("iq_matvec_dev", rc, L)

    def step():
        for i in range(len(SHAPES)):
            launch(i)

    with torch.cuda.stream(s):
        for _ in range(max(3, args.warmup)):
            step()
    torch.cuda.synchronize()

    # one step = one CUDA-graph replay of the 5 launches, so host launch overhead
    # never leaves the GPU idle inside the timed region
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step, stream=s, capture_error_mode="thread_local"):
        step()
    # per-shape graphs of R back-to-back launches: average launch duration of
    # each kernel with no per-replay gap (the LM head's 199 MB exceeds L2, so
    # each launch reads HBM; the small shapes are L2-resident in this form and
    # are reported for information only)
    R = 20
    g_shape = []
    for i in range(len(SHAPES)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            for _ in range(R):
                launch(i)
        g_shape.append(g)
    torch.cuda.synchronize()

    t_start, t_end = _events(2)
    clk = Clocks(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    time.sleep(0.3)
    with torch.cuda.stream(s):
        for _ in range(3):
            g_step.replay()
        t_start.record(s)
        for k in range(args.steps):
            g_step.replay()
        t_end.record(s)
    torch.cuda.synchronize()
    clocks = clk.stop()
    if dist:
        dist.barrier()
    ms_total = t_start.elapsed_time(t_end)
    reps = 5
    per_launch_ms = []
    with torch.cuda.stream(s):
        for i in range(len(SHAPES)):
            g_shape[i].replay()
            e0, e1 = _events(2)
            e0.record(s)
            for _ in range(reps):
                g_shape[i].replay()
            e1.record(s)
            torch.cuda.synchronize()
            per_launch_ms.append(e0.elapsed_time(e1) / (reps * R))
    ms_total = _max_over_ranks(dist, ms_total)
    per_launch_ms = [_max_over_ranks(dist, t) for t in per_launch_ms]

    # e2e: the public host-pointer drop-in iq_matmul_vec, pinned host buffers,
    # H2D of x and D2H of out inside the timed region every call
    hx = [torch.from_numpy(x).pin_memory().numpy() for w, x in ins]
    ho = [torch.empty(N, dtype=torch.int64).pin_memory().numpy() for K, N in SHAPES]
    for (w, x), (K, N) in zip(ins, SHAPES):
        iq.weight_register(w, N, K)
    e2e_steps = max(10, args.steps // 10)

    def e2e_step():
        for (w, x), hxx, hoo, (K, N) in zip(ins, hx, ho, SHAPES):
            iq.matmul_vec(hoo, w, hxx, N, K)
    for _ in range(3):
        e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    # the drop-in result must equal the device path's (same inputs)
    for o, hoo in zip(outs, ho):
        assert (o.cpu().numpy() == hoo).all(), "drop-in and device path disagree"
    iq.weight_cache_clear()

    peak, peak_kind = measured_peak()
    dom = len(SHAPES) - 1   # the 2048x32000 LM head: 69% of the step's bytes
    K, N = SHAPES[dom]
    ach = shape_bytes[dom] / (per_launch_ms[dom] / 1e3) / 1e9
    step_gbs = step_bytes * args.steps / (ms_total / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": MACS_PER_STEP * args.steps * world / (ms_total / 1e3) / 1e9,
        "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int64", "data": "synthetic", "config": workload_config(),
        "roofline": {
            "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)",
            "kernel": ("k_matvec" if raw else "k_matvec_planes") + f" {K}x{N} (LM head)",
            "bytes_per_launch": shape_bytes[dom], "launch_ms": per_launch_ms[dom],
            "traffic": load_traffic(),
            "note": "achieved = bytes of the stored form one launch reads (iq_packed_bytes: byte-plane "
                    "window + row sums + sparse residual, plus x and out) / average launch duration "
                    "(CUDA events around 100 back-to-back launches); traffic = ncu dram bytes of one "
                    "launch (profiles/); the int64 form the reference streams is 8 B/weight "
                    "(int64_equiv_gbs)"},
        "step_roofline": {"bytes_per_step": step_bytes, "gbs": step_gbs, "frac": step_gbs / peak,
                          "int64_equiv_gbs": BYTES_PER_STEP * args.steps / (ms_total / 1e3) / 1e9},
        "per_launch_us": {f"{K}x{N}": t * 1e3 for (K, N), t in zip(SHAPES, per_launch_ms)},
        "planes_stored": None if raw else {f"{K}x{N}": list(pk.info()) for pk, (K, N) in zip(packed, SHAPES)},
        "e2e": {"value": MACS_PER_STEP * e2e_steps * world / e2e_s / 1e9, "unit": UNIT,
                "h2d_bytes_per_step": sum(8 * K for K, N in SHAPES),
                "d2h_bytes_per_step": sum(8 * N for K, N in SHAPES),
                "api": "iq_matmul_vec (host pointers, weights registered)"},
        "gpu_launches": args.steps * len(SHAPES),
        "clocks": clocks,
    }
    for pk in packed:
        pk.free()
    del dev, outs
    torch.cuda.empty_cache()
    if world == 1 and rank == 0 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(ins)
    return line


def cpu_baseline_cfg0(budget_s=8.0):
    """The reference's own llama_forward (oracle/_ref) on 1 core at TinyLlama
    shape. Bounded sample: the 22 layers share layer 0's seeded weights (same
    work per token as 22 distinct layers; 0.38 GB instead of 8.3 GB of host
    weights to generate), forwards at positions 0, 1, 2, ... for ~budget_s."""
    orc = _oracle()
    R = orc.ref()
    if R is None:
        return None
    c = configs.TINYLLAMA
    d, V = c["dim"], c["vocab"]
    one = np.full(d, 1 << 48, dtype=np.int64)
    lay = [one if len(sh) == 1 else orc.synth_weights(0, configs.layer_name(0, t), sh)
           for t, sh in zip(configs.LAYER_TENSORS, configs.layer_shapes(c))]
    emb = orc.synth_weights(0, "model.embed_tokens.weight", (V, d))
    lm = orc.synth_weights(0, "lm_head.weight", (V, d))
    fn = np.full(d, 1 << 48, dtype=np.int64)
    ptrs = (ctypes.c_void_p * (9 * c["n_layers"]))(*([a.ctypes.data for a in lay] * c["n_layers"]))
    cfg9 = (ctypes.c_int * 9)(*configs.cfg9(c))
    h = R.ref_model_create(cfg9, orc.p(emb), orc.p(fn), orc.p(lm), ptrs)
    toks = orc.synth_tokens(0, "prompt:0", 64, V)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s and n < 64:
        R.ref_model_forward(h, int(toks[n]), n, None)
        n += 1
    dt = time.perf_counter() - t0
    R.ref_model_free(h)
    return {"value": n / dt, "unit": "tokens/s", "cores": 1, "kind": "reference",
            "sample": f"{n} reference llama_forward calls (positions 0..{n - 1}) at TinyLlama shape, "
                      f"22 layers sharing layer 0's weights, single thread, {dt:.1f} s"}


def cfg0_leg(args, rank, world, local, dist, nid):
    """Config 0: TinyLlama greedy decode at batch 1, output-row tensor
    parallelism over the ranks (NCCL all-gathers) when world > 1."""
    import iq
    c = configs.TINYLLAMA
    t0 = time.perf_counter()
    m = iq.Model(c, device=local, tp_rank=rank, tp_size=world, nccl_id=nid)
    m.synth(0, threads=max(1, (os.cpu_count() or 1) // world))
    t_load = time.perf_counter() - t0
    prompt = iq.synth_tokens(0, "prompt:0", 8, c["vocab"])
    m.generate(prompt, 32)   # first use (graphs, NCCL connections); fills the cache to pos 38
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    toks, _ = m.generate(prompt, 32)
    e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    pos0, dec = 39, 64
    m.decode_steps_timed(pos0, 3)
    ms = _max_over_ranks(dist, m.decode_steps_timed(pos0, dec))
    wb, _ = m.weight_bytes()
    sh = iq.tp_shard_info(c, world, rank)
    kv_bytes = 8 * 2 * c["n_layers"] * sh["nkv"] * c["head_dim"] * (pos0 + 1 + dec / 2)
    step_s = ms / 1e3 / dec
    peak, peak_kind = measured_peak()
    ach = (wb + kv_bytes) / step_s / 1e9
    m.close()
    out = {"metric": "TinyLlama greedy decode tokens/s (B=1), bit-exact", "value": dec / (ms / 1e3),
           "unit": "tokens/s", "ms_per_token": ms / dec, "n_gpus": world,
           "parallelism": f"tp{world}", "decode_positions": f"{pos0}..{pos0 + dec - 1}", "load_s": t_load,
           "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                        "peak_source": peak_kind, "kernel": "whole decode step (per GPU)",
                        "bytes_per_token_per_gpu": wb + kv_bytes,
                        "note": "stored-form weight bytes of every matvec + LM head "
                                "(iq_model_weight_bytes) + KV reads, per token per GPU"},
           "e2e": {"value": (len(toks) - len(prompt)) / e2e_s, "unit": "tokens/s",
                   "h2d_bytes_per_step": 4 * len(prompt), "d2h_bytes_per_step": 4 * len(toks),
                   "api": "iq_generate (8-token prompt + 32 greedy tokens per call, prefill included)"}}
    if world == 1 and rank == 0 and not args.no_cpu:
        out["cpu_baseline"] = cpu_baseline_cfg0()
    return out


def cpu_baseline_cfg2(budget_s=6.0):
    """Config 2 on the CPU: rows of the reference's own matmul_vec, 1 core."""
    orc = _oracle()
    fn, kind = cpu_reference_lib()
    rows = configs.CFG2_ROWS
    mac, tt, desc = 0, 0.0, []
    for tag, K, N in configs.CFG2_SHAPES:
        wn, xn = configs.gemm_names(tag, K, N, rows)
        w = orc.synth_weights(2, wn, (N, K))
        X = orc.synth_acts(2, xn, (8, K))
        o = np.empty(N, np.int64)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s / 4 and n < 8:
            fn(o, w, X[n], N, K, 1)
            n += 1
        tt += time.perf_counter() - t0
        mac += n * K * N
        desc.append(f"{tag}:{n}")
    return {"value": mac / tt / 1e9, "unit": "GMAC/s", "cores": 1, "kind": kind,
            "sample": "rows of X through matmul_vec, single thread (" + ", ".join(desc) + f"), {tt:.1f} s"}


def cfg2_leg(args):
    """Config 2: M=512 prefill GEMM on the fused TinyLlama projections
    (tcgen05 kind::i8 byte planes), one GPU."""
    import torch
    import iq
    rows = configs.CFG2_ROWS
    s = torch.cuda.Stream()
    per, tot_mac, tot_ms, i8_ops = {}, 0, 0.0, 0
    for tag, K, N in configs.CFG2_SHAPES:
        wn, xn = configs.gemm_names(tag, K, N, rows)
        w = torch.from_numpy(iq.synth_weights(2, wn, (N, K))).cuda()
        X = torch.from_numpy(iq.synth_acts(2, xn, (rows, K))).cuda()
        pk = iq.PackedTC(w, N, K)
        npl = pk.info()[0]
        out = torch.empty((rows, N), dtype=torch.int64, device="cuda")
        reps = 20
        with torch.cuda.stream(s):
            for _ in range(3):
                iq.gemm_tc_dev(out, pk, X, rows, stream=s)
            e0, e1 = _events(2)
            e0.record(s)
            for _ in range(reps):
                iq.gemm_tc_dev(out, pk, X, rows, stream=s)
            e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        macs = rows * K * N
        # int8 tensor work: every Q16.48 MAC is npl weight planes x 8 activation digits
        ops = 2 * macs * npl * 8
        per[tag] = {"K": K, "N": N, "ms": ms, "gmacs": macs / ms / 1e6, "planes": npl,
                    "int8_tops": ops / ms / 1e9}
        tot_mac += macs
        tot_ms += ms
        i8_ops += ops
        pk.free()
        del w, X, out
    torch.cuda.empty_cache()
    peak_tops, _ = iq.bench_i8_peak(20000)   # measured now, on this GPU
    tops = i8_ops / tot_ms / 1e9
    out = {"metric": "Q16.48 prefill GEMM GMAC/s, config 2 (M=512, 4 fused TinyLlama projections), bit-exact",
           "value": tot_mac / tot_ms / 1e6, "unit": "GMAC/s", "n_gpus": 1, "per_shape": per,
           "roofline": {"bound": "tensor", "achieved": tops, "unit": "int8 TOP/s", "peak": peak_tops,
                        "frac": tops / peak_tops,
                        "peak_source": "measured in this run: iq_bench_i8_peak (tcgen05.mma kind::i8, "
                                       "M128 N256 K32 from shared memory, one CTA per SM)",
                        "kernel": "k_gemm_tc (all four shapes)",
                        "note": "achieved = int8 MACs the byte-plane identity needs (planes x 8 digits per "
                                "Q16.48 MAC) x 2 / GEMM time"}}
    if not args.no_cpu:
        out["cpu_baseline"] = cpu_baseline_cfg2()
    return out


def run_ours(args):
    import torch
    import iq
    rank, world, local, dist, nid = _tp_setup()
    line = cfg1_leg(args, rank, world, local, dist)
    if not args.headline_only:
        line["cfg0_decode"] = cfg0_leg(args, rank, world, local, dist, nid)
        torch.cuda.empty_cache()
        if world == 1:
            line["cfg2_gemm"] = cfg2_leg(args)
    if rank == 0:
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------- model workloads

def _tp_setup():
    """rank / world / local from torchrun, NCCL id shared from rank 0."""
    import torch
    import iq
    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    iq.set_device(local)
    dist, nid = None, None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        obj = [iq.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    return rank, world, local, dist, nid


def _max_over_ranks(dist, v):
    import torch
    if not dist:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def run_model_workload(args):
    """cfg0: TinyLlama greedy decode (B=1); cfg3: batch-64 decode after 2048-token
    prefills; cfg4: Llama-2-7B shape, 2048-token prefill + 64 decode tokens.
    N > 1: output-row tensor parallelism over the ranks (NCCL all-gathers)."""
    import torch
    import iq
    rank, world, local, dist, nid = _tp_setup()
    wl = args.workload
    if wl == "cfg0":
        cfg, ci, B, plen, dec, pos0 = dict(configs.TINYLLAMA), 0, 1, 8, max(args.steps, 32), 40
    elif wl == "cfg3":
        cfg, ci, B, plen, dec, pos0 = dict(configs.TINYLLAMA, max_seq=2176), 3, 64, 2048, 128, 2048
    else:
        cfg, ci, B, plen, dec, pos0 = dict(configs.LLAMA7B), 4, 1, 2048, 64, 2048
    t0 = time.perf_counter()
    m = iq.Model(cfg, max_batch=B, device=local, tp_rank=rank, tp_size=world, nccl_id=nid)
    m.synth(ci, threads=max(1, (os.cpu_count() or 1) // world))
    t_load = time.perf_counter() - t0
    prompts = np.stack([iq.synth_tokens(ci, f"prompt:{b}", plen, cfg["vocab"]) for b in range(B)])
    # e2e through the public API: prefill (+ first token) from host prompts.
    # B == 1: one untimed call first (a prompt of up to one 1024-row prefill
    # chunk), so the timed call does not pay first-use costs (NCCL connection
    # set-up, scratch growth); B > 1 prefills 64 x 2048 tokens, which amortise them.
    if B == 1:
        m.generate(prompts[0][:min(plen, 1040)], 1)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if B == 1:
        toks, _ = m.generate(prompts[0], 1)
    else:
        outs = m.generate_batch(prompts, 1)
    t_prefill = _max_over_ranks(dist, time.perf_counter() - t0)
    # decode: graph replays of the whole step (all B sequences), device-timed
    m.decode_steps_timed(pos0, 3)
    clk = Clocks(local)
    clk.start()
    time.sleep(0.2)
    ms = m.decode_steps_timed(pos0, dec)
    clocks = clk.stop()
    ms = _max_over_ranks(dist, ms)
    if getattr(args, "profile_step", False):
        # one decode step inside a profiler range (ncu --profile-from-start off)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        m.decode_steps_timed(pos0, 1)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    # e2e decode through generate(): prompt in, tokens out (host buffers)
    e2e = None
    if wl == "cfg0":
        t0 = time.perf_counter()
        toks, _ = m.generate(prompts[0], 32)
        e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
        e2e = {"value": (len(toks) - plen) / e2e_s, "unit": "tokens/s",
               "h2d_bytes_per_step": 4 * plen, "d2h_bytes_per_step": 4 * (plen + 32),
               "api": "iq_generate (8-token prompt + 32 greedy tokens, per call)"}
    tok_s = B * dec / (ms / 1e3)
    d, L, V, it = cfg["dim"], cfg["n_layers"], cfg["vocab"], cfg["inter"]
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    wbytes, _ = m.weight_bytes()   # this rank's packed weight bytes read per decode step
    kv_bytes = 8 * 2 * L * kvd * (pos0 + dec / 2) * B / world
    peak, peak_kind = measured_peak()
    step_s = ms / 1e3 / dec
    ach = (wbytes + kv_bytes) / step_s / 1e9  # per GPU
    line = {
        "metric": {"cfg0": "TinyLlama greedy decode tokens/s (B=1), bit-exact",
                   "cfg3": "TinyLlama batch-64 decode tokens/s after 2048-token prefills, bit-exact",
                   "cfg4": "Llama-2-7B-shape decode tokens/s after a 2048-token prefill, bit-exact"}[wl],
        "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": dec, "warmup": 3,
        "ms_per_step": ms / dec, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int64", "data": "synthetic", "config": {"workload": wl, "batch": B, "prompt": plen,
                                                          "decode_from_pos": pos0,
                                                          "parallelism": f"tp{world}"},
        "prefill_s": t_prefill, "prefill_tokens_per_s": B * plen / t_prefill, "load_s": t_load,
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                     "peak_source": peak_kind, "kernel": "decode step (all kernels)",
                     "bytes_per_step_per_gpu": wbytes + kv_bytes,
                     "bytes_note": "packed weight bytes (iq_model_weight_bytes) + int64 KV reads",
                     "traffic": None},
        "gpu_launches": None, "clocks": clocks,
    }
    if e2e:
        line["e2e"] = e2e
    if rank == 0:
        print(json.dumps(line))
    m.close()
    if dist:
        dist.destroy_process_group()


def run_gemm_workload(args):
    """cfg2: M=512 prefill GEMM on the fused TinyLlama projections (tcgen05)."""
    import torch
    import iq
    torch.cuda.set_device(0)
    rows = configs.CFG2_ROWS
    s = torch.cuda.Stream()
    per, tot_mac, tot_ms = {}, 0, 0.0
    for tag, K, N in configs.CFG2_SHAPES:
        wn, xn = configs.gemm_names(tag, K, N, rows)
        w = torch.from_numpy(iq.synth_weights(2, wn, (N, K))).cuda()
        X = torch.from_numpy(iq.synth_acts(2, xn, (rows, K))).cuda()
        pk = iq.PackedTC(w, N, K)
        out = torch.empty((rows, N), dtype=torch.int64, device="cuda")
        reps = max(10, args.steps // 100)
        with torch.cuda.stream(s):
            for _ in range(args.warmup):
                iq.gemm_tc_dev(out, pk, X, rows, stream=s)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                iq.gemm_tc_dev(out, pk, X, rows, stream=s)
            e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        macs = rows * K * N
        per[tag] = {"K": K, "N": N, "ms": ms, "gmacs": macs / ms / 1e6, "int8_tops": 128 * macs / ms / 1e9}
        tot_mac += macs
        tot_ms += ms
        pk.free()
    print(json.dumps({"metric": "Q16.48 prefill GEMM GMAC/s, config 2 (M=512), bit-exact", "value": tot_mac / tot_ms / 1e6,
                      "unit": "GMAC/s", "n_gpus": 1, "higher_is_better": True, "dtype": "int64",
                      "data": "synthetic", "config": {"workload": "cfg2", "rows": rows}, "per_shape": per}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--headline-only", action="store_true",
                    help="config 1 only (no config-0 decode / config-2 GEMM extras)")
    ap.add_argument("--profile-step", action="store_true",
                    help="model workloads: run one extra decode step inside cudaProfilerStart/Stop")
    ap.add_argument("--workload", default="cfg1", choices=["cfg1", "cfg0", "cfg2", "cfg3", "cfg4"],
                    help="cfg1 (default, the headline): M=1 matvec microbench")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg1":
        run_ours(args)
    elif args.workload == "cfg2":
        run_gemm_workload(args)
    else:
        run_model_workload(args)


if __name__ == "__main__":
    main()
