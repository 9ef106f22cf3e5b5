"""GPU parity tests: every kernel, through the C ABI, bit-exact against the
oracle (C restatement) on the same seeded inputs, plus the reference goldens."""
import ctypes
import json
import os

import numpy as np
import pytest

import configs
import iq
import oracle as orc

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
ONE = 1 << 48


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rand_full(rng, shape):
    return rng.integers(-2 ** 63, 2 ** 63 - 1, shape, dtype=np.int64)


# ------------------------------------------------------------------ matvec

@pytest.mark.parametrize("M,N", [(1, 1), (1, 2), (3, 17), (5, 64), (7, 65), (64, 1000), (33, 2048),
                                 (1000, 63), (129, 4097), (17, 40000)])
@pytest.mark.parametrize("dist", ["full", "cfg"])
def test_matvec_dev_edges(M, N, dist):
    import torch
    rng = np.random.default_rng(M * 7919 + N)
    if dist == "full":
        w, x = rand_full(rng, (M, N)), rand_full(rng, (N,))
    else:
        w = orc.synth_weights(1, f"w:{M}x{N}", (M, N))
        x = orc.synth_acts(1, f"x:{M}x{N}", (N,))
    want = orc.matmul_vec(w, x)
    dw, dx = dev(w), dev(x)
    do = torch.empty(M, dtype=torch.int64, device="cuda")
    iq.matvec_dev(do, dw, dx, M, N)
    assert (host(do) == want).all()


def test_matvec_unaligned_weight_pointer():
    """A weight base that is 8- but not 16-byte aligned takes the scalar-load path."""
    import torch
    rng = np.random.default_rng(5)
    M, N = 37, 300
    w, x = rand_full(rng, (M, N)), rand_full(rng, (N,))
    buf = dev(np.concatenate([np.zeros(1, np.int64), w.ravel()]))
    dx = dev(x)
    do = torch.empty(M, dtype=torch.int64, device="cuda")
    lib = iq.lib()
    rc = lib.iq_matvec_dev(ctypes.c_void_p(do.data_ptr()), ctypes.c_void_p(buf.data_ptr() + 8),
                           ctypes.c_void_p(dx.data_ptr()), M, N, None)
    assert rc == 0
    assert (host(do) == orc.matmul_vec(w, x)).all()


def test_matvec_cfg1_golden_and_dropin():
    """Config-1 shapes through the drop-in matmul_vec(out, weight, in, M, N) on host
    pointers, checked against the reference's own outputs (golden hash)."""
    for g in json.load(open(os.path.join(GOLD, "matvec_cfg1.json"))):
        K, N = g["K"], g["N"]
        w = orc.synth_weights(1, g["weight"], (N, K))
        x = orc.synth_acts(1, g["act"], (K,))
        out = np.empty(N, dtype=np.int64)
        iq.matmul_vec(out, w, x, N, K)
        assert orc.fnv_hash(out) == g["out_hash"], (K, N)
        out2 = np.zeros(N, dtype=np.int64)
        iq.matmul_vec(out2, w, x, N, K)   # second call: cached weights
        assert (out2 == out).all()
        iq.weight_unregister(w)


def test_dropin_weight_cache_rekeys_on_shape():
    rng = np.random.default_rng(11)
    w = rand_full(rng, (64 * 64,))
    x = rand_full(rng, (64,))
    o1 = np.empty(64, np.int64)
    iq.matmul_vec(o1, w, x, 64, 64)
    assert (o1 == orc.matmul_vec(w.reshape(64, 64), x)).all()
    o2 = np.empty(128, np.int64)
    iq.matmul_vec(o2, w, x[:32].copy(), 128, 32)   # same pointer, new shape
    assert (o2 == orc.matmul_vec(w.reshape(128, 32), x[:32].copy())).all()
    iq.weight_cache_clear()


# ------------------------------------------------------------------ gemm

@pytest.mark.parametrize("rows,M,N", [(2, 5, 7), (31, 64, 129), (33, 65, 1000), (64, 256, 2048),
                                      (100, 300, 5632)])
def test_gemm_dev_vs_oracle(rows, M, N):
    import torch
    rng = np.random.default_rng(rows + M + N)
    w, X = rand_full(rng, (M, N)), rand_full(rng, (rows, N))
    want = orc.matmul_rows(w, X)
    do = torch.empty((rows, M), dtype=torch.int64, device="cuda")
    iq.gemm_dev(do, dev(w), dev(X), rows, M, N)
    assert (host(do) == want).all()


# ------------------------------------------------------------------ fp_math

def det_grid():
    """The determinism gate's input grid (fp_determinism.c:101-137)."""
    g = [0, ONE, -ONE, ONE // 2, -(ONE // 2), 1, -1, ONE + 1, ONE - 1, 32000 * ONE, -32000 * ONE,
         181 * ONE, 7 * ONE, -7 * ONE, 2 * ONE, 10 * ONE]
    for e in range(-44, 15):
        p = ONE << e if e >= 0 else ONE >> -e
        g += [p, -p]
    st = 0x9E3779B97F4A7C15
    M64 = (1 << 64) - 1
    span = 32000 * ONE
    for _ in range(4096):
        st ^= (st << 13) & M64
        st ^= st >> 7
        st ^= (st << 17) & M64
        mag = st % span
        g.append(mag if st & 1 else -mag)
    return np.array(g, dtype=np.int64)


def test_fp_ports_reproduce_determinism_subhashes():
    """Device ports of fp_mul/div/sqrt/sqrt_fast/inv_sqrt/exp/log/sincos/sigmoid/silu
    over the gate's grid give the reference's golden sub-hashes."""
    import torch
    gd = json.load(open(os.path.join(GOLD, "determinism.json")))
    g = det_grid()
    n = len(g)
    assert n == 4230
    y = g[(np.arange(n) * 7 + 3) % n]
    xp = np.abs(g)
    xp = np.where(xp < 1024, xp + 1024, xp)
    forty, twenty = 40 * ONE, 20 * ONE
    ea = (g.view(np.uint64) % np.uint64(forty)).astype(np.int64) - twenty

    def run(fn, x, yy=None):
        do = torch.empty(len(x), dtype=torch.int64, device="cuda")
        iq.fp_dev(fn, dev(x), dev(yy) if yy is not None else None, do, len(x))
        return host(do)

    assert f"{orc.fnv_hash(run('mul', g, y)):016x}" == gd["sub:fp_mul"]
    nz = y != 0
    assert f"{orc.fnv_hash(run('div', g[nz], y[nz])):016x}" == gd["sub:fp_div"]
    assert f"{orc.fnv_hash(run('sqrt', xp)):016x}" == gd["sub:fp_sqrt"]
    assert f"{orc.fnv_hash(run('sqrt_fast', xp)):016x}" == gd["sub:fp_sqrt_fast"]
    assert f"{orc.fnv_hash(run('inv_sqrt', xp)):016x}" == gd["sub:fp_inv_sqrt"]
    assert f"{orc.fnv_hash(run('log', xp)):016x}" == gd["sub:fp_log"]
    assert f"{orc.fnv_hash(run('exp', ea)):016x}" == gd["sub:fp_exp"]
    assert f"{orc.fnv_hash(run('cos', g)):016x}" == gd["sub:fp_sincos_cos"]
    assert f"{orc.fnv_hash(run('sin', g)):016x}" == gd["sub:fp_sincos_sin"]
    assert f"{orc.fnv_hash(run('sigmoid', g)):016x}" == gd["sub:fp_sigmoid"]
    assert f"{orc.fnv_hash(run('silu', g)):016x}" == gd["sub:fp_silu"]


@pytest.mark.parametrize("fn", list(range(13)))
def test_fp_ports_random_vs_oracle(fn):
    import torch
    rng = np.random.default_rng(fn)
    x = np.concatenate([rand_full(rng, 3000), rng.integers(-50 * ONE, 50 * ONE, 3000)]).astype(np.int64)
    y = np.roll(x, 5)
    if fn == 1:
        y[y == 0] = 1
    if fn == 12:
        x = rng.integers(-3 * ONE, 3 * ONE, x.size).astype(np.int64)
        y = rng.integers(0, 20, x.size).astype(np.int64)
    want = orc.fp_vec(fn, x, y)
    do = torch.empty(x.size, dtype=torch.int64, device="cuda")
    iq.fp_dev(fn, dev(x), dev(y), do, x.size)
    assert (host(do) == want).all()


def test_fp_div_fast_path_edges_vs_oracle():
    """fp_div's estimate-and-correct path at its edges: quotients near 2^50 (the
    switch to the long division), divisors near 2^61, exact quotients (remainder
    0), remainders of |b| - 1, softmax-like numerators over sums, and the
    extreme magnitudes (INT64_MIN, +-1)."""
    import torch
    rng = np.random.default_rng(77)
    M = (1 << 63) - 1
    xs, ys = [], []
    for _ in range(3000):   # quotient near 2^50 +- a little
        b = int(rng.integers(1, 1 << 40))
        q = (1 << 50) + int(rng.integers(-4, 5))
        a = (q * b) >> 48
        for da in (-1, 0, 1):
            if 0 <= a + da <= M:
                xs.append(a + da); ys.append(b)
    for _ in range(3000):   # divisors near 2^61
        b = (1 << 61) + int(rng.integers(-8, 9))
        a = int(rng.integers(0, M))
        xs.append(a); ys.append(b)
    for _ in range(3000):   # exact quotients and remainders of b - 1
        b = int(rng.integers(1, 1 << 55))
        q = int(rng.integers(0, 1 << 49))
        n = q * b            # = a << 48 exactly when 2^48 divides n
        a = n >> 48
        xs += [a, a + 1, max(a - 1, 0)]; ys += [b, b, b]
    for _ in range(3000):   # softmax numerators e <= 2^48 over sums up to ~2^60
        S = int(rng.integers(1 << 48, 1 << 60))
        e = int(rng.integers(0, (1 << 48) + 1))
        xs.append(e); ys.append(S)
    ext = [-(1 << 63), M, 1, -1, 0, 1 << 48, -(1 << 48), 3, (1 << 62) + 7]
    for a in ext:
        for b in ext:
            if b != 0:
                xs.append(a); ys.append(b)
    x = np.array(xs, dtype=np.int64)
    y = np.array(ys, dtype=np.int64)
    sg = rng.integers(0, 4, x.size)
    x = np.where(sg & 1, -x, x).astype(np.int64)   # INT64_MIN stays INT64_MIN
    y = np.where(sg & 2, -y, y).astype(np.int64)
    want = orc.fp_vec(1, x, y)
    do = torch.empty(x.size, dtype=torch.int64, device="cuda")
    iq.fp_dev(1, dev(x), dev(y), do, x.size)
    got = host(do)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(int(x[i]), int(y[i]), int(got[i]), int(want[i])) for i in bad[:5]]


def test_rmsnorm_softmax_vs_oracle():
    import torch
    rng = np.random.default_rng(1)
    for rows, dim in ((1, 1), (3, 7), (4, 2048), (2, 5632)):
        x = rng.integers(-8 * ONE, 8 * ONE, (rows, dim)).astype(np.int64)
        w = rng.integers(-2 * ONE, 2 * ONE, dim).astype(np.int64)
        want = np.empty_like(x)
        for r in range(rows):
            orc.O.iqo_rmsnorm(orc.p(want[r]), orc.p(np.ascontiguousarray(x[r])), orc.p(w), dim)
        do = torch.empty((rows, dim), dtype=torch.int64, device="cuda")
        iq.rmsnorm_dev(do, dev(x), dev(w), rows, dim)
        assert (host(do) == want).all()
        s = rng.integers(-30 * ONE, 30 * ONE, (rows, dim)).astype(np.int64)
        want = s.copy()
        for r in range(rows):
            row = np.ascontiguousarray(want[r])
            orc.O.iqo_softmax(orc.p(row), dim)
            want[r] = row
        ds = dev(s)
        iq.softmax_dev(ds, rows, dim)
        assert (host(ds) == want).all()


# ------------------------------------------------------------ packed planes

@pytest.mark.parametrize("M,N", [(1, 1), (3, 17), (5, 64), (16, 32), (17, 33), (64, 1000), (33, 2048),
                                 (1000, 63), (129, 4097), (7, 40000), (2048, 2048), (256, 2048),
                                 (2560, 2048), (5000, 300), (9600, 64)])
@pytest.mark.parametrize("dist", ["full", "cfg"])
def test_matvec_packed_vs_oracle(M, N, dist):
    """Byte-plane tensor-core matvec: exact on full-range int64 (mod 2^128 wrap)
    and on config-distributed inputs; repeated launches (row scratch resets).
    Shapes reach the row-owned kernel with clusters of 1 (1000x63, 2560x2048),
    2 (2048x2048), 4 (256x2048) and 8 CTAs (129x4097), row-owned over two
    waves (5000x300), the stream-K kernel with staged digits (9600 rows: more
    than two waves of row tiles) and with digits read from global memory
    (7x40000)."""
    import torch
    rng = np.random.default_rng(M * 31 + N)
    if dist == "full":
        w, x = rand_full(rng, (M, N)), rand_full(rng, (N,))
    else:
        w = orc.synth_weights(1, f"w:{M}x{N}", (M, N))
        x = orc.synth_acts(1, f"x:{M}x{N}", (N,))
    want = orc.matmul_vec(w, x)
    pk = iq.Packed(dev(w), M, N)
    # full-range weights keep byte planes; config weights take the 2-byte bf16
    # form on the config shapes (rows too long to stage keep planes)
    if dist == "full" or N > 12768:
        assert pk.fmt() == "planes"
    elif M * N >= 256 * 2048:
        assert pk.fmt() == "bf16"
    dx = dev(x)
    for _ in range(2):
        do = torch.zeros(M, dtype=torch.int64, device="cuda")
        iq.matvec_packed_dev(do, pk, dx)
        assert (host(do) == want).all()
    pk.free()


# ------------------------------------------------------------- tcgen05 GEMM

@pytest.mark.parametrize("rows,M,N", [(2, 5, 7), (31, 64, 129), (33, 130, 1000), (64, 256, 2048),
                                      (100, 300, 5632), (512, 128, 256), (512, 2560, 300)])
@pytest.mark.parametrize("dist", ["full", "cfg"])
def test_gemm_tc_vs_oracle(rows, M, N, dist):
    """tcgen05 kind::i8 byte-plane GEMM: exact on full-range int64 and on
    config-distributed inputs; padding of rows (128), x-rows (32) and K (128);
    split-K with 128-bit partials (small grids) and the single-pass epilogue
    (512 x 2560: enough tiles to fill the GPU without splitting)."""
    import torch
    rng = np.random.default_rng(rows * 7 + M + N)
    if dist == "full":
        w, X = rand_full(rng, (M, N)), rand_full(rng, (rows, N))
    else:
        w = orc.synth_weights(2, f"w:{M}x{N}", (M, N))
        X = orc.synth_acts(2, f"X:{rows}x{N}", (rows, N))
    want = orc.matmul_rows(w, X)
    pk = iq.PackedTC(dev(w), M, N)
    do = torch.zeros((rows, M), dtype=torch.int64, device="cuda")
    iq.gemm_tc_dev(do, pk, dev(X), rows)
    got = host(do)
    assert iq.device_status() == 0
    assert (got == want).all()
    pk.free()


def _weights_with_planes(rng, n, shape):
    """int64 weights that need exactly n bytes as signed integers, boundaries included."""
    lo, hi = -(1 << (8 * n - 1)), (1 << (8 * n - 1)) - 1
    w = rng.integers(lo, hi, shape, dtype=np.int64, endpoint=True)
    flat = w.reshape(-1)
    flat[0], flat[-1] = lo, hi
    return w


@pytest.mark.parametrize("n", list(range(1, 9)))
def test_plane_count_matvec_and_gemm(n):
    """Packing keeps only the byte planes the weights need (top one signed);
    results stay exact for every plane count, at the signed range boundaries."""
    import torch
    rng = np.random.default_rng(100 + n)
    M, N, rows = 37, 1000, 5
    w = _weights_with_planes(rng, n, (M, N))
    x, X = rand_full(rng, (N,)), rand_full(rng, (rows, N))
    pk = iq.Packed(dev(w), M, N)
    do = torch.zeros(M, dtype=torch.int64, device="cuda")
    iq.matvec_packed_dev(do, pk, dev(x))
    assert (host(do) == orc.matmul_vec(w, x)).all()
    pt = iq.PackedTC(dev(w), M, N)
    dg = torch.zeros((rows, M), dtype=torch.int64, device="cuda")
    iq.gemm_tc_dev(dg, pt, dev(X), rows)
    assert (host(dg) == orc.matmul_rows(w, X)).all()
    pk.free(); pt.free()


def test_plane_window_config_weights():
    """bf16-derived config weights keep planes 3..5 (3 bytes per weight) and put
    the few weights with nonzero low bytes into the sparse residual."""
    import torch
    w = orc.synth_weights(1, "w:window", (2048, 2048))
    pk = iq.Packed(dev(w), 2048, 2048, fmt="planes")
    np_, p0, nnz = pk.info()
    low = (w.view(np.uint64) & np.uint64((1 << 8 * p0) - 1)) != 0
    assert (np_, p0) == (3, 3) and nnz == int(low.sum()) and 0 < nnz < 2048 * 2048 // 1024
    x = orc.synth_acts(1, "x:window", (2048,))
    do = torch.zeros(2048, dtype=torch.int64, device="cuda")
    iq.matvec_packed_dev(do, pk, dev(x))
    assert (host(do) == orc.matmul_vec(w, x)).all()
    pk.free()


@pytest.mark.parametrize("M,N", [(300, 2048), (9600, 64)])
def test_plane_window_residual_edges(M, N):
    """Weights whose high bytes fit planes 3..5 with planted low-byte entries:
    a row holding many of them, first and last rows and columns, negative
    weights and full-range activations (row-owned and stream-K kernels)."""
    import torch
    rng = np.random.default_rng(M + N)
    w = rng.integers(-(1 << 23), 1 << 23, (M, N), dtype=np.int64) << 24   # bytes 3..5 only
    planted = [(7, k) for k in range(0, N, max(1, N // 40))] + [(0, 0), (M - 1, N - 1), (M // 2, 1)]
    for r, k in planted:
        w[r, k] += int(rng.integers(1, 1 << 24))
    w[3, 5] = -int(rng.integers(1, 1 << 24))    # a negative weight with low bytes
    x = rand_full(rng, (N,))
    pk = iq.Packed(dev(w), M, N)
    np_, p0, nnz = pk.info()
    assert p0 == 3 and np_ == 3 and nnz == int(((w.view(np.uint64) & np.uint64(0xFFFFFF)) != 0).sum())
    for _ in range(2):
        do = torch.zeros(M, dtype=torch.int64, device="cuda")
        iq.matvec_packed_dev(do, pk, dev(x))
        assert (host(do) == orc.matmul_vec(w, x)).all()
    pk.free()


def test_gemm_plane_window_and_residual():
    """tcgen05 GEMM on weights whose high bytes fit planes 3..5, with three
    planted low-byte entries (few enough for the GEMM's residual): window
    (3, 3, 3); config weights keep bytes 2..5; exact with split-K (5 rows)
    and in one pass (300 rows)."""
    import torch
    rng = np.random.default_rng(77)
    M = N = 2048
    w = rng.integers(-(1 << 23), 1 << 23, (M, N), dtype=np.int64) << 24
    w[0, 0] += 12345
    w[7, 1000] -= 777
    w[M - 1, N - 1] += (1 << 24) - 1
    pt = iq.PackedTC(dev(w), M, N)
    assert pt.info() == (3, 3, 3)
    for rows in (5, 300):
        X = rand_full(rng, (rows, N))
        dg = torch.zeros((rows, M), dtype=torch.int64, device="cuda")
        iq.gemm_tc_dev(dg, pt, dev(X), rows)
        assert iq.device_status() == 0
        assert (host(dg) == orc.matmul_rows(w, X)).all(), rows
    pt.free()
    wc = orc.synth_weights(2, "w:tcwindow", (2560, 2048))
    pc = iq.PackedTC(dev(wc), 2560, 2048)
    np_, p0, nnz = pc.info()
    assert (np_, p0) == (4, 2) and nnz == int(((wc.view(np.uint64) & np.uint64(0xFFFF)) != 0).sum())
    X = orc.synth_acts(2, "X:tcwindow", (64, 2048))
    dg = torch.zeros((64, 2560), dtype=torch.int64, device="cuda")
    iq.gemm_tc_dev(dg, pc, dev(X), 64)
    assert (host(dg) == orc.matmul_rows(wc, X)).all()
    pc.free()


# ---------------------------------------------------- config-2 reference golden

def test_gemm_tc_cfg2_shapes_match_reference_golden():
    """Config 2 at its own shapes (512 rows of QKV 2048->2560, O 2048->2048,
    gate+up 2048->11264, down 5632->2048): the tcgen05 GEMM's outputs hash to
    the values the reference's own matmul_vec produced row by row
    (tests/golden/gemm_cfg2.json, made by make_golden.py --cfg2)."""
    import torch
    for g in json.load(open(os.path.join(GOLD, "gemm_cfg2.json"))):
        K, N, rows = g["K"], g["N"], g["rows"]
        w = iq.synth_weights(2, g["weight"], (N, K))
        X = iq.synth_acts(2, g["act"], (rows, K))
        pk = iq.PackedTC(dev(w), N, K)
        do = torch.zeros((rows, N), dtype=torch.int64, device="cuda")
        iq.gemm_tc_dev(do, pk, dev(X), rows)
        got = host(do)
        assert iq.device_status() == 0
        assert [orc.fnv_hash(got[r]) for r in range(0, rows, 64)] == g["row_hashes"], g["tag"]
        assert orc.fnv_hash(got) == g["out_hash"], g["tag"]
        pk.free()


# ---------------------------------------------------------- bounded waits

def test_bounded_wait_gives_up_and_reports_timeout():
    """A wait on an mbarrier that nothing arrives at gives up after its limit
    (1 ms here), records IQ_ERR_TIMEOUT, and the host reads it once: the next
    read is IQ_OK again, and the context stays usable."""
    assert iq.device_status() == 0
    assert iq.lib().iq_wait_selftest(1000000) == 0
    assert iq.device_status() == -5   # IQ_ERR_TIMEOUT
    assert iq.device_status() == 0
    test_matvec_dev_edges(3, 17, "full")   # a later launch still runs correctly


# ------------------------------------------- drop-in cache: changed host weights

def test_dropin_detects_new_matrix_at_the_same_address():
    """The reference's streaming path frees each layer after use and the next
    layer can land at the same address (llama_int.c:2840-2872). Overwriting the
    host matrix in place must never return the previous matrix's results: the
    default sampled fingerprint and the full hash both catch it."""
    rng = np.random.default_rng(21)
    M, N = 300, 2048
    buf = np.empty((M, N), np.int64)
    x = orc.synth_acts(1, "x:stale", (N,))
    try:
        for mode in ("sampled", "full", "none"):
            iq.weight_check_mode(mode)
            iq.weight_cache_clear()
            for layer in range(3):
                buf[:] = orc.synth_weights(1, f"w:stale{layer}", (M, N))
                out = np.empty(M, np.int64)
                iq.matmul_vec(out, buf, x, M, N)
                if mode != "none" or layer == 0:
                    assert (out == orc.matmul_vec(buf, x)).all(), (mode, layer)
            # one changed value in a sampled position (the first) is seen too
            if mode != "none":
                buf[0, 0] += 1 << 40
                out = np.empty(M, np.int64)
                iq.matmul_vec(out, buf, x, M, N)
                assert (out == orc.matmul_vec(buf, x)).all(), mode
    finally:
        iq.weight_check_mode("sampled")
        iq.weight_cache_clear()


def test_dropin_full_mode_finds_reloaded_layers_by_content():
    """Full-hash mode: a layer re-read into a fresh buffer (another address)
    reuses its packed copy; results stay exact; the LRU byte limit evicts."""
    M, N = 256, 1024
    x = orc.synth_acts(1, "x:reload", (N,))
    mats = [orc.synth_weights(1, f"w:reload{i}", (M, N)) for i in range(3)]
    try:
        iq.weight_check_mode("full")
        iq.weight_cache_clear()
        for token in range(3):
            for i, w in enumerate(mats):
                fresh = w.copy()           # new buffer each time, like the streaming loader
                out = np.empty(M, np.int64)
                iq.matmul_vec(out, fresh, x, M, N)
                assert (out == orc.matmul_vec(w, x)).all(), (token, i)
                del fresh
        entries, nbytes = iq.weight_cache_stats()
        assert entries == 3 and nbytes > 0
        iq.weight_cache_limit(nbytes - 1)   # one byte short: the least recently used goes
        assert iq.weight_cache_stats()[0] == 2
        out = np.empty(M, np.int64)
        iq.matmul_vec(out, mats[0].copy(), x, M, N)
        assert (out == orc.matmul_vec(mats[0], x)).all()
    finally:
        iq.weight_cache_limit(64 << 30)
        iq.weight_check_mode("sampled")
        iq.weight_cache_clear()


# ------------------------------------------------------------- bf16 form

def _bf16_weights(rng, shape, outliers):
    """bf16-derived weights (bfloat16_to_q1648 of N(0, 0.02) values) with
    planted weights the bf16 form cannot hold: |w| >= 0.25, exponent-255 codes
    (+-32000.0), tiny truncated values, and non-bf16 int64 values, at the first
    and last rows and columns and in one crowded row."""
    import torch
    f = torch.from_numpy(rng.normal(0, 0.02, shape).astype(np.float32)).bfloat16()
    bits = f.view(torch.int16).numpy().astype(np.uint16)
    conv = np.vectorize(orc.O.iqo_bf16_to_q1648, otypes=[np.int64])
    w = conv(bits)
    M, N = shape
    if outliers:
        spots = [(0, 0), (M - 1, N - 1), (0, N - 1), (M - 1, 0)] + [(M // 2, k) for k in range(0, N, 7)]
        vals = [orc.O.iqo_bf16_to_q1648(0x3F00), orc.O.iqo_bf16_to_q1648(0xBF40), orc.O.iqo_bf16_to_q1648(0x7F85),
                orc.O.iqo_bf16_to_q1648(0xFF80), orc.O.iqo_bf16_to_q1648(0x2A31), orc.O.iqo_bf16_to_q1648(0xAA31),
                (1 << 40) + 12345, -(1 << 50) - 7]
        for i, (r, k) in enumerate(spots):
            w[r, k] = vals[i % len(vals)]
    return w


@pytest.mark.parametrize("M,N", [(1, 1), (17, 33), (300, 2048), (2048, 2048), (256, 2048), (129, 4097),
                                 (5000, 300), (9600, 64), (64, 12768)])
@pytest.mark.parametrize("outliers", [False, True])
def test_bf16_form_vs_oracle(M, N, outliers):
    """The 2-byte bf16 form (in-kernel bf16 -> byte planes, u = v + 2^22 bias,
    2^22 sum x correction, whole-weight residual) equals the oracle bit for bit,
    forced on every shape: row-owned kernel with clusters of 1..8, two waves,
    stream-K (9600 rows), the longest row it accepts (N = 12768), padding of
    rows and columns (-0.25 pad weights), and planted weights it cannot hold."""
    import torch
    rng = np.random.default_rng(M * 7 + N)
    w = _bf16_weights(rng, (M, N), outliers)
    x = rand_full(rng, (N,))
    want = orc.matmul_vec(w, x)
    pk = iq.Packed(dev(w), M, N, fmt="bf16")
    assert pk.fmt() == "bf16"
    dx = dev(x)
    for _ in range(2):
        do = torch.zeros(M, dtype=torch.int64, device="cuda")
        iq.matvec_packed_dev(do, pk, dx)
        assert (host(do) == want).all()
    pk.free()


def test_bf16_form_rejects_unstageable_rows_and_full_range_stays_exact():
    import torch
    w = torch.zeros((4, 13000), dtype=torch.int64, device="cuda")
    with pytest.raises(iq.IQError) as e:
        iq.Packed(w, 4, 13000, fmt="bf16")
    assert e.value.status == -8   # IQ_ERR_UNSUPPORTED
    rng = np.random.default_rng(3)
    w = rand_full(rng, (40, 300))     # nothing representable: every weight in the residual
    x = rand_full(rng, (300,))
    pk = iq.Packed(dev(w), 40, 300, fmt="bf16")
    do = torch.zeros(40, dtype=torch.int64, device="cuda")
    iq.matvec_packed_dev(do, pk, dev(x))
    assert (host(do) == orc.matmul_vec(w, x)).all()
    pk.free()
    pk = iq.Packed(dev(w), 40, 300)
    assert pk.fmt() == "planes"       # the automatic choice never picks it here
    pk.free()
