"""CPU checks of the integer identities the CUDA kernels are built on, in exact
Python integers (the GPU tests check the kernels themselves bit-for-bit):

* byte planes with a signed top plane, a stored window p0..p0+np-1 and the
  sparse low-byte residual (iq_planes.cuh, iq_tc_gemm.cuh);
* the GEMM epilogue's digit fold in two 64-bit halves (iq_tc_gemm.cuh);
* the 32-bit limb form of the attention score dot (iq_layer.cuh, k_attn_scores).
All sums are taken mod 2^128, as the kernels' (and the reference's) int128."""
import random

M128 = (1 << 128) - 1


def s64(x):
    x &= (1 << 64) - 1
    return x - (1 << 64) if x >> 63 else x


def s32(x):
    x &= 0xFFFFFFFF
    return x - (1 << 32) if x >> 31 else x


def byte(w, p):
    return (w >> (8 * p)) & 0xFF


def plane_dot(ws, xs, p0, np_):
    """sum x w from stored planes p0..p0+np-1 of w_hi (top signed), the x digits,
    the 2^63 row-sum correction and the sparse residual of w_lo."""
    mask = (1 << (8 * p0)) - 1
    acc = 0
    for i in range(np_):
        p = p0 + i
        for j in range(8):
            pij = 0
            for w, x in zip(ws, xs):
                b = byte(w, p)
                if i == np_ - 1 and b >= 128:
                    b -= 256                       # top stored plane is signed
                pij += b * byte(x + (1 << 63), j)  # digits of x_u = x + 2^63
            acc += pij << (8 * (p + j))
    acc -= sum(w & ~mask for w in ws) << 63        # 2^63 * sum w_hi
    acc += sum(x * (w & mask) for w, x in zip(ws, xs) if w & mask)   # residual
    return acc & M128


def needed_bytes(w):
    m = ~w if w < 0 else w
    return (m.bit_length() + 1 + 7) // 8


def test_plane_window_identity():
    rng = random.Random(5)
    for trial in range(60):
        n = rng.choice([1, 7, 32])
        top = rng.randint(1, 8)
        ws = [rng.randint(-(1 << (8 * top - 1)), (1 << (8 * top - 1)) - 1) for _ in range(n)]
        xs = [s64(rng.getrandbits(64)) for _ in range(n)]
        exact = sum(w * x for w, x in zip(ws, xs)) & M128
        t = max(needed_bytes(w) for w in ws)
        for p0 in range(t):
            assert plane_dot(ws, xs, p0, t - p0) == exact, (trial, p0)


def test_gemm_fold_halves():
    """sum_j v_j 2^(8j) over 8 int32 digit sums equals lo + hi 2^32, lo/hi each
    summing 4 terms with shifts <= 24 inside int64."""
    rng = random.Random(6)
    for _ in range(20000):
        v = [rng.randint(-(1 << 31), (1 << 31) - 1) for _ in range(8)]
        lo = sum(v[j] << (8 * j) for j in range(4))
        hi = sum(v[4 + j] << (8 * j) for j in range(4))
        assert -(1 << 63) <= lo < (1 << 63) and -(1 << 63) <= hi < (1 << 63)
        assert lo + (hi << 32) == sum(v[j] << (8 * j) for j in range(8))


def test_limb_score_dot():
    rng = random.Random(7)
    for trial in range(300):
        hd = rng.choice([1, 32, 64, 128, 256])
        if trial % 4 == 0:
            ext = [-(1 << 63), (1 << 63) - 1, 0, -1]
            q = [rng.choice(ext) for _ in range(hd)]
            k = [rng.choice(ext) for _ in range(hd)]
        else:
            q = [s64(rng.getrandbits(64)) for _ in range(hd)]
            k = [s64(rng.getrandbits(64)) for _ in range(hd)]
        H, L = [0, 0, 0], [0, 0, 0]
        for a, b in zip(q, k):
            limbs = (a & 0x3FFFFF, (a >> 22) & 0x3FFFFF, a >> 44)
            kh, ks = b >> 32, s32((b & 0xFFFFFFFF) ^ 0x80000000)
            for i, ai in enumerate(limbs):
                H[i] += ai * kh
                L[i] += ai * ks
        for v in H + L:
            assert -(1 << 63) <= v < (1 << 63)      # int64 partial sums never overflow
        dot = sum((H[i] << (32 + 22 * i)) + (L[i] << (22 * i)) for i in range(3)) + (sum(q) << 31)
        assert dot & M128 == sum(a * b for a, b in zip(q, k)) & M128, trial


# ------------------------------------------------------------ bf16 form

def bf_encode(w):
    """Restates iq_planes.cuh bf_encode: the bf16 bits that hold w exactly as
    v 2^24 (v in [-2^22, 2^22), <= 8 significant bits), else -1."""
    if w & 0xFFFFFF:
        return -1
    v = w >> 24
    if not -(1 << 22) <= v < (1 << 22):
        return -1
    if v == 0:
        return 0
    a = abs(v)
    e2 = a.bit_length() - 1
    tz = (a & -a).bit_length() - 1
    if e2 - tz >= 8:
        return -1
    return (0x8000 if v < 0 else 0) | ((e2 + 103) << 7) | (((a << 7) >> e2) & 0x7F)


def bf_u(bits):
    """u = low 23 bits of fp32 fma.rm(f, 2^24, 1.5*2^23) for the bf16 value f:
    here the exact sum is an integer in [2^23, 2^24), so any rounding mode gives
    it; numpy's fp32 (round to nearest) shows the bit pattern."""
    import numpy as np
    f = np.array([bits << 16], dtype=np.uint32).view(np.float32)[0]
    r = np.float32(np.float64(f) * 16777216.0 + 12582912.0)
    assert np.float64(r) == np.float64(f) * 16777216.0 + 12582912.0   # exact
    return int(np.array([r], dtype=np.float32).view(np.uint32)[0]) & 0x7FFFFF


def test_bf16_encode_decode_exact_and_u_bias():
    import oracle as orc
    rng = random.Random(5)
    seen = 0
    for bits in list(range(0, 0x10000, 37)) + [0xBE80, 0x3E80, 0x0001]:
        w = orc.O.iqo_bf16_to_q1648(bits)
        enc = bf_encode(w)
        if enc < 0:
            continue
        seen += 1
        # the stored bits decode (bfloat16_to_q1648) to the same weight
        assert orc.O.iqo_bf16_to_q1648(enc) == w, hex(bits)
        assert bf_u(enc) == (w >> 24) + (1 << 22), hex(bits)
    assert seen > 1000
    assert bf_u(0xBE80) == 0            # padding: -0.25 -> u = 0
    assert bf_u(0) == 1 << 22           # +0.0 -> v = 0


def test_bf16_form_dot_identity():
    """sum x w = 2^24 (sum_k x_u u - 2^63 U - 2^22 X) + residual (mod 2^128), with
    x_u = x + 2^63, u = v + 2^22, U = sum u, X = sum x; weights the form cannot
    hold are v = 0 and go to the residual whole."""
    import oracle as orc
    rng = random.Random(9)
    for trial in range(40):
        n = rng.randint(1, 70)
        ws = []
        for _ in range(n):
            kind = rng.random()
            if kind < 0.8:   # bf16-derived, config-like
                ws.append(orc.O.iqo_bf16_to_q1648(rng.choice(range(0x3000, 0x3F00)) | rng.choice([0, 0x8000])))
            elif kind < 0.9:
                ws.append(rng.randint(-(1 << 63), (1 << 63) - 1))
            else:
                ws.append(orc.O.iqo_bf16_to_q1648(rng.randint(0, 0xFFFF)))
        xs = [rng.randint(-(1 << 63), (1 << 63) - 1) for _ in range(n)]
        want = sum(x * w for x, w in zip(xs, ws)) & M128
        acc = U = X = res = 0
        for x, w in zip(xs, ws):
            e = bf_encode(w)
            v = (w >> 24) if e >= 0 else 0
            u = v + (1 << 22)
            acc += (x + (1 << 63)) * u
            U += u
            X += x
            res += x * (w - (v << 24))
        got = ((acc - (U << 63) - (X << 22)) << 24) + res
        assert got & M128 == want, trial


# ---- tensor-core attention and fp_div (exact Python integers) -------------

M64 = (1 << 64) - 1


def _bytes_signed_top(x):
    """7 unsigned bytes and a signed top byte: x = sum_i b_i 2^(8i)."""
    u = x & M64
    b = [(u >> (8 * i)) & 0xFF for i in range(8)]
    if b[7] >= 128:
        b[7] -= 256
    return b


def _fp_mul(a, b):
    return ((a * b) >> 48) & M64


def test_score_diagonals_mod_2_112():
    """k_attn_scores_tc: sum over diagonals s = i + j <= 13 of 2^(8s) sum_d q_i k_j,
    each diagonal within int32, recombined in three int64 groups, gives the
    reference's (q . k >> 48) mod 2^64 (the (7, 7) pair only adds multiples of 2^112)."""
    rng = random.Random(5)
    for hd in (32, 64, 128, 256):
        for _ in range(40):
            mode = rng.randrange(3)
            def val():
                if mode == 0:
                    return rng.randrange(-(1 << 63), 1 << 63)
                if mode == 1:
                    return rng.choice([-(1 << 63), (1 << 63) - 1, -1, 0, 1])
                return rng.randrange(-(1 << 52), 1 << 52)
            q = [val() for _ in range(hd)]
            k = [val() for _ in range(hd)]
            want = (sum(a * b for a, b in zip(q, k)) >> 48) & M64
            qb = [_bytes_signed_top(a) for a in q]
            kb = [_bytes_signed_top(b) for b in k]
            D = [0] * 14
            for i in range(8):
                for j in range(8):
                    if i + j > 13:
                        continue
                    D[i + j] += sum(kb[d][i] * qb[d][j] for d in range(hd))
            assert all(-(1 << 31) <= v < (1 << 31) for v in D)
            G0 = sum(D[s] << (8 * s) for s in range(5))
            G1 = sum(D[s] << (8 * (s - 5)) for s in range(5, 10))
            G2 = sum(D[s] << (8 * (s - 10)) for s in range(10, 14))
            assert all(-(1 << 61) <= g < (1 << 61) for g in (G0, G1, G2))
            dot = (G0 + (G1 << 40) + (G2 << 80)) % (1 << 128)
            assert (dot >> 48) & M64 == want


def _r_pieces(p, v):
    """R = (p v) mod 2^48 from 32-bit pieces, as k_attn_pv_tc's PTX block:
    lo(p) lo(v) mod 2^32 + 2^32 ((hi(lo(p) lo(v)) + lo(p) hi(v) + hi(p) lo(v)) mod 2^16)."""
    vu = v & M64
    plo, phi, vlo, vhi = p & 0xFFFFFFFF, p >> 32, vu & 0xFFFFFFFF, vu >> 32
    w = plo * vlo
    hi = ((w >> 32) + plo * vhi + phi * vlo) & 0xFFFF
    return (w & 0xFFFFFFFF) + (hi << 32)


def test_pv_floor_identity_and_remainder_pieces():
    """k_attn_pv_tc: sum_t fp_mul(p_t, v_t) = (sum p v - sum R) / 2^48 mod 2^64 with
    R_t = (p_t v_t) mod 2^48 from 32-bit pieces; the products' byte-plane diagonals
    (p: 7 unsigned bytes, v: signed top) in int32; the four int64 limb sums
    weighted 2^0, 2^32, 2^64, 2^96 recombine to the same value."""
    rng = random.Random(9)
    for T in (1, 7, 64, 256):
        for _ in range(30):
            ps = [rng.choice([0, 1 << 48, rng.randrange(0, (1 << 48) + 1), rng.randrange(0, 1 << 40)])
                  for _ in range(T)]
            vs = [rng.choice([rng.randrange(-(1 << 63), 1 << 63), rng.randrange(-(1 << 50), 1 << 50),
                              -(1 << 63), (1 << 63) - 1]) for _ in range(T)]
            want = sum(_fp_mul(p, v) for p, v in zip(ps, vs)) & M64
            for p, v in zip(ps, vs):
                assert _r_pieces(p, v) == (p * v) % (1 << 48)
            Rsum = sum(_r_pieces(p, v) for p, v in zip(ps, vs))
            assert Rsum < 1 << 56
            pb = [[(p >> (8 * j)) & 0xFF for j in range(7)] for p in ps]
            vb = [_bytes_signed_top(v) for v in vs]
            D = [0] * 14
            for i in range(8):
                for j in range(7):
                    D[i + j] += sum(vb[t][i] * pb[t][j] for t in range(T))
            assert all(-(1 << 31) <= x < (1 << 31) for x in D)
            G = [0, 0, 0, 0]
            for s in range(14):
                G[s >> 2] += D[s] << (8 * (s & 3))
            G[0] -= Rsum
            assert all(-(1 << 63) <= g < (1 << 63) for g in G)
            X = (G[0] + (G[1] << 32) + (G[2] << 64) + (G[3] << 96)) % (1 << 128)
            assert X % (1 << 48) == 0
            assert (X >> 48) & M64 == want


def _fp_div_ref(a, b):
    ma, mb = abs(a), abs(b)
    q = ((ma << 48) // mb) & M64
    return q if (a < 0) == (b < 0) else (-q) & M64


def _fp_div_fast(a, b):
    """The device fp_div: a double estimate of |a| 2^48 / |b| corrected by one
    exact remainder step while it is below 2^50 and |b| < 2^61."""
    ma, mb = abs(a) & M64, abs(b) & M64
    qd = float(ma) * 281474976710656.0 / float(mb)
    if qd < 2.0 ** 50 and mb < (1 << 61):
        q = int(qd)
        r = ((ma << 48) - q * mb) & M64
        if r >= 1 << 63:
            r -= 1 << 64
        if r < 0:
            q -= 1
        elif r >= mb:
            q += 1
    else:
        q = ((ma << 48) // mb) & M64
    return q if (a < 0) == (b < 0) else (-q) & M64


def test_fp_div_estimate_and_correct():
    rng = random.Random(13)
    cases = []
    for _ in range(20000):
        b = rng.randrange(1, 1 << rng.randrange(1, 63))
        k = rng.randrange(4)
        if k == 0:
            a = ((1 << 50) + rng.randrange(-4, 5)) * b >> 48
        elif k == 1:
            a = (rng.randrange(0, 1 << 49) * b >> 48) + rng.randrange(-1, 2)
        elif k == 2:
            b = (1 << 61) + rng.randrange(-8, 9)
            a = rng.randrange(0, 1 << 63)
        else:
            a = rng.randrange(0, 1 << rng.randrange(1, 64))
        cases.append((max(0, min(a, (1 << 63) - 1)), b))
    ext = [-(1 << 63), (1 << 63) - 1, 1, -1, 1 << 48, 3]
    for a in ext:
        for b in ext:
            cases.append((a, b))
    for a, b in cases:
        for sa, sb in ((1, 1), (-1, 1), (1, -1), (-1, -1)):
            x, y = sa * a, sb * b
            if not (-(1 << 63) <= x < (1 << 63) and -(1 << 63) <= y < (1 << 63)) or y == 0:
                continue
            assert _fp_div_fast(x, y) == _fp_div_ref(x, y), (x, y)


def test_unsigned_square_equals_fp_mul_r_r():
    """fp_exp's squarings: fp_mul(r, r) from the unsigned square of |r|."""
    rng = random.Random(17)
    for _ in range(20000):
        r = rng.randrange(-(1 << 63), 1 << 63)
        m = abs(r) & M64
        assert (((m * m) >> 48) & M64) == (((r * r) >> 48) & M64)
