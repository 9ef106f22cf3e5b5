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
