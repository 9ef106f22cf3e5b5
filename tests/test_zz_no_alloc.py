"""The allocation-free matvec entry point (iq_matvec_packed_noalloc_dev).

It exists for callers that cannot call cudaMalloc when they run -- for example
a process whose device memory belongs to an external pool or budget, or a
latency-critical loop that must not meet an allocation's implicit
synchronisation. Its scratch is a fixed array inside the library. This file is
named so that pytest collects it last; it must pass alone and after the rest.
"""
import ctypes

import numpy as np
import pytest

import iq
import oracle as orc

pytestmark = pytest.mark.gpu


def _run(name, out, pk, x):
    # iq._sp(None) names torch's current stream (cudaStreamLegacy for torch's
    # default stream, whose handle 0 the library would read as its own stream),
    # so both calls are ordered after the torch fills of `out` below
    L = iq.lib()
    rc = getattr(L, name)(ctypes.c_void_p(out.data_ptr()), pk.h, ctypes.c_void_p(x.data_ptr()), iq._sp(None))
    assert rc == 0, (name, rc)


# (2048, 2048) and (33, 5000) run the row-owned kernel, which needs no scratch;
# (32000, 2048) runs the stream-K kernel with staged x digits and (4096, 16384)
# the stream-K kernel without them (K beyond the staging limit), both of which
# split rows between warps through the fixed array.
@pytest.mark.parametrize("M,N", [(2048, 2048), (33, 5000), (32000, 2048), (4096, 16384)])
def test_noalloc_matches_regular_entry_point_twice(M, N):
    """Two calls in a row through the C ABI: each equals iq_matvec_packed_dev's
    output exactly (the tests' tolerance for integer work is zero)."""
    import torch
    rng = np.random.default_rng(M + N)
    w = rng.integers(-2 ** 63, 2 ** 63 - 1, (M, N), dtype=np.int64)
    dw = torch.from_numpy(w).cuda()
    pk = iq.Packed(dw, M, N)
    for call in range(2):
        x = torch.from_numpy(rng.integers(-2 ** 63, 2 ** 63 - 1, N, dtype=np.int64)).cuda()
        want = torch.zeros(M, dtype=torch.int64, device="cuda")
        got = torch.full((M,), 7, dtype=torch.int64, device="cuda")
        _run("iq_matvec_packed_dev", want, pk, x)
        _run("iq_matvec_packed_noalloc_dev", got, pk, x)
        torch.cuda.synchronize()
        assert torch.equal(got, want), call
    if M == 2048:  # and the oracle agrees
        assert (got.cpu().numpy() == orc.matmul_vec(w, x.cpu().numpy())).all()
    pk.free()


def test_noalloc_rejects_more_rows_than_its_fixed_scratch():
    import torch
    M, N = 32768 + 16, 32
    pk = iq.Packed(torch.zeros((M, N), dtype=torch.int64, device="cuda"), M, N)
    x = torch.zeros(N, dtype=torch.int64, device="cuda")
    out = torch.zeros(M, dtype=torch.int64, device="cuda")
    L = iq.lib()
    rc = L.iq_matvec_packed_noalloc_dev(ctypes.c_void_p(out.data_ptr()), pk.h,
                                        ctypes.c_void_p(x.data_ptr()), iq._sp(None))
    assert rc == -6  # IQ_ERR_RANGE
    pk.free()
