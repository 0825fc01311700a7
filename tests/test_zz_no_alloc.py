"""dk_row_stats_noalloc, the allocation-free row statistics, against dk_row_stats.

The variant is for callers that cannot let the library allocate device memory (a
real-time audio thread that must not block on cudaMalloc/cudaFree, or a host whose own pool
owns all device memory): its scratch is a fixed device array instead of a buffer grown with
cudaMalloc.  This file is collected last so that a run stopping at the first failure has
run every other test before it; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def _stats(dcb, torch, fn, x, rows, L):
    st = torch.full((2 * rows,), float("nan"), device="cuda")
    r = fn(C.c_void_p(x.data_ptr()), rows, L, C.c_void_p(st.data_ptr()),
           C.c_void_p(st.data_ptr() + 4 * rows))
    torch.cuda.synchronize()
    return r, st[:rows].cpu().numpy(), st[rows:].cpu().numpy()


def test_noalloc_matches_row_stats_twice(torch_cuda):
    torch = torch_cuda
    import demucs_cuda_b200 as dcb
    L_ = dcb.lib()
    rng = np.random.default_rng(11)
    # two calls in a row with different shapes: the second one must not see the first one's
    # partials (a long-row case with 336 chunks per row, then many short rows)
    for rows, L in ((8, 2_752_512), (37, 20_000)):
        x = (rng.standard_normal((rows, L)) * 3 + 0.5).astype(np.float32)
        xt = torch.from_numpy(x).cuda()
        _, m_ref, v_ref = _stats(dcb, torch, L_.dk_row_stats, xt, rows, L)
        dcb.check(True, "dk_row_stats")
        r, m, v = _stats(dcb, torch, L_.dk_row_stats_noalloc, xt, rows, L)
        dcb.check(r == 0, "dk_row_stats_noalloc")
        assert rel_l2(m, m_ref) < 1e-5 and rel_l2(v, v_ref) < 1e-5
        xd = x.astype(np.float64)
        assert rel_l2(v, xd.var(axis=1)) < 1e-5
        assert np.abs(m - xd.mean(axis=1)).max() < 1e-5
    assert dcb.device_fault() == 0


def test_noalloc_rejects_oversized(torch_cuda):
    torch = torch_cuda
    import demucs_cuda_b200 as dcb
    L_ = dcb.lib()
    x = torch.zeros(16, device="cuda")
    st = torch.zeros(2 * 50_000, device="cuda")
    # 50000 rows x 1 chunk exceeds the 43690 reserved partials: rejected before any launch
    r = L_.dk_row_stats_noalloc(C.c_void_p(x.data_ptr()), 50_000, 1, C.c_void_p(st.data_ptr()),
                                C.c_void_p(st.data_ptr() + 4 * 50_000))
    assert r == -1
    with pytest.raises(dcb.BackendError, match="reserves"):
        dcb.check(True, "oversized")


def test_noalloc_reports_only_its_own_errors(torch_cuda):
    """An error left pending on this thread by an earlier, unrelated call does not make a
    good call fail; a call whose factors would overflow the partials product is rejected
    before any launch."""
    torch = torch_cuda
    import demucs_cuda_b200 as dcb
    L_ = dcb.lib()
    dcb.check(True, "clean start")
    assert L_.dcb_set_option(b"no-such-option", 1) == -1   # records an error, left pending
    x = torch.randn(4, 1000, device="cuda")
    st = torch.zeros(8, device="cuda")
    r = L_.dk_row_stats_noalloc(C.c_void_p(x.data_ptr()), 4, 1000, C.c_void_p(st.data_ptr()),
                                C.c_void_p(st.data_ptr() + 16))
    torch.cuda.synchronize()
    assert r == 0
    assert "no-such-option" in L_.dcb_last_error(1).decode()
    xd = x.double().cpu().numpy()
    assert np.abs(st[:4].cpu().numpy() - xd.mean(axis=1)).max() < 1e-5
    # 3 rows x 2^27 chunks: each factor is checked before the product
    r = L_.dk_row_stats_noalloc(C.c_void_p(x.data_ptr()), 3, 1 << 40, C.c_void_p(st.data_ptr()),
                                C.c_void_p(st.data_ptr() + 16))
    assert r == -1
    with pytest.raises(dcb.BackendError, match="reserves"):
        dcb.check(True, "overflowing factors")
