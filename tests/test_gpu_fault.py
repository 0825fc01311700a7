"""Failure detection without a GPU fault: a bounded device-side wait that expires.

Every mbarrier wait in the tensor-core kernels gives up after a wall-clock limit, records a
bit in the device fault word and lets the grid end, so a broken pipeline never hangs the
GPU.  This test shortens the limit (option "wait_limit_ms") and makes one GEMM CTA keep its
first operand stage (option "test_withhold_arrive": the stage is never released, the wait
for it is a flag nothing sets).  The kernel must return on its own, the host must read the
fault through dcb_device_fault(), and once the word is cleared the same call must run
clean with the right result.
"""
import time

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

# umma.cuh: operand stage never filled / never released / accumulator never completed.
# Every role of the stuck CTA is waiting; whichever wait began first expires first (the
# epilogue's, on the accumulator) and the others then see the word and end.
FAULT_FULL, FAULT_EMPTY, FAULT_DONE = 1, 2, 4


def test_bounded_wait_expires_then_recovers(torch_cuda):
    torch = torch_cuda
    import demucs_cuda_b200 as dcb
    rng = np.random.default_rng(9)
    M, N, K = 256, 256, 4096   # 64 K blocks per tile: more than the operand ring holds
    A = rng.standard_normal((M, K)).astype(np.float16)
    B = rng.standard_normal((N, K)).astype(np.float16)
    want = A.astype(np.float64) @ B.astype(np.float64).T
    At, Bt = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    assert dcb.device_fault() == 0
    limit0 = dcb.set_option("wait_limit_ms", 200)
    assert limit0 == 2000
    try:
        dcb.set_option("test_withhold_arrive", 1)
        t0 = time.time()
        dcb.gemm_half(At, Bt)
        torch.cuda.synchronize()   # returns: the waits gave up instead of hanging
        dt = time.time() - t0
        fault = dcb.device_fault(clear=False)
        print(f"withheld stage: kernel returned after {dt:.2f} s, fault word {fault:#x}")
        assert fault & (FAULT_FULL | FAULT_EMPTY | FAULT_DONE), fault
        assert dt < 30
        # the hook is one-shot: it was consumed by the faulting launch
        assert dcb.set_option("test_withhold_arrive", 0) == 0
        # while the word is set, later launches of the library end at once
        C_ = torch.full((1, M, N), 7.0, device="cuda")
        dcb.gemm_half(At, Bt, C_)
        torch.cuda.synchronize()
        assert (C_ == 7.0).all()
        assert dcb.device_fault(clear=True) == fault
        assert dcb.device_fault() == 0
    finally:
        dcb.set_option("test_withhold_arrive", 0)
        dcb.set_option("wait_limit_ms", limit0)
        dcb.device_fault(clear=True)   # never leave the word set for later tests
    got = dcb.gemm_half(At, Bt)
    torch.cuda.synchronize()
    assert rel_l2(got.cpu().numpy()[0], want) < 2e-5
    assert dcb.device_fault() == 0
