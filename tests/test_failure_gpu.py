"""Failure detection on the GPU without a GPU fault: a bounded device wait
runs out on a barrier that nothing ever arrives at, the kernel returns, the
host reads the timeout from the status and the device error word, and the
context stays usable. The wait is the same helper every hand-off in the GEMM,
decode and MoE kernels uses; only its limit is shortened (1 ms instead of 2 s).
The reference has no device-side waits; its failure handling is per-case
exception capture (kernelevalplus-main/llm_kernel_test/unified_test_runner.py:454-461)."""
import time

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu

KQ_ERR_INVALID, KQ_ERR_TIMEOUT = 1, 5
DEV_TIMEOUT_FULL = 1


def test_bounded_wait_gives_up(cuda):
    import kq
    from kq import _lib
    kq.device_error()  # start from a clear error word
    L = kq.lib()
    s = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    st = L.kq_selftest_wait_timeout(1_000_000, s)
    dt = time.perf_counter() - t0
    assert st == KQ_ERR_TIMEOUT, (st, _lib.last_error())
    assert "gave up" in _lib.last_error()
    assert dt < 1.0, f"a 1 ms device wait took {dt:.3f} s to give up"
    assert kq.device_error() == DEV_TIMEOUT_FULL
    assert kq.device_error() == 0  # read clears it
    # the context is still usable: an operator afterwards is correct
    rng = np.random.default_rng(3)
    M, N, K = 4, 256, 512
    w = Q.make_blocks("q4_0", rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    got = kq.gemm_f32act(torch.from_numpy(w).to(cuda), torch.from_numpy(x).to(cuda), M, N, K, "q4_0", "f32")
    ok, msg = Q.check_close(got.cpu().numpy(), Q.gemm_f32act("q4_0", w, x, M, N, K, Q.ACT_F32))
    assert ok, msg
    assert kq.device_error() == 0


@pytest.mark.parametrize("limit_ns", [0, -5, 3_000_000_000])
def test_bounded_wait_limit_checked(cuda, limit_ns):
    import kq
    st = kq.lib().kq_selftest_wait_timeout(limit_ns, torch.cuda.current_stream().cuda_stream)
    assert st == KQ_ERR_INVALID
