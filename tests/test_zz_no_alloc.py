"""The allocation-free GEMM entry point (kq_gemm_f32act_noalloc).

Some callers cannot call cudaMalloc: a serving runtime whose allocator has
already reserved nearly all of HBM, or a latency-critical step that must not
synchronise the device on a first-call allocation. This entry point stages the
quantised activations in a fixed 1 MiB __device__ array instead. The test calls
it through the C ABI twice in a row (different inputs, so a stale staging
buffer would show) and checks each result against the oracle with the bar the
other tests use. For GEMV shapes (M <= 8) both entry points run the same
kernel, so the result must also equal kq_gemm_f32act's bit for bit; for
M > 8 the allocating entry point runs the split-fp16 kernel (its fp16
operands need workspace) while this one runs the int8 tensor-core kernel, so
the two agree to the parity bar, not bitwise. It lives in its own file,
collected last, and passes alone or after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _call(fn, wtype, w, x, M, N, K, mode):
    import kq
    out = torch.empty((M, N), dtype=torch.float32, device=w.device)
    st = fn(kq.WTYPES[wtype], w.data_ptr(), x.data_ptr(), out.data_ptr(), M, N, K, kq.ACT_MODES[mode],
            torch.cuda.current_stream().cuda_stream)
    assert st == 0, kq._lib.last_error()
    return out


@pytest.mark.parametrize("wtype,M,N,K", [("q4_0", 1, 4096, 4096), ("q8_0", 8, 1000, 2048), ("q4_1", 40, 384, 1024),
                                         ("q8_0", 128, 256, 4096)])
def test_noalloc_matches_allocating_entry(cuda, wtype, M, N, K):
    import kq
    L = kq.lib()
    rng = np.random.default_rng(M + N)
    w = _dev(Q.make_blocks(wtype, rng, N, K), cuda)
    for call in range(2):  # two calls in a row: the shared array keeps the previous call's contents
        xh = rng.standard_normal((M, K)).astype(np.float32) * (1 + call)
        x = _dev(xh, cuda)
        got = _call(L.kq_gemm_f32act_noalloc, wtype, w, x, M, N, K, "f32")
        alloc = _call(L.kq_gemm_f32act, wtype, w, x, M, N, K, "f32")
        torch.cuda.synchronize()
        ref = Q.gemm_f32act(wtype, w.cpu().numpy(), xh, M, N, K, Q.ACT_F32)
        for name, t in (("noalloc", got), ("allocating", alloc)):
            ok, msg = Q.check_close(t.cpu().numpy(), ref)
            assert ok, f"call {call} {name}: {msg}"
        ok, msg = Q.check_close(got.cpu().numpy(), alloc.cpu().numpy())  # the two entry points, directly
        assert ok, f"call {call} noalloc vs kq_gemm_f32act: {msg}"
        if M <= 8:
            assert torch.equal(got, alloc), f"call {call}: not bit-identical to kq_gemm_f32act"
        # the no-alloc kernels record wait timeouts in a word of their own
        code = ctypes.c_int(-1)
        assert L.kq_noalloc_device_error(ctypes.byref(code), torch.cuda.current_stream().cuda_stream) == 0
        assert code.value == 0, f"call {call}: no-alloc device error word {code.value}"
    assert kq.device_error() == 0


def test_noalloc_rejects_oversize(cuda):
    import kq
    L = kq.lib()
    M, N, K = 512, 64, 4096  # staging 2.5 MiB > 1 MiB
    w = torch.zeros(N * (K // 32) * 18, dtype=torch.uint8, device=cuda)
    x = torch.zeros((M, K), dtype=torch.float32, device=cuda)
    out = torch.empty((M, N), dtype=torch.float32, device=cuda)
    st = L.kq_gemm_f32act_noalloc(0, w.data_ptr(), x.data_ptr(), out.data_ptr(), M, N, K, 2, None)
    assert st == 1
    assert "exceeds the fixed" in kq._lib.last_error()
