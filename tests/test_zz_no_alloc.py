"""The allocation-free matmul_dw entry point (rnn_gemm_dw_noalloc_dev).

It exists for callers that may not allocate device memory — a framework that
keeps every byte of device memory in its own pool, or a loop that cannot pay
cudaMalloc's implicit synchronisation — so it takes no context and keeps its
split-K partial sums in a fixed device array inside the library.  This test
drives it through the C ABI and compares it with the allocating entry point
(rnn_gemm_dw_dev) on two calls in a row: the second call must not be disturbed
by what the first left in the shared array.  The file sorts last so a run that
stops at its first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-4  # relative Frobenius, the bar of every parity test here


def rel(got, want):
    got = got.double().cpu().numpy()
    want = want.double().cpu().numpy()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want))


@pytest.mark.parametrize("m,n,k", [(768, 256, 8192), (37, 29, 3000)])
def test_noalloc_matches_allocating_entry_two_calls(m, n, k):
    from rustnn_b200 import _lib, ops

    L = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(k * m, device="cuda", generator=g)
    b = torch.randn(k * n, device="cuda", generator=g)
    c0 = torch.randn(m * n, device="cuda", generator=g)
    want = c0.clone()
    got = c0.clone()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        ops.matmul_dw(m, n, k, a, b, want)  # existing entry point, C += A^T B
        code = L.rnn_gemm_dw_noalloc_dev(m, n, k, C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()),
                                         C.c_void_p(got.data_ptr()), stream)
        assert code == 0, L.rnn_last_error()
        torch.cuda.synchronize()
        assert rel(got, want) < TOL, (call, rel(got, want))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from rustnn_b200 import _lib

    L = _lib.lib()
    x = torch.zeros(4, device="cuda")
    p = C.c_void_p(x.data_ptr())
    code = L.rnn_gemm_dw_noalloc_dev(4096, 1024, 8, p, p, p, None)  # m*n beyond the limit
    assert code == -1
    assert b"limit" in L.rnn_last_error()
