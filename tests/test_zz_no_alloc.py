"""The allocation-free matmul_dw entry point (rnn_gemm_dw_noalloc_dev).

It exists for callers that may not allocate device memory — a framework that
keeps every byte of device memory in its own pool, or a loop that cannot pay
cudaMalloc's implicit synchronisation — so it takes no context and keeps its
split-K partial sums in a fixed device array inside the library.  This test
drives it through the C ABI and compares it with the CPU oracle's matmul_dw
(gemm.rs:555-598) and with the allocating entry point (rnn_gemm_dw_dev) on
two calls in a row: the second call must not be disturbed by what the first
left in the shared array.  After every call the status query must report no
kernel timeout.  The file sorts last so a run that stops at its first failure
has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-4  # relative Frobenius, the bar of every parity test here
LIMIT = 2_097_152  # largest m*n the entry accepts (half its 16-MiB scratch)


def rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want))


# (1024, 1152, 4096) runs two K splits whose partial planes fill 2.36 M of the
# array's 4.19 M floats; (2048, 1024, 512) is m*n at the limit exactly.
@pytest.mark.parametrize("m,n,k", [(768, 256, 8192), (37, 29, 3000), (1024, 1152, 4096), (2048, 1024, 512)])
def test_noalloc_matches_oracle_two_calls(m, n, k):
    from rustnn_b200 import _lib, ops

    L = _lib.lib()
    rng = O.Rng(m * 7 + n * 3 + k)
    a = rng.rand_vec(k * m)
    b = rng.rand_vec(k * n)
    c0 = rng.rand_vec(m * n)
    want = c0.copy()
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    got = torch.from_numpy(c0).cuda()
    alloc = got.clone()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        want = O.matmul_dw(m, n, k, a, b, want)  # C += A^T B on the CPU
        ops.matmul_dw(m, n, k, ad, bd, alloc)  # the allocating entry point
        code = L.rnn_gemm_dw_noalloc_dev(m, n, k, C.c_void_p(ad.data_ptr()), C.c_void_p(bd.data_ptr()),
                                         C.c_void_p(got.data_ptr()), stream)
        assert code == 0, L.rnn_last_error()
        assert L.rnn_gemm_dw_noalloc_status(stream) == 0, L.rnn_last_error()
        g = got.cpu().numpy()
        assert rel(g, want) < TOL, (call, rel(g, want))
        assert rel(g, alloc.cpu().numpy()) < TOL, (call, rel(g, alloc.cpu().numpy()))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from rustnn_b200 import _lib

    L = _lib.lib()
    x = torch.zeros(4, device="cuda")
    p = C.c_void_p(x.data_ptr())
    code = L.rnn_gemm_dw_noalloc_dev(LIMIT + 1, 1, 8, p, p, p, None)  # one element past the limit
    assert code == -1
    assert b"limit" in L.rnn_last_error()
    code = L.rnn_gemm_dw_noalloc_dev(4096, 1024, 8, p, p, p, None)
    assert code == -1
    assert L.rnn_gemm_dw_noalloc_status(None) == 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_on_a_second_device_after_the_first():
    """The entry's per-device state (the scratch array's address, each tile
    width's shared-memory opt-in) is set up again for device 1 after device
    0 in the same process."""
    from rustnn_b200 import _lib

    L = _lib.lib()
    m, n, k = 768, 256, 8192
    rng = O.Rng(11)
    a, b, c0 = rng.rand_vec(k * m), rng.rand_vec(k * n), rng.rand_vec(m * n)
    want = O.matmul_dw(m, n, k, a, b, c0.copy())
    for dev in (0, 1):
        with torch.cuda.device(dev):
            ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
            got = torch.from_numpy(c0).cuda()
            stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            code = L.rnn_gemm_dw_noalloc_dev(m, n, k, C.c_void_p(ad.data_ptr()), C.c_void_p(bd.data_ptr()),
                                             C.c_void_p(got.data_ptr()), stream)
            assert code == 0, L.rnn_last_error()
            assert L.rnn_gemm_dw_noalloc_status(stream) == 0, L.rnn_last_error()
            assert rel(got.cpu().numpy(), want) < TOL, dev
