"""The allocation-free GEMM entry point (tsfm_sgemm_nt_noalloc), called through the C ABI.

Some callers of this library cannot allocate device memory while running (cudaMalloc/cudaFree
synchronise the whole device; real-time loops forbid allocation after start-up; a process-wide
pool may own all device memory). For them the library keeps its scratch in a fixed array of its
own. This test checks, on two calls in a row, that the allocation-free entry point returns what
the ordinary seam entry point tsfm_sgemm_nt returns (same 1e-4 tolerance as the seam's own test),
that device free memory does not change across a call once the first call has set the array up,
that strided operands leave the padding of C untouched, and that the size limit holds exactly on
both sides of its boundary (a product too large for the array is rejected rather than run).

The file is named to be collected last, so a run that stops at the first failure has already run
every other test; it passes alone in a fresh process as well.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsfm_b200 as tb  # noqa: E402

pytestmark = pytest.mark.gpu


def seam(A, B, alpha):
    """tsfm_sgemm_nt on host copies (the existing entry point)."""
    m, k = A.shape
    n = B.shape[0]
    a = np.ascontiguousarray(A.cpu().numpy())
    b = np.ascontiguousarray(B.cpu().numpy())
    c = np.zeros((m, n), np.float32)
    assert tb.lib.tsfm_sgemm_nt(m, n, k, alpha, a.ctypes.data, k, b.ctypes.data, k, c.ctypes.data, n, None) == 0
    return c


def noalloc(A, B, C, alpha, stream):
    m, k = A.shape
    n = B.shape[0]
    return tb.lib.tsfm_sgemm_nt_noalloc(m, n, k, alpha, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0),
                                        C.data_ptr(), C.stride(0), stream)


def test_noalloc_matches_seam_on_two_calls_in_a_row():
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(1234)
    # Both calls use the same kernel instances (N <= 128 tiles), so the second call cannot load
    # new device code either.
    shapes = [(37, 29, 23, 0.7), (300, 100, 257, 1.0)]
    for call, (m, n, k, alpha) in enumerate(shapes):
        A = (torch.rand(m, k, generator=g) * 2 - 1).to(dev)
        B = (torch.rand(n, k, generator=g) * 2 - 1).to(dev)
        C = torch.full((m, n), float("nan"), device=dev)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = noalloc(A, B, C, alpha, stream)
        free_after = torch.cuda.mem_get_info()[0]
        assert st == 0, tb.last_error()
        if call > 0:
            assert free_after == free_before  # nothing allocated once set up
        want = seam(A, B, alpha)
        np.testing.assert_allclose(C.cpu().numpy(), want, atol=1e-4)
        ref = alpha * (A.double() @ B.double().T)
        assert (C.double() - ref).abs().max().item() <= 1e-4


def test_noalloc_strided_operands_keep_padding():
    # Row strides above the logical widths: lda, ldb > k and ldc > n (a multiple of 4, so the
    # output goes through the TMA-store epilogue). The padding columns of C hold NaN sentinels that
    # must survive; the padding of A and B holds NaN that must never be read.
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(99)
    m, n, k, lda, ldb, ldc = 200, 72, 100, 112, 104, 80
    Ab = torch.full((m, lda), float("nan"))
    Bb = torch.full((n, ldb), float("nan"))
    Ab[:, :k] = torch.rand(m, k, generator=g) * 2 - 1
    Bb[:, :k] = torch.rand(n, k, generator=g) * 2 - 1
    Ab, Bb = Ab.to(dev), Bb.to(dev)
    Cb = torch.full((m, ldc), float("nan"), device=dev)
    st = tb.lib.tsfm_sgemm_nt_noalloc(m, n, k, 1.0, Ab.data_ptr(), lda, Bb.data_ptr(), ldb, Cb.data_ptr(), ldc,
                                      stream)
    assert st == 0, tb.last_error()
    ref = Ab[:, :k].double() @ Bb[:, :k].double().T
    assert (Cb[:, :n].double() - ref).abs().max().item() <= 1e-4
    assert torch.isnan(Cb[:, n:]).all()


def test_noalloc_limit_on_both_sides_of_the_boundary():
    # k = 64: the four split parts take (m + n) * 64 floats each pair, and the array holds
    # 2^21 - 64 floats of parts: m + n = 32767 is the largest product that fits.
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=dev).manual_seed(5)
    k, n = 64, 767
    for m, ok in ((32000, True), (32001, False)):
        A = torch.rand(m, k, device=dev, generator=g) * 2 - 1
        B = torch.rand(n, k, device=dev, generator=g) * 2 - 1
        C = torch.zeros(m, n, device=dev)
        st = tb.lib.tsfm_sgemm_nt_noalloc(m, n, k, 1.0, A.data_ptr(), k, B.data_ptr(), k, C.data_ptr(), n, stream)
        if ok:
            assert st == 0, tb.last_error()
            ref = A.double() @ B.double().T
            assert (C.double() - ref).abs().max().item() <= 1e-4
        else:
            assert tb.STATUS_NAMES[st] == "INVALID_ARGUMENT"
            assert "scratch limit" in tb.last_error()


def test_noalloc_rejects_products_beyond_its_scratch():
    dev = torch.device("cuda:0")
    m, n, k = 2048, 2048, 1024  # (m + n) * k = 4M floats > 2M
    A = torch.zeros(m, k, device=dev)
    B = torch.zeros(n, k, device=dev)
    C = torch.zeros(m, n, device=dev)
    st = noalloc(A, B, C, 1.0, torch.cuda.current_stream().cuda_stream)
    assert tb.STATUS_NAMES[st] == "INVALID_ARGUMENT"
    assert "scratch limit" in tb.last_error()
