"""The allocation-free C entry point ``r9k_gemm_bf16_noalloc`` against the torch op ``r9k::gemm_bf16``.

Collected last on purpose: the entry point's scratch lives in one device array shared by every call,
so it is exercised both in a fresh process and after the rest of the suite has run kernels.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from r9700_stack_b200 import _native

    _native.ops()  # builds if stale and loads the library into this process
    lib = ctypes.CDLL(_native.lib_path())
    fn = lib.r9k_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                   ctypes.c_void_p]
    return fn


def _call(fn, w, x, out, alpha, status):
    N, K = w.shape
    M = x.shape[0]
    return fn(w.data_ptr(), w.stride(0), x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), N, M, K,
              alpha, status.data_ptr() if status is not None else None, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("N,M,K", [(5120, 1, 5120), (2048, 16, 4096), (768, 40, 2048), (1000, 7, 320)])
def test_noalloc_matches_torch_op(N, M, K):
    from r9700_stack_b200 import _native

    fn = _lib()
    torch.manual_seed(N + M)
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    x = torch.randn(M, K, device="cuda").bfloat16()
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(1 << 22, dtype=torch.float32, device="cuda")
    _native.ops().gemm_bf16(w, x, ref, None, 0.5, status, ws)
    fp32 = (x.float() @ w.float().T) * 0.5
    for _ in range(2):  # two calls in a row: the scratch counters must come back to zero
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _call(fn, w, x, out, 0.5, status) == 0
        torch.cuda.synchronize()
        assert int(status[0]) == 0, status.tolist()
        torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(out.float(), fp32, rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_oversize():
    fn = _lib()
    w = torch.zeros(256, 128, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(65, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(65, 256, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert _call(fn, w, x, out, 1.0, status) == -2  # R9K_NOALLOC_ETOOLARGE: M > 64
    bad = torch.zeros(8, 96, dtype=torch.bfloat16, device="cuda")
    assert _call(fn, w[:, :96], bad, out, 1.0, status) == -1  # K not a multiple of 64


@pytest.mark.parametrize("pad", [8, 64])
def test_noalloc_padded_strides_without_status(pad):
    """Row strides wider than the rows (ldw > K, ldx > K, ldo > N) and no status word; the weights
    are written by the kernel immediately before the call on the same stream."""
    from r9700_stack_b200 import _native

    fn = _lib()
    N, M, K = 1536, 12, 1024
    torch.manual_seed(pad)
    wbig = torch.zeros(N, K + pad, dtype=torch.bfloat16, device="cuda")
    xbig = torch.randn(M, K + pad, device="cuda").bfloat16()
    obig = torch.full((M, N + pad), 7.0, dtype=torch.bfloat16, device="cuda")
    src = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    w, x, out = wbig[:, :K], xbig[:, :K], obig[:, :N]
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(1 << 22, dtype=torch.float32, device="cuda")
    _native.ops().gemm_bf16(src, x.contiguous(), ref, None, 1.0, status, ws)
    for _ in range(2):
        wbig.zero_()
        w.copy_(src)  # the producing kernel runs right before the GEMM on this stream
        assert _call(fn, w, x, out, 1.0, None) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)
        assert bool((obig[:, N:] == 7.0).all()), "wrote past the output rows"


def test_noalloc_rejects_misaligned_output():
    fn = _lib()
    w = torch.zeros(256, 128, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    obig = torch.zeros(4 * 256 + 8, dtype=torch.bfloat16, device="cuda")
    out = obig[1:1 + 4 * 256].view(4, 256)  # 2-byte offset: not 16-byte aligned
    assert _call(fn, w, x, out, 1.0, None) == -1
    out2 = torch.zeros(4, 260, dtype=torch.bfloat16, device="cuda")[:, :256]  # ldo = 260: not a multiple of 8
    assert _call(fn, w, x, out2, 1.0, None) == -1


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second visible GPU")
def test_noalloc_second_device():
    """The first call on another device sets that device up (its own scratch address)."""
    from r9700_stack_b200 import _native

    fn = _lib()
    with torch.cuda.device(1):
        N, M, K = 1024, 8, 512
        w = (torch.randn(N, K, device="cuda:1") * 0.05).bfloat16()
        x = torch.randn(M, K, device="cuda:1").bfloat16()
        status = torch.zeros(4, dtype=torch.int32, device="cuda:1")
        ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda:1")
        ws = torch.zeros(1 << 22, dtype=torch.float32, device="cuda:1")
        _native.ops().gemm_bf16(w, x, ref, None, 1.0, status, ws)
        for _ in range(2):
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda:1")
            assert _call(fn, w, x, out, 1.0, status) == 0
            torch.cuda.synchronize(1)
            assert int(status[0]) == 0
            torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)
