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
              alpha, status.data_ptr(), torch.cuda.current_stream().cuda_stream)


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
