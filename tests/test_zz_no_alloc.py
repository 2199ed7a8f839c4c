"""The allocation-free C entry point of the split-K GEMM
(``b200_gemm_bf16_noalloc`` in csrc/gemm/gemm_noalloc.cu), called through
ctypes exactly as a C caller would, against the workspace-backed torch op and
an fp32 torch reference. Named so that it is collected after every other test
file: it must also pass after the rest of the suite has used the kernels."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, EINVAL, ETOOBIG = 0, 1, 2


def _lib():
    from vllm_sm70_b200 import _ext

    lib = ctypes.CDLL(str(_ext.SO_PATH))
    f = lib.b200_gemm_bf16_noalloc
    f.restype = ctypes.c_int
    i, p = ctypes.c_int, ctypes.c_void_p
    f.argtypes = [p, i, p, i, p, i, i, i, i, i, i, p]
    lib.b200_gemm_bf16_noalloc_last_error.restype = ctypes.c_char_p
    lib.b200_gemm_bf16_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    return lib


def _call(lib, out, a, w, cfg, splits):
    M, K = a.shape
    N = w.shape[0]
    return lib.b200_gemm_bf16_noalloc(a.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), N, M, N, K,
                                      cfg, splits, torch.cuda.current_stream().cuda_stream)


# (M, N, K, cfg, splits): swap-AB 16 x4 splits, swap-AB 32 with a ragged M,
# a plain 128x128 tile without split.
CASES = [(64, 2048, 4096, 2, 4), (200, 1024, 2048, 3, 2), (256, 4096, 1024, 1, 1)]


@pytest.mark.parametrize("M,N,K,cfg,splits", CASES)
def test_noalloc_matches_workspace_entry_point(b200_ops, M, N, K, cfg, splits):
    lib = _lib()
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ref_ws = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    b200_ops.gemm_bf16_out(ref_ws, a, w, cfg, splits)
    ref32 = a.float() @ w.float().t()
    for _ in range(2):  # two calls in a row: the counters re-arm between them
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc = _call(lib, out, a, w, cfg, splits)
        assert rc == OK, lib.b200_gemm_bf16_noalloc_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref_ws, atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(out.float(), ref32, atol=5e-2, rtol=2e-2)
    st = ctypes.c_uint(123)
    assert lib.b200_gemm_bf16_noalloc_status(ctypes.byref(st)) == OK
    assert st.value == 0


def test_noalloc_rejects_oversized_split(b200_ops):
    lib = _lib()
    M, N, K = 256, 8192, 4096  # swap-AB 32 x 8 splits: 64 MiB of partials > static region
    a = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), 7.0, device="cuda", dtype=torch.bfloat16)
    assert _call(lib, out, a, w, 3, 8) == ETOOBIG
    assert b"too small" in lib.b200_gemm_bf16_noalloc_last_error()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.b200_gemm_bf16_noalloc(a.data_ptr(), K, w.data_ptr(), K, out.data_ptr(), N, M, N, 100,
                                    3, 1, stream)  # K not a multiple of 8
    assert rc == EINVAL
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched


def test_noalloc_on_two_devices(b200_ops):
    """One process driving two GPUs: the entry point's per-device set-up (the
    static scratch address and the kernel's shared-memory limit) must run on
    each device, so the second device's calls succeed as well."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    lib = _lib()
    M, N, K, cfg, splits = 64, 2048, 4096, 2, 4
    prev = torch.cuda.current_device()
    try:
        for dev in (0, 1, 0, 1):
            torch.cuda.set_device(dev)
            g = torch.Generator(device="cuda").manual_seed(11 + dev)
            a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
            w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
            out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
            rc = _call(lib, out, a, w, cfg, splits)
            assert rc == OK, (dev, lib.b200_gemm_bf16_noalloc_last_error())
            torch.cuda.synchronize()
            torch.testing.assert_close(out.float(), a.float() @ w.float().t(), atol=5e-2, rtol=2e-2)
            st = ctypes.c_uint(123)
            assert lib.b200_gemm_bf16_noalloc_status(ctypes.byref(st)) == OK
            assert st.value == 0
    finally:
        torch.cuda.set_device(prev)
