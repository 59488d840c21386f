"""Allocation-free split-K GEMM entry point, called through its exported C symbol.

The C entry point ``nsb_gemm_bf16_splitk_noalloc`` (csrc/include/gemm_noalloc.h)
keeps its split-K scratch in static device memory. Its output must match the torch
binding of the same kernel (``gemm_test`` with the same forced split count) on two
consecutive calls: the second call checks that the first left the arrival counters
at zero. This file is collected last so that it also runs after every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")

LL = ctypes.c_longlong


def _lib():
    import nanospec_b200._C as ext
    lib = ctypes.CDLL(ext.__file__)  # the already-loaded extension library
    f = lib.nsb_gemm_bf16_splitk_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, LL, LL, LL, ctypes.c_void_p, ctypes.c_int, LL, LL, LL,
                  ctypes.c_void_p, LL, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.nsb_gemm_noalloc_error.restype = ctypes.c_char_p
    lib.nsb_gemm_noalloc_setup.argtypes = [ctypes.c_int]
    lib.nsb_gemm_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
    return lib


def _call(lib, a, a_mn, b, b_mn, out, M, N, K, splits):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.nsb_gemm_bf16_splitk_noalloc(a.data_ptr(), int(a_mn), a.size(0), a.size(1), a.stride(0),
                                            b.data_ptr(), int(b_mn), b.size(0), b.size(1), b.stride(0),
                                            out.data_ptr(), out.stride(0), M, N, K, splits, stream)


@cuda
@pytest.mark.parametrize("M,N,K,a_mn,b_mn,splits", [
    (512, 56, 2048, False, False, 4),    # swap-AB-like small N, K-major operands
    (256, 128, 1024, True, False, 3),    # MN-major A
    (384, 192, 1536, False, True, 2),    # MN-major B, 192-wide tiles
    (300, 40, 640, False, False, 1),     # no split, ragged M and N
])
def test_noalloc_gemm_matches_torch_entry(M, N, K, a_mn, b_mn, splits):
    from nanospec_b200.ops._ext import cuda_ops
    C = cuda_ops()
    lib = _lib()
    assert lib.nsb_gemm_noalloc_setup(torch.cuda.current_device()) == 0, lib.nsb_gemm_noalloc_error()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", generator=g).bfloat16()
    b = torch.randn((K, N) if b_mn else (N, K), device="cuda", generator=g).bfloat16()
    ref = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm_test(a, a_mn, b, b_mn, ref, splits)
    af = a.float().t() if a_mn else a.float()
    bf = b.float().t() if b_mn else b.float()
    exact = af @ bf.t()
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    for _ in range(2):
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        torch.cuda.synchronize()
        rc = _call(lib, a, a_mn, b, b_mn, out, M, N, K, splits)
        assert rc == 0, lib.nsb_gemm_noalloc_error()
        torch.cuda.synchronize()
        st = ctypes.c_int(-1)
        assert lib.nsb_gemm_noalloc_status(ctypes.byref(st)) == 0 and st.value == 0
        torch.testing.assert_close(out.float(), ref.float(), rtol=0, atol=0)
        err = (out.float() - exact).abs().max().item()
        assert err <= 2e-2 * exact.abs().max().item(), err
        del out
    assert torch.cuda.memory_allocated() == before


@cuda
def test_noalloc_gemm_rejects_oversized_scratch():
    lib = _lib()
    M, N, K = 4096, 256, 4096  # 8 splits x 4096 x 256 floats = 32 MiB > 4 MiB scratch
    a = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    rc = _call(lib, a, False, b, False, out, M, N, K, 8)
    assert rc == 2
    assert b"scratch holds at most" in lib.nsb_gemm_noalloc_error()
    assert _call(lib, a, False, b, False, out, M, N, K, 17) == 1


def _raw(lib, ptr, a_mn, a_rows, a_cols, a_ld, b_mn, b_rows, b_cols, b_ld, out_ptr, out_ld, M, N, K, splits):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.nsb_gemm_bf16_splitk_noalloc(ptr, a_mn, a_rows, a_cols, a_ld, ptr, b_mn, b_rows, b_cols, b_ld,
                                            out_ptr, out_ld, M, N, K, splits, stream)


@cuda
def test_noalloc_gemm_argument_checks_launch_nothing():
    """Arguments the entry point must refuse before it builds a tensor map or
    launches: these calls only pass sizes (the buffer is far smaller than the
    sizes claim, which is safe because nothing is read)."""
    lib = _lib()
    buf = torch.zeros(4096, device="cuda", dtype=torch.bfloat16)
    p = buf.data_ptr()
    # more than NSB_GEMM_NOALLOC_MAX_TILES tiles in a split launch: 4097 tiles of 128 x 64, 2 splits
    M = 128 * 4097
    assert _raw(lib, p, 0, M, 256, 256, 0, 64, 256, 256, p, 64, M, 64, 256, 2) == 2
    assert b"exceed the maximum" in lib.nsb_gemm_noalloc_error()
    # output misaligned by 2 bytes
    assert _raw(lib, p, 0, 128, 64, 64, 0, 64, 64, 64, p + 2, 64, 128, 64, 64, 1) == 1
    assert b"16-byte aligned" in lib.nsb_gemm_noalloc_error()
    # a_rows != M
    assert _raw(lib, p, 0, 127, 64, 64, 0, 64, 64, 64, p, 64, 128, 64, 64, 1) == 1
    assert b"shapes do not match" in lib.nsb_gemm_noalloc_error()
    # row stride shorter than the row
    assert _raw(lib, p, 0, 128, 64, 32, 0, 64, 64, 64, p, 64, 128, 64, 64, 1) == 1
    assert _raw(lib, p, 0, 128, 64, 64, 0, 64, 64, 56, p, 64, 128, 64, 64, 1) == 1
    assert b"row stride smaller" in lib.nsb_gemm_noalloc_error()
    # null operand
    assert lib.nsb_gemm_bf16_splitk_noalloc(None, 0, 128, 64, 64, p, 0, 64, 64, 64, p, 64, 128, 64, 64, 1,
                                            None) == 1
    # reset, then the status word reads zero
    assert lib.nsb_gemm_noalloc_reset(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    st = ctypes.c_int(-1)
    assert lib.nsb_gemm_noalloc_status(ctypes.byref(st)) == 0 and st.value == 0


@cuda
def test_noalloc_gemm_unsplit_has_no_tile_limit():
    """An unsplit product uses no scratch: more tiles than the counter area holds
    still runs, and matches the torch entry (which may pick another tile plan for
    this many tiles) and the fp32 product."""
    from nanospec_b200.ops._ext import cuda_ops
    lib = _lib()
    M, N, K = 128 * 4097, 64, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    ref = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ops().gemm_test(a, False, b, False, ref, 1)
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    assert _call(lib, a, False, b, False, out, M, N, K, 1) == 0, lib.nsb_gemm_noalloc_error()
    exact = a.float() @ b.float().t()
    torch.cuda.synchronize()
    scale = exact.abs().max().item()
    assert (out.float() - ref.float()).abs().max().item() <= 1e-2 * scale
    assert (out.float() - exact).abs().max().item() <= 2e-2 * scale
