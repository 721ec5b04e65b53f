"""The exported no-allocation grouped-GEMM C entry point against the ordinary
entry point (``revealaiccl_b200.ops.grouped_gemm``), called through ctypes.

Collected last on purpose (file name): it must also pass after every other
GPU test has run in the same process."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from revealaiccl_b200.ops._native import kernels

    lib = ctypes.CDLL(kernels().__file__)
    f = lib.raiccl_grouped_gemm_noalloc
    f.restype = ctypes.c_int
    ll, i, p = ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p
    f.argtypes = [i, p, ll, ll, ll, p, ll, ll, p, i, i, i, i, p, p, p, p, ll, i, i, ctypes.c_ulonglong, p]
    lib.raiccl_grouped_gemm_noalloc_status.restype = ctypes.c_int
    lib.raiccl_grouped_gemm_noalloc_status.argtypes = [p, p]
    lib.raiccl_grouped_gemm_noalloc_max_segments.restype = ctypes.c_int
    lib.raiccl_grouped_gemm_noalloc_error_string.restype = ctypes.c_char_p
    lib.raiccl_grouped_gemm_noalloc_error_string.argtypes = [ctypes.c_int]
    return lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call(lib, A, B, segs, n, bn, act, bias, row_scale, out, stream):
    return lib.raiccl_grouped_gemm_noalloc(
        0 if A.dtype == torch.bfloat16 else 1, _ptr(A), A.shape[0], A.shape[1], A.stride(0),
        _ptr(B), B.shape[0], B.stride(0), _ptr(segs), segs.shape[0], n, bn, act,
        _ptr(bias), None, _ptr(row_scale), _ptr(out), out.stride(0), int(out.dtype == torch.bfloat16),
        0, 0, ctypes.c_void_p(stream.cuda_stream))


def _case(seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    E, n, k = 3, 128, 512
    rows = [130, 0, 257]
    m = sum(rows)
    A = torch.randn(m, k, generator=g).bfloat16().to(dev)
    B = (torch.randn(E * n, k, generator=g) / k ** 0.5).bfloat16().to(dev)
    bias = (torch.randn(E * n, generator=g) * 0.1).to(dev)
    scale = torch.rand(m, generator=g).to(dev)
    segs_list, a0 = [], 0
    for e, r in enumerate(rows):
        segs_list.append((a0, r, (e + seed) % E, 0, a0))
        a0 += r
    return A, B, bias, scale, segs_list, n


def test_noalloc_matches_entry_point_twice():
    from revealaiccl_b200.ops import grouped_gemm as gg

    lib = _lib()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream(dev)
    for seed in (0, 1):  # two calls in a row reuse the same device scratch
        A, B, bias, scale, segs_list, n = _case(seed, dev)
        segs = gg.make_segments(segs_list, dev)
        ref = torch.zeros(A.shape[0], n, device=dev)
        gg.grouped_gemm(A, B, segs, n=n, act="gelu", bias=bias, row_scale=scale, out=ref, bn=64, check=True)
        out = torch.full((A.shape[0], n), float("nan"), device=dev)
        rc = _call(lib, A, B, segs, n, 64, gg.ACT_IDS["gelu"], bias, scale, out, stream)
        assert rc == 0, lib.raiccl_grouped_gemm_noalloc_error_string(rc)
        st = (ctypes.c_int * 8)()
        assert lib.raiccl_grouped_gemm_noalloc_status(ctypes.cast(st, ctypes.c_void_p),
                                                      ctypes.c_void_p(stream.cuda_stream)) == 0
        torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)


def test_noalloc_rejects_oversize_and_bad_slot():
    from revealaiccl_b200.ops import grouped_gemm as gg

    lib = _lib()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream(dev)
    cap = lib.raiccl_grouped_gemm_noalloc_max_segments()
    A, B, bias, scale, segs_list, n = _case(2, dev)
    out = torch.zeros(A.shape[0], n, device=dev)
    big = gg.make_segments([(0, 0, 0, 0, 0)] * (cap + 1), dev)
    rc = _call(lib, A, B, big, n, 64, 0, None, None, out, stream)
    assert rc == -1 and b"1024" in lib.raiccl_grouped_gemm_noalloc_error_string(rc)
    bad = gg.make_segments([(0, 4, 0, 1, 0)], dev)  # out_slot 1: only slot 0 exists here
    assert _call(lib, A, B, bad, n, 64, 0, None, None, out, stream) == 0
    assert lib.raiccl_grouped_gemm_noalloc_status(None, ctypes.c_void_p(stream.cuda_stream)) == 5
    assert torch.count_nonzero(out) == 0
    # the next good call starts from a clean status
    segs = gg.make_segments(segs_list, dev)
    ref = torch.zeros(A.shape[0], n, device=dev)
    gg.grouped_gemm(A, B, segs, n=n, out=ref, bn=64, check=True)
    assert _call(lib, A, B, segs, n, 64, 0, None, None, out, stream) == 0
    assert lib.raiccl_grouped_gemm_noalloc_status(None, ctypes.c_void_p(stream.cuda_stream)) == 0
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
