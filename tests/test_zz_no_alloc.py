"""The allocation-free grouped-GEMM C entry point, called through its exported
symbol with ctypes.

``raiccl_grouped_gemm_noalloc`` serves callers that cannot allocate device
memory: a C or C++ program with neither torch nor an allocator of its own, or
code that must not grow its memory footprint.  Its working memory is one
file-scope device array, so these tests check that (1) two calls in a row
give the same output as the ordinary entry point (``ops.grouped_gemm``, which
takes caller-allocated tables) across input / output dtypes and the row-map
scatter, (2) the tf32 path matches a plain fp32 PyTorch reference, and (3)
bad arguments are rejected before launch or, for segment contents, through
the device status with nothing written.

Collected last on purpose (file name): it must pass after every other GPU
test has run in the same process, and alone in a fresh process."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

BAD_ARGUMENT = -2
STATUS_BOUNDS = 4
STATUS_CONFIG = 5


def _lib():
    from revealaiccl_b200.ops._native import kernels

    lib = ctypes.CDLL(kernels().__file__)
    f = lib.raiccl_grouped_gemm_noalloc
    f.restype = ctypes.c_int
    ll, i, p = ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p
    # the prototype of csrc/include/gg_noalloc.h
    f.argtypes = [i, p, ll, ll, ll, p, ll, ll, p, i, i, i, i, p, p, p, p, ll, ll, i, i, ctypes.c_ulonglong, p]
    lib.raiccl_grouped_gemm_noalloc_status.restype = ctypes.c_int
    lib.raiccl_grouped_gemm_noalloc_status.argtypes = [p, p]
    lib.raiccl_grouped_gemm_noalloc_max_segments.restype = ctypes.c_int
    lib.raiccl_grouped_gemm_noalloc_error_string.restype = ctypes.c_char_p
    lib.raiccl_grouped_gemm_noalloc_error_string.argtypes = [ctypes.c_int]
    return lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call(lib, A, B, segs, n, bn, act, bias, row_map, row_scale, out, stream, *, out_rows=None, ldo=None):
    return lib.raiccl_grouped_gemm_noalloc(
        0 if A.dtype == torch.bfloat16 else 1, _ptr(A), A.shape[0], A.shape[1], A.stride(0),
        _ptr(B), B.shape[0], B.stride(0), _ptr(segs), segs.shape[0], n, bn, act,
        _ptr(bias), _ptr(row_map), _ptr(row_scale), _ptr(out),
        out.shape[0] if out_rows is None else out_rows, out.stride(0) if ldo is None else ldo,
        int(out.dtype == torch.bfloat16), 0, 0, ctypes.c_void_p(stream.cuda_stream))


def _status(lib, stream):
    return lib.raiccl_grouped_gemm_noalloc_status(None, ctypes.c_void_p(stream.cuda_stream))


def _case(seed, dev, dtype=torch.bfloat16, mapped=False):
    g = torch.Generator(device="cpu").manual_seed(seed)
    E, n, k = 3, 128, 512
    rows = [130, 0, 257]
    m = sum(rows)
    A = torch.randn(m, k, generator=g).to(dtype).to(dev)
    B = (torch.randn(E * n, k, generator=g) / k ** 0.5).to(dtype).to(dev)
    bias = (torch.randn(E * n, generator=g) * 0.1).to(dev)
    scale = torch.rand(m, generator=g).to(dev)
    row_map = torch.randperm(m, generator=g).to(torch.int32).to(dev) if mapped else None
    segs_list, a0 = [], 0
    for e, r in enumerate(rows):
        segs_list.append((a0, r, (e + seed) % E, 0, a0))
        a0 += r
    return A, B, bias, scale, row_map, segs_list, n


CASES = [  # (fp32 inputs, bf16 output, row map)
    (False, False, False), (False, True, False), (False, False, True), (False, True, True),
    (True, False, False), (True, False, True),
]


@pytest.mark.parametrize("in_fp32,out_bf16,mapped", CASES)
def test_noalloc_matches_entry_point_twice(in_fp32, out_bf16, mapped):
    from revealaiccl_b200.ops import grouped_gemm as gg

    lib = _lib()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream(dev)
    out_dtype = torch.bfloat16 if out_bf16 else torch.float32
    tol = 2e-2 if out_bf16 else 2e-3
    for seed in (0, 1):  # two calls in a row reuse the same device scratch
        A, B, bias, scale, row_map, segs_list, n = _case(seed, dev, torch.float32 if in_fp32 else torch.bfloat16,
                                                        mapped)
        segs = gg.make_segments(segs_list, dev)
        ref = torch.zeros(A.shape[0], n, device=dev, dtype=out_dtype)
        gg.grouped_gemm(A, B, segs, n=n, act="gelu", bias=bias, row_map=row_map, row_scale=scale, out=ref, bn=64,
                        check=True)
        out = torch.full((A.shape[0], n), float("nan"), device=dev, dtype=out_dtype)
        rc = _call(lib, A, B, segs, n, 64, gg.ACT_IDS["gelu"], bias, row_map, scale, out, stream)
        assert rc == 0, lib.raiccl_grouped_gemm_noalloc_error_string(rc)
        st = (ctypes.c_int * 8)()
        assert lib.raiccl_grouped_gemm_noalloc_status(ctypes.cast(st, ctypes.c_void_p),
                                                      ctypes.c_void_p(stream.cuda_stream)) == 0
        torch.testing.assert_close(out, ref, atol=tol, rtol=tol)


def test_noalloc_tf32_matches_fp32_reference():
    """The tf32 path against a plain fp32 PyTorch computation of the same op."""
    from revealaiccl_b200.ops import grouped_gemm as gg

    lib = _lib()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream(dev)
    A, B, bias, scale, row_map, segs_list, n = _case(3, dev, torch.float32, mapped=True)
    segs = gg.make_segments(segs_list, dev)
    out = torch.full((A.shape[0], n), float("nan"), device=dev)
    assert _call(lib, A, B, segs, n, 128, gg.ACT_IDS["relu"], bias, row_map, scale, out, stream) == 0
    assert _status(lib, stream) == 0
    ref = torch.full_like(out, float("nan"))
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        Ac, Bc = A.double().cpu(), B.double().cpu()
        for a0, r, e, _, _ in segs_list:
            if r == 0:
                continue
            y = Ac[a0:a0 + r] @ Bc[e * n:(e + 1) * n].T + bias[e * n:(e + 1) * n].double().cpu()
            y = torch.relu(y) * scale[a0:a0 + r].double().cpu()[:, None]
            ref[row_map[a0:a0 + r].long()] = y.float().to(dev)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.testing.assert_close(out, ref, atol=5e-3, rtol=5e-3)


def test_noalloc_rejects_oversize_and_bad_segments():
    from revealaiccl_b200.ops import grouped_gemm as gg

    lib = _lib()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream(dev)
    cap = lib.raiccl_grouped_gemm_noalloc_max_segments()
    A, B, bias, scale, _, segs_list, n = _case(2, dev)
    m = A.shape[0]
    out = torch.zeros(m, n, device=dev)
    big = gg.make_segments([(0, 0, 0, 0, 0)] * (cap + 1), dev)
    rc = _call(lib, A, B, big, n, 64, 0, None, None, None, out, stream)
    assert rc == -1 and b"1024" in lib.raiccl_grouped_gemm_noalloc_error_string(rc)

    # segment contents are checked on the device: status set, nothing written
    bad = {
        "out_slot": ([(0, 4, 0, 1, 0)], None, STATUS_CONFIG),        # only slot 0 exists here
        "expert": ([(0, 4, 3, 0, 0)], None, STATUS_BOUNDS),          # rows_b / N = 3 experts
        "a_rows": ([(m - 2, 4, 0, 0, 0)], None, STATUS_BOUNDS),      # past rows_a
        "out_rows": ([(0, 4, 0, 0, m - 2)], None, STATUS_BOUNDS),    # past out_rows
    }
    for name, (seg, row_map, code) in bad.items():
        s = gg.make_segments(seg, dev)
        assert _call(lib, A, B, s, n, 64, 0, None, row_map, None, out, stream) == 0, name
        assert _status(lib, stream) == code, name
        assert torch.count_nonzero(out) == 0, name
    wild = torch.arange(m, dtype=torch.int32, device=dev)
    wild[1] = m  # one mapped output row past out_rows
    s = gg.make_segments([(0, 4, 0, 0, 0)], dev)
    assert _call(lib, A, B, s, n, 64, 0, None, wild, None, out, stream) == 0
    assert _status(lib, stream) == STATUS_BOUNDS
    assert torch.count_nonzero(out) == 0

    # host-side argument checks: rejected before anything is enqueued
    segs = gg.make_segments(segs_list, dev)
    flat = torch.zeros(m * n + 4, device=dev)
    shifted = flat[1:1 + m * n].view(m, n)  # 4 bytes past a 16-byte boundary
    assert _call(lib, A, B, segs, n, 64, 0, None, None, None, shifted, stream) == BAD_ARGUMENT
    assert _call(lib, A, B, segs, n, 64, 0, None, None, None, out, stream, ldo=n - 16) == BAD_ARGUMENT
    assert _call(lib, A, B, segs, n, 64, 0, None, None, None, out, stream, ldo=n + 1) == BAD_ARGUMENT
    bias_flat = torch.zeros(bias.numel() + 1, device=dev)
    assert _call(lib, A, B, segs, n, 64, 0, bias_flat[1:], None, None, out, stream) == BAD_ARGUMENT
    assert _call(lib, A, B, segs, n, 16, gg.ACT_IDS["swiglu"], None, None, None, out, stream) == BAD_ARGUMENT

    # the next good call starts from a clean status
    ref = torch.zeros(m, n, device=dev)
    gg.grouped_gemm(A, B, segs, n=n, out=ref, bn=64, check=True)
    assert _call(lib, A, B, segs, n, 64, 0, None, None, None, out, stream) == 0
    assert _status(lib, stream) == 0
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)
