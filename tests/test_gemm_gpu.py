"""Numerics of the tcgen05 grouped GEMM against a plain PyTorch fp32 reference."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _gg():
    from revealaiccl_b200.ops import grouped_gemm as gg
    return gg


def _ref(A, B, segs_list, n, act, bias=None, row_scale=None, out_rows=None):
    out = torch.zeros((out_rows, n if act != "swiglu" else n // 2), dtype=torch.float32, device=A.device)
    for (a0, rows, e, _slot, o0) in segs_list:
        x = A[a0:a0 + rows].float()
        w = B[e * n:(e + 1) * n].float()
        y = x @ w.t()
        if bias is not None:
            y = y + bias.view(-1, n)[e]
        if act == "relu":
            y = torch.relu(y)
        elif act == "gelu":
            y = torch.nn.functional.gelu(y)
        elif act == "silu":
            y = torch.nn.functional.silu(y)
        if row_scale is not None:
            y = y * row_scale[a0:a0 + rows, None]
        out[o0:o0 + rows] = y
    return out


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (256, 256, 512), (300, 64, 1024)])
def test_bf16_dense_single_segment(m, n, k):
    gg = _gg()
    torch.manual_seed(0)
    dev = torch.device("cuda")
    A = torch.randn(m, k, device=dev).bfloat16()
    B = torch.randn(n, k, device=dev).bfloat16() / k ** 0.5
    segs_list = [(0, m, 0, 0, 0)]
    segs = gg.make_segments(segs_list, dev)
    out = torch.zeros(m, n, device=dev)
    gg.grouped_gemm(A, B, segs, n=n, out=out, check=True)
    ref = _ref(A, B, segs_list, n, "none", out_rows=m)
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-3)


def test_tf32_relu_partial_tiles():
    gg = _gg()
    torch.manual_seed(1)
    dev = torch.device("cuda")
    m, n, k = 300, 32, 2048
    A = torch.randn(m, k, device=dev)
    B = torch.randn(n, k, device=dev) / k ** 0.5
    bias = torch.randn(n, device=dev) * 0.01
    segs_list = [(0, m, 0, 0, 0)]
    out = torch.zeros(m, n, device=dev)
    gg.grouped_gemm(A, B, gg.make_segments(segs_list, dev), n=n, act="relu", bias=bias, out=out, check=True)
    ref = _ref(A, B, segs_list, n, "relu", bias=bias, out_rows=m)
    torch.testing.assert_close(out, ref, atol=5e-3, rtol=5e-3)


def test_tf32_n16_k32():
    gg = _gg()
    torch.manual_seed(2)
    dev = torch.device("cuda")
    m, n, k = 200, 16, 32
    A = torch.randn(m, k, device=dev)
    B = torch.randn(2 * n, k, device=dev) / k ** 0.5
    segs_list = [(0, 120, 1, 0, 0), (120, 80, 0, 0, 120)]
    out = torch.zeros(m, n, device=dev)
    gg.grouped_gemm(A, B, gg.make_segments(segs_list, dev), n=n, out=out, check=True)
    ref = _ref(A, B, segs_list, n, "none", out_rows=m)
    torch.testing.assert_close(out, ref, atol=3e-3, rtol=3e-3)


def test_bf16_multi_segment_rowmap_scale_gelu_bf16_out():
    gg = _gg()
    torch.manual_seed(3)
    dev = torch.device("cuda")
    k, n, E = 256, 128, 3
    seg_rows = [(0, 130, 2), (200, 0, 1), (200, 57, 0), (400, 256, 1)]
    total = 700
    A = torch.randn(total, k, device=dev).bfloat16()
    B = (torch.randn(E * n, k, device=dev) / k ** 0.5).bfloat16()
    bias = torch.randn(E * n, device=dev) * 0.1
    scale = torch.rand(total, device=dev)
    perm = torch.randperm(total, device=dev).int()
    segs_list = [(a0, r, e, 0, a0) for (a0, r, e) in seg_rows]
    out = torch.zeros(total, n, device=dev, dtype=torch.bfloat16)
    gg.grouped_gemm(A, B, gg.make_segments(segs_list, dev), n=n, act="gelu", bias=bias,
                    row_map=perm, row_scale=scale, out=out, check=True)
    ref_rows = _ref(A, B, segs_list, n, "gelu", bias=bias, row_scale=scale, out_rows=total)
    ref = torch.zeros_like(ref_rows)
    valid = torch.zeros(total, dtype=torch.bool, device=dev)
    for (a0, r, e) in seg_rows:
        valid[a0:a0 + r] = True
    ref[perm.long()[valid]] = ref_rows[valid]
    got = out.float()
    mask = torch.zeros(total, dtype=torch.bool, device=dev)
    mask[perm.long()[valid]] = True
    torch.testing.assert_close(got[mask], ref[mask], atol=2e-2, rtol=2e-2)


def test_bf16_swiglu():
    gg = _gg()
    torch.manual_seed(4)
    dev = torch.device("cuda")
    m, k, f, E = 260, 512, 256, 2
    A = torch.randn(m, k, device=dev).bfloat16()
    wg = (torch.randn(E, f, k, device=dev) / k ** 0.5).bfloat16()
    wu = (torch.randn(E, f, k, device=dev) / k ** 0.5).bfloat16()
    bn = 256
    B = gg.swiglu_interleave(wg, wu, bn).reshape(E * 2 * f, k)
    segs_list = [(0, 100, 1, 0, 0), (100, 160, 0, 0, 100)]
    out = torch.zeros(m, f, device=dev)
    gg.grouped_gemm(A, B, gg.make_segments(segs_list, dev), n=2 * f, act="swiglu", bn=bn, out=out, check=True)
    ref = torch.zeros(m, f, device=dev)
    for (a0, r, e, _, o0) in segs_list:
        x = A[a0:a0 + r].float()
        g = x @ wg[e].float().t()
        u = x @ wu[e].float().t()
        ref[o0:o0 + r] = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(out, ref, atol=5e-3, rtol=5e-3)


@pytest.mark.parametrize("dtype,act,bn", [("tf32", "gelu", 256), ("tf32", "none", 128), ("bf16", "relu", 64),
                                          ("bf16", "swiglu", 256)])
def test_cta_pair_kernel_matches_fp32_reference_and_single_cta(dtype, act, bn):
    """The CTA-pair kernel (256-row tiles on clusters of two SMs) against the fp32
    reference and bit-for-bit against the one-CTA kernel on ragged segments."""
    gg = _gg()
    torch.manual_seed(7)
    dev = torch.device("cuda")
    k, f, E = 512, 256, 3
    n = 2 * f if act == "swiglu" else f
    seg_rows = [(0, 300, 2), (300, 0, 1), (300, 57, 0), (400, 513, 1), (913, 129, 2)]
    total = 1100
    dt = torch.float32 if dtype == "tf32" else torch.bfloat16
    A = torch.randn(total, k, device=dev).to(dt)
    if act == "swiglu":
        wg = (torch.randn(E, f, k, device=dev) / k ** 0.5).to(dt)
        wu = (torch.randn(E, f, k, device=dev) / k ** 0.5).to(dt)
        B = gg.swiglu_interleave(wg, wu, bn).reshape(E * n, k)
    else:
        B = (torch.randn(E * n, k, device=dev) / k ** 0.5).to(dt)
    bias = None if act == "swiglu" else torch.randn(E * n, device=dev) * 0.1
    segs_list = [(a0, r, e, 0, a0) for (a0, r, e) in seg_rows]
    segs = gg.make_segments(segs_list, dev)
    width = f if act == "swiglu" else n
    outs = {}
    for pair in (True, False):
        out = torch.full((total, width), float("nan"), device=dev)
        gg.grouped_gemm(A, B, segs, n=n, act=act, bias=bias, out=out, bn=bn, check=True, pair=pair)
        outs[pair] = out
    valid = torch.zeros(total, dtype=torch.bool, device=dev)
    for (a0, r, e) in seg_rows:
        valid[a0:a0 + r] = True
    if act == "swiglu":
        ref = torch.zeros(total, f, device=dev)
        for (a0, r, e, _, o0) in segs_list:
            x = A[a0:a0 + r].float()
            ref[o0:o0 + r] = torch.nn.functional.silu(x @ wg[e].float().t()) * (x @ wu[e].float().t())
    else:
        ref = _ref(A, B, segs_list, n, act, bias=bias, out_rows=total)
    tol = 5e-3 if dtype == "tf32" else 2e-2
    torch.testing.assert_close(outs[True][valid], ref[valid], atol=tol, rtol=tol)
    assert torch.equal(outs[True][valid], outs[False][valid])
    assert torch.isnan(outs[True][~valid]).all()  # rows outside every segment are never written


@pytest.mark.parametrize("dtype,act,out_dtype", [("tf32", "gelu", torch.float32), ("bf16", "none", torch.bfloat16),
                                                 ("bf16", "silu", torch.float32)])
def test_cta_pair_swapped_tail_tiles(dtype, act, out_dtype):
    """Swapped tail tiles (weights as the 256-row operand, a short tail's tokens
    as N) against the fp32 reference, with a row map and row scales, on tails
    of 1..129 rows, an expert of one row and an empty segment."""
    gg = _gg()
    torch.manual_seed(11)
    dev = torch.device("cuda")
    k, n, E = 384, 512, 4
    seg_rows = [(0, 300, 2), (300, 0, 1), (300, 1, 0), (301, 513, 3), (814, 257, 1), (1071, 16, 2),
                (1087, 17, 0), (1104, 384, 3), (1488, 385, 1)]
    total = 1873
    dt = torch.float32 if dtype == "tf32" else torch.bfloat16
    A = torch.randn(total, k, device=dev).to(dt)
    B = (torch.randn(E * n, k, device=dev) / k ** 0.5).to(dt)
    bias = torch.randn(E * n, device=dev) * 0.1
    perm = torch.randperm(total, device=dev).to(torch.int32)
    scale = torch.rand(total, device=dev) + 0.5
    segs_list = [(a0, r, e, 0, a0) for (a0, r, e) in seg_rows]
    segs = gg.make_segments(segs_list, dev)
    valid = torch.zeros(total, dtype=torch.bool, device=dev)
    for (a0, r, e) in seg_rows:
        valid[a0:a0 + r] = True
    outs = {}
    for swap in (128, 0):
        out = torch.full((total, n), float("nan"), device=dev, dtype=out_dtype)
        gg.grouped_gemm(A, B, segs, n=n, act=act, bias=bias, row_map=perm, row_scale=scale, out=out, bn=256,
                        check=True, pair=True, swap_max=swap)
        outs[swap] = out.float()
    ref_rows = _ref(A, B, segs_list, n, act, bias=bias, row_scale=scale, out_rows=total)
    ref = torch.full((total, n), float("nan"), device=dev)
    ref[perm.long()[valid]] = ref_rows[valid]
    written = torch.zeros(total, dtype=torch.bool, device=dev)
    written[perm.long()[valid]] = True
    tol = 5e-3 if dtype == "tf32" else 3e-2
    torch.testing.assert_close(outs[128][written], ref[written], atol=tol, rtol=tol)
    torch.testing.assert_close(outs[128][written], outs[0][written], atol=tol, rtol=tol)
    assert torch.isnan(outs[128][~written]).all()  # rows outside every segment are never written
