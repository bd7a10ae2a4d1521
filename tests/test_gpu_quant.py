"""Quantized weights on the GPU (Q4_0, Q5_0, Q8_0: the types whose activations are Q8_0 blocks) against the C
oracle, which test_oracle.py pins bit-exactly to nibble's own quantizer, block dots and dequantization
(src/quant.cpp). The reference quantizes each activation row, adds per-block float terms in block order, and
dequantizes embedding rows with one float product per element; the GPU does the same operations, so every result
here is required to be bit-identical."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

TYPES = {"q4_0": (oracle.Q4_0, 3), "q5_0": (oracle.Q5_0, 4), "q8_0": (oracle.Q8_0, 5)}  # oracle id, ABI code


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("name", sorted(TYPES))
@pytest.mark.parametrize("n", [1, 3, 8, 9, 20])
def test_quant_matmul_bit_exact(nbl_ctx, name, n):
    """n <= 8 is the GEMV (one launch); 9 and 20 rows the tensor-core GEMM. Widths of 96 (3 blocks), 2048 (two full
    rounds of 32 blocks) and 5632 (176 blocks: a partial last round)."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(n * 10 + cdt)
    for ne1, ne0 in [(37, 96), (300, 2048), (64, 5632)]:
        w = oracle.random_q_blocks(rng, odt, ne1, ne0)
        x = (rng.standard_normal((n, ne0)) * 2).astype(np.float32)
        wt = nbl_ctx.weight(w, cdt, ne0)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        ref = oracle.matmul_q(w, odt, ne0, ne1, x, n)
        assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), (ne1, ne0)
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_quant_matmul_multi_and_zero_blocks(nbl_ctx, name):
    """matmul_multi over three weights of one type (one launch) equals the oracle; an all-zero activation block
    (scale 0) and a tiny-magnitude block quantize like the reference."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(cdt)
    ne0 = 256
    x = rng.standard_normal((2, ne0)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 32:64] *= 1e-30
    ws = [oracle.random_q_blocks(rng, odt, r, ne0) for r in (128, 16, 16)]
    wts = [nbl_ctx.weight(w, cdt, ne0) for w in ws]
    ys = [torch.full((2, w.shape[0]), float("nan"), device="cuda") for w in ws]
    nbl_ctx.matmul_multi(wts, dev(x), ys, 2)
    for w, y in zip(ws, ys):
        ref = oracle.matmul_q(w, odt, ne0, w.shape[0], x, 2)
        assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32))
    for wt in wts:
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_quant_gemv_wide_rows(nbl_ctx, name):
    """Wide rows: 256 and 640 blocks per row (several rounds of 32 block terms per lane), with 3 and 8 activation
    rows."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(33 + cdt)
    for ne1, ne0, n in [(40, 8192, 3), (24, 20480, 8)]:
        w = oracle.random_q_blocks(rng, odt, ne1, ne0)
        x = (rng.standard_normal((n, ne0)) * 2).astype(np.float32)
        wt = nbl_ctx.weight(w, cdt, ne0)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        ref = oracle.matmul_q(w, odt, ne0, ne1, x, n)
        assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), (ne1, ne0, n)
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
@pytest.mark.parametrize("n", [9, 127, 128, 257])
def test_quant_gemm_bit_exact(nbl_ctx, name, n):
    """More than 8 activation rows run on the tensor cores (one kind::i8 MMA per block, terms added in block
    order by the epilogue). Shapes cover a width below one 128-byte stage (32), a block count that is not a
    multiple of the 4 blocks per stage (160 = 5 blocks), weight-row counts that are not a multiple of the 128-row
    tile, and token counts on both sides of the 128-row token tile."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(n * 7 + cdt)
    for ne1, ne0 in [(129, 32), (200, 160), (300, 1024)]:
        w = oracle.random_q_blocks(rng, odt, ne1, ne0)
        x = (rng.standard_normal((n, ne0)) * 3).astype(np.float32)
        x[n // 2, :32] = 0.0  # a zero block: scale 0, terms +0
        wt = nbl_ctx.weight(w, cdt, ne0)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        ref = oracle.matmul_q(w, odt, ne0, ne1, x, n)
        got = host(y)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (
            ne1, ne0, int((got.view(np.uint32) != ref.view(np.uint32)).sum()))
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_quant_gemm_large_grid(nbl_ctx, name):
    """Enough tiles (75 weight-row tiles x 4 activation-row tiles of 128) for the one-CTA-per-SM layout with
    128-row activation tiles; the smaller cases above run the two-CTAs-per-SM layout with 64-row tiles."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(70 + cdt)
    ne1, ne0, n = 9600, 96, 400
    w = oracle.random_q_blocks(rng, odt, ne1, ne0)
    x = (rng.standard_normal((n, ne0)) * 3).astype(np.float32)
    wt = nbl_ctx.weight(w, cdt, ne0)
    y = torch.full((n, ne1), float("nan"), device="cuda")
    nbl_ctx.matmul(wt, dev(x), y, n)
    ref = oracle.matmul_q(w, odt, ne0, ne1, x, n)
    got = host(y)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), int((got.view(np.uint32) != ref.view(np.uint32)).sum())
    wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_quant_gemm_multi(nbl_ctx, name):
    """matmul_multi on the tensor-core path: five weights of one type (a group of four in one launch, then one),
    with row counts that end mid-tile, and the same weights again so the cached operands are reused."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(90 + cdt)
    ne0, n = 512, 45
    ws = [oracle.random_q_blocks(rng, odt, r, ne0) for r in (256, 100, 100, 640, 33)]
    wts = [nbl_ctx.weight(w, cdt, ne0) for w in ws]
    for rep in range(2):
        x = (rng.standard_normal((n, ne0)) * (rep + 1)).astype(np.float32)
        ys = [torch.full((n, w.shape[0]), float("nan"), device="cuda") for w in ws]
        nbl_ctx.matmul_multi(wts, dev(x), ys, n)
        for w, y in zip(ws, ys):
            ref = oracle.matmul_q(w, odt, ne0, w.shape[0], x, n)
            assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), (rep, w.shape)
    for wt in wts:
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_quant_embed_bit_exact(nbl_ctx, name):
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(40 + cdt)
    table = oracle.random_q_blocks(rng, odt, 500, 192, scale=0.5)
    ids = np.array([0, 499, 7, 7, 250], np.int32)
    t = nbl_ctx.weight(table, cdt, 192)
    out = torch.full((ids.size, 192), float("nan"), device="cuda")
    nbl_ctx.embed(t, ids, out)
    ref = oracle.dequantize_rows(table, odt, 192, 500)[ids]
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))
    t.close()
