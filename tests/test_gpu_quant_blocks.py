"""Quantized weights on the GPU whose activations are Q8_1 blocks (Q5_1) or Q8_K super-blocks (Q4_K, Q5_K, Q6_K),
against the C oracle, which test_oracle.py pins bit-exactly to nibble's own quantizers, block dots and
dequantization (src/quant.cpp) and to CpuBackend's SIMD kernels. The reference quantizes each activation row,
keeps eight float accumulators per k-quant row (one per element index mod 8) plus the min-term total, and adds them
in a fixed order; the GPU does the same operations in the same order, so every result here is required to be
bit-identical."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

TYPES = {"q5_1": (oracle.Q5_1, 6), "q4_k": (oracle.Q4_K, 7), "q5_k": (oracle.Q5_K, 8), "q6_k": (oracle.Q6_K, 9)}


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _acts(rng, n, ne0):
    """Activation rows with an all-zero 256-element span, a tiny-magnitude one and a tied largest magnitude of
    both signs (the Q8_K scale comes from the first)."""
    x = (rng.standard_normal((n, ne0)) * 2).astype(np.float32)
    x[0, :256] = 0.0
    if n > 1:
        x[1, :256] *= 1e-30
    if n > 2 and ne0 >= 512:
        x[2, 256:512] = np.clip(x[2, 256:512], -2.0, 2.0)
        x[2, 256 + 3], x[2, 256 + 40] = 6.0, -6.0
    return x


def _widths(odt):
    return [(37, 96), (300, 2048), (64, 5632)] if odt == oracle.Q5_1 else [(37, 256), (300, 2048), (64, 5632)]


@pytest.mark.parametrize("name", sorted(TYPES))
@pytest.mark.parametrize("n", [1, 3, 5, 8, 9, 64])
def test_block_quant_matmul_bit_exact(nbl_ctx, name, n):
    """Row counts that fill, and end inside, the 4 activation rows one warp takes; widths of 1, 8 and 22
    super-blocks (Q5_1: 3, 64 and 176 blocks, the last a partial round of 32 per lane)."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(n * 13 + cdt)
    for ne1, ne0 in _widths(odt):
        w = oracle.random_q_blocks(rng, odt, ne1, ne0)
        x = _acts(rng, n, ne0)
        wt = nbl_ctx.weight(w, cdt, ne0)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        ref = oracle.matmul_q(w, odt, ne0, ne1, x, n)
        got = host(y)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (
            ne1, ne0, int((got.view(np.uint32) != ref.view(np.uint32)).sum()))
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_block_quant_matmul_many_rows(nbl_ctx, name):
    """A prefill-sized call (300 activation rows) and decode-sized ones whose weight row counts give the decode
    kernel 8 (20,000 rows), 4 (4,000) and 2 (2,048) weight rows per CTA."""
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(200 + cdt)
    for ne1, ne0, n in [(96, 512, 300), (20000, 256, 2), (4000, 512, 8), (2048, 256, 1)]:
        w = oracle.random_q_blocks(rng, odt, ne1, ne0)
        x = _acts(rng, n, ne0)
        wt = nbl_ctx.weight(w, cdt, ne0)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        ref = oracle.matmul_q(w, odt, ne0, ne1, x, n)
        assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), (ne1, ne0, n)
        wt.close()


def test_block_quant_matmul_multi_mixed_types(nbl_ctx):
    """matmul_multi over weights of different block types sharing x (a Q4_K_M-style attention block: Q4_K Q and K,
    Q6_K V, a Q5_K and a Q5_1 projection): each output equals the oracle's for its own weight."""
    import torch
    rng = np.random.default_rng(321)
    ne0, n = 1024, 6
    plan = [(oracle.Q4_K, 7, 256), (oracle.Q4_K, 7, 64), (oracle.Q6_K, 9, 64), (oracle.Q5_K, 8, 100),
            (oracle.Q5_1, 6, 40)]
    ws = [oracle.random_q_blocks(rng, odt, rows, ne0) for odt, _, rows in plan]
    wts = [nbl_ctx.weight(w, cdt, ne0) for w, (_, cdt, _) in zip(ws, plan)]
    x = _acts(rng, n, ne0)
    ys = [torch.full((n, rows), float("nan"), device="cuda") for _, _, rows in plan]
    nbl_ctx.matmul_multi(wts, dev(x), ys, n)
    for w, y, (odt, _, rows) in zip(ws, ys, plan):
        ref = oracle.matmul_q(w, odt, ne0, rows, x, n)
        assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), odt
    for wt in wts:
        wt.close()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_block_quant_embed_bit_exact(nbl_ctx, name):
    import torch
    odt, cdt = TYPES[name]
    rng = np.random.default_rng(50 + cdt)
    ne0 = 512
    table = oracle.random_q_blocks(rng, odt, 300, ne0, scale=0.5)
    ids = np.array([0, 299, 7, 7, 150], np.int32)
    t = nbl_ctx.weight(table, cdt, ne0)
    out = torch.full((ids.size, ne0), float("nan"), device="cuda")
    nbl_ctx.embed(t, ids, out)
    ref = oracle.dequantize_rows(table, odt, ne0, 300)[ids]
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))
    t.close()


def test_block_quant_rejects_partial_blocks(nbl_ctx):
    import nibble_b200 as nb
    with pytest.raises(nb.NibbleError, match="256-element blocks"):
        nbl_ctx.weight(np.zeros((2, 144), np.uint8), 7, 128)
