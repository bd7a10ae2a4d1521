"""The model's non-attention Backend ops on the GPU (embed, matmul, rmsnorm, add, copy, silu_mul;
src/backend/backend.h:54-70) against the C oracle, which test_oracle.py pins bit-exactly to nibble's own scalar
kernels (src/backend/cpu/ref_ops.cpp).

Tolerances: embed, add and copy are bit-identical. matmul may differ only by fp32 summation order: every output
is within the recursive-summation bound 2 * ne0 * 2^-24 * sum_k |x_k w_k| of the reference's left-to-right sum.
rmsnorm runs the reference's double arithmetic and differs at most in the order of the double sum (<= 1 ulp of
the float result). silu_mul differs by CUDA's expf against the C library's (a few ulp).
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _weights(rng, ne1, ne0, dt):
    w = (rng.standard_normal((ne1, ne0)) * 0.2).astype(np.float32)
    return oracle.f32_to_fp16_bits(w).view(np.float16) if dt == "f16" else w


def _summation_bound(w, x):
    wf = w.astype(np.float32) if w.dtype == np.float16 else w
    return 2.0 * w.shape[1] * 2.0 ** -24 * (np.abs(x).astype(np.float64) @ np.abs(wf).T.astype(np.float64))


@pytest.mark.parametrize("dt", ["f32", "f16"])
@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 9, 33, 128, 130])
def test_matmul_matches_oracle(nbl_ctx, dt, n):
    """n <= 8 runs the weight-streaming GEMV (one instantiation per n), n > 8 the tensor-core GEMM (kind::f16 /
    kind::tf32 on operands split into terms); all within the bound of the reference's fp32 sum."""
    import torch
    rng = np.random.default_rng(n * 7 + (dt == "f16"))
    for ne1, ne0 in [(37, 72), (1000, 256), (96, 2048)]:
        w = _weights(rng, ne1, ne0, dt)
        x = rng.standard_normal((n, ne0)).astype(np.float32)
        wt = nbl_ctx.weight(w)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        got = host(y)
        ref = oracle.matmul(w.view(np.uint16) if dt == "f16" else w, x, n)
        assert np.all(np.abs(got - ref) <= _summation_bound(w, x) + 1e-30), (ne1, ne0)
        wt.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_matmul_gemm_large_grid(nbl_ctx, dt):
    """Enough tiles (32 weight-row tiles x 5 activation-row tiles of 128) for the 128-row activation tiles of the
    tensor-core GEMM (the cases above use 64-row tiles), with a K tail (ne0 = 4 mod 32) and a 4-row weight tail."""
    import torch
    rng = np.random.default_rng(55 + (dt == "f16"))
    ne1, ne0, n = 4100, 260, 640
    w = _weights(rng, ne1, ne0, dt)
    x = rng.standard_normal((n, ne0)).astype(np.float32)
    wt = nbl_ctx.weight(w)
    y = torch.full((n, ne1), float("nan"), device="cuda")
    nbl_ctx.matmul(wt, dev(x), y, n)
    got = host(y)
    ref = oracle.matmul(w.view(np.uint16) if dt == "f16" else w, x, n)
    assert np.all(np.abs(got - ref) <= _summation_bound(w, x) + 1e-30)
    wt.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_matmul_unaligned_rows_and_pointers(nbl_ctx, dt):
    """Widths that are not whole 16-byte chunks, and an activation pointer off the 16-byte grid, take the scalar
    GEMV (and, for 12 rows of width 9, the CUDA-core GEMM); results are the same function."""
    import torch
    rng = np.random.default_rng(3)
    for ne1, ne0, n, off in [(45, 66, 3, 0), (33, 70, 1, 0), (40, 64, 2, 1), (17, 9, 12, 1)]:
        w = _weights(rng, ne1, ne0, dt)
        x = rng.standard_normal((n, ne0)).astype(np.float32)
        xd = torch.zeros(n * ne0 + off, device="cuda")
        xd[off:] = dev(x.ravel())
        y = torch.zeros((n, ne1), device="cuda")
        wt = nbl_ctx.weight(w)
        nbl_ctx.matmul(wt, xd.data_ptr() + 4 * off, y, n)
        ref = oracle.matmul(w.view(np.uint16) if dt == "f16" else w, x, n)
        assert np.all(np.abs(host(y) - ref) <= _summation_bound(w, x) + 1e-30)
        wt.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_matmul_fallback_gemm_for_untileable_widths(nbl_ctx, dt):
    """Row widths the tensor-core GEMM's TMA cannot tile (not a multiple of 8 for F16, 4 for F32) with n > 8 rows run
    the library's fp32 CUDA-core GEMM: partial 64 x 64 tiles on both sides and a K tail, within the bound of the
    reference's fp32 sum."""
    import torch
    rng = np.random.default_rng(77 + (dt == "f16"))
    for ne1, ne0, n in [(130, 37, 70), (65, 1001, 9), (200, 9, 129), (1, 3, 300)]:
        w = _weights(rng, ne1, ne0, dt)
        x = rng.standard_normal((n, ne0)).astype(np.float32)
        wt = nbl_ctx.weight(w)
        y = torch.full((n, ne1), float("nan"), device="cuda")
        nbl_ctx.matmul(wt, dev(x), y, n)
        ref = oracle.matmul(w.view(np.uint16) if dt == "f16" else w, x, n)
        assert np.all(np.abs(host(y) - ref) <= _summation_bound(w, x) + 1e-30), (ne1, ne0, n)
        wt.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_embed_bit_exact(nbl_ctx, dt):
    import torch
    rng = np.random.default_rng(11)
    table = _weights(rng, 500, 192, dt)
    ids = np.array([0, 499, 7, 7, 250, 1], np.int32)
    t = nbl_ctx.weight(table)
    out = torch.full((ids.size, 192), float("nan"), device="cuda")
    nbl_ctx.embed(t, ids, out)
    ref = oracle.embed(table.view(np.uint16) if dt == "f16" else table, ids)
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))
    t.close()


def test_embed_rejects_out_of_range_id_with_reference_message(nbl_ctx):
    import torch
    import nibble_b200 as nb
    t = nbl_ctx.weight(np.zeros((7, 4), np.float32))
    out = torch.zeros((2, 4), device="cuda")
    for bad in (7, -1):
        with pytest.raises(nb.NibbleError, match=rf"embed: token id {bad} out of range \(n_vocab 7\)"):
            nbl_ctx.embed(t, np.array([0, bad], np.int32), out)
    t.close()


@pytest.mark.parametrize("d", [4, 64, 896, 2048, 4097])
def test_rmsnorm_matches_oracle(nbl_ctx, d):
    import torch
    rng = np.random.default_rng(d)
    n = 5
    x = (rng.standard_normal((n, d)) * 3).astype(np.float32)
    w = rng.standard_normal(d).astype(np.float32)
    wt = nbl_ctx.weight(w)
    for eps in (1e-6, 1e-5):
        y = torch.full((n, d), float("nan"), device="cuda")
        nbl_ctx.rmsnorm(dev(x), wt, y, n, eps)
        got, ref = host(y), oracle.rmsnorm(x, w, n, eps)
        assert np.all(np.abs(got - ref) <= np.spacing(np.abs(ref)))  # at most one float ulp
    wt.close()


def test_rmsnorm_known_answer(nbl_ctx):
    """tests/test_ref_ops.cpp:33-37: x = {1,2,3,4}, unit weight, eps 0 -> x / sqrt(7.5)."""
    import torch
    wt = nbl_ctx.weight(np.ones(4, np.float32))
    y = torch.zeros((1, 4), device="cuda")
    nbl_ctx.rmsnorm(dev(np.array([[1, 2, 3, 4]], np.float32)), wt, y, 1, 0.0)
    assert np.allclose(host(y)[0], np.array([1, 2, 3, 4]) / np.sqrt(7.5), rtol=1e-6, atol=1e-7)
    wt.close()


@pytest.mark.parametrize("count,off", [(1, 0), (7, 0), (4096, 0), (100003, 0), (1001, 1)])
def test_add_copy_silu_mul(nbl_ctx, count, off):
    """off = 1 puts both operands one float past a 16-byte boundary (the scalar path)."""
    import torch
    rng = np.random.default_rng(count + off)
    a = (rng.standard_normal(count) * 6).astype(np.float32)
    b = rng.standard_normal(count).astype(np.float32)
    da = torch.zeros(count + off, device="cuda")
    db = torch.zeros(count + off, device="cuda")
    da[off:] = dev(a)
    db[off:] = dev(b)
    pa, pb = da.data_ptr() + 4 * off, db.data_ptr() + 4 * off
    nbl_ctx.add(pa, pb, count)
    assert np.array_equal(host(da)[off:].view(np.uint32), oracle.add(a, b).view(np.uint32))
    da[off:] = dev(a)
    nbl_ctx.silu_mul(pa, pb, count)
    ref = oracle.silu_mul(a, b)
    got = host(da)[off:]
    assert np.all(np.abs(got - ref) <= 4 * np.spacing(np.abs(ref)) + 1e-37)
    dc = torch.zeros(count, device="cuda")
    nbl_ctx.copy(dc, pb, count)
    assert np.array_equal(host(dc), b)


def test_silu_mul_known_answer(nbl_ctx):
    """tests/test_ref_ops.cpp:98-103."""
    g = dev(np.array([0, 1], np.float32))
    nbl_ctx.silu_mul(g, dev(np.array([2, 3], np.float32)), 2)
    assert np.allclose(host(g), [0.0, 3.0 / (1.0 + np.exp(-1.0))], rtol=1e-6, atol=1e-7)


def test_weight_data_reports_the_upload(nbl_ctx):
    import ctypes as C
    import torch
    from nibble_b200 import _abi
    w = np.arange(12, dtype=np.float32).reshape(3, 4)
    wt = nbl_ctx.weight(w)
    p, dt, ne0, ne1 = C.c_void_p(), C.c_int32(), C.c_int64(), C.c_int64()
    assert _abi.lib.nbl_weight_data(wt.handle, C.byref(p), C.byref(dt), C.byref(ne0), C.byref(ne1)) == 0
    assert (dt.value, ne0.value, ne1.value) == (0, 4, 3)
    back = torch.empty(12, device="cuda")
    back.copy_(torch.as_tensor(np.zeros(12, np.float32)))
    nbl_ctx.copy(back, p.value, 12)
    assert np.array_equal(host(back), w.ravel())
    wt.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_matmul_multi_equals_separate_calls_large(nbl_ctx, dt):
    """Two weights large enough that their joint launch takes 128-row activation tiles while each alone takes 64
    (and the first alone splits K): still bit for bit equal to the separate calls."""
    import torch
    rng = np.random.default_rng(7 + (dt == "f16"))
    ne0, n, rows = 512, 256, [8192, 8192, 100]
    ws = [nbl_ctx.weight(_weights(rng, r, ne0, dt)) for r in rows]
    x = dev(rng.standard_normal((n, ne0)).astype(np.float32))
    ys = [torch.full((n, r), float("nan"), device="cuda") for r in rows]
    nbl_ctx.matmul_multi(ws, x, ys, n)
    for w, y, r in zip(ws, ys, rows):
        single = torch.full((n, r), float("nan"), device="cuda")
        nbl_ctx.matmul(w, x, single, n)
        assert np.array_equal(host(y).view(np.uint32), host(single).view(np.uint32)), r
    for w in ws:
        w.close()


@pytest.mark.parametrize("dt", ["f32", "f16"])
@pytest.mark.parametrize("n", [1, 4, 8, 20])
def test_matmul_multi_equals_separate_calls(nbl_ctx, dt, n):
    """Backend::matmul_multi's contract (backend.h:57-58): results equal separate matmul calls -- here bit for bit,
    for a Q/K/V-like triple (one GEMV launch for n <= 8) and five weights (more than one launch holds)."""
    import torch
    rng = np.random.default_rng(n + 100 * (dt == "f16"))
    ne0 = 256
    for rows in ([256, 64, 64], [96, 32, 512, 8, 40]):
        ws = [nbl_ctx.weight(_weights(rng, r, ne0, dt)) for r in rows]
        x = dev(rng.standard_normal((n, ne0)).astype(np.float32))
        ys = [torch.full((n, r), float("nan"), device="cuda") for r in rows]
        nbl_ctx.matmul_multi(ws, x, ys, n)
        for w, y, r in zip(ws, ys, rows):
            single = torch.full((n, r), float("nan"), device="cuda")
            nbl_ctx.matmul(w, x, single, n)
            assert np.array_equal(host(y).view(np.uint32), host(single).view(np.uint32))
        for w in ws:
            w.close()
