"""Pins the CPU oracle (oracle/nbl_oracle.c) before anything is checked against it.

* The reference's own known-answer cases, restated (tests/test_ref_ops.cpp:41-96, :130-135 in nibble).
* The committed golden fixtures made by nibble's own compiled code (tests/golden/make_golden.py): the scalar
  restatement must be bit-identical to cpu::attention_heads / cpu::rope / softmax_inplace / fp16.h, and within
  the reference's own SIMD tolerance of CpuBackend::attention (tests/test_ops.cpp:195-216: 2e-6 per unit of q
  scale).
* Live comparison with oracle/_ref when it is built (this container; skipped where the reference tree is absent).
"""
import glob
import math
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b, eps=1e-6, margin=1e-7):
    return abs(a - b) <= margin + eps * abs(b)


# ---------------------------------------------------------------- known answers (test_ref_ops.cpp)
def test_rope_known_answers():
    c1, s1, c2, s2 = math.cos(1.0), math.sin(1.0), math.cos(0.01), math.sin(0.01)
    x = np.array([1, 0, 1, 0], np.float32)
    y = oracle.rope(x, 1, 4, 1, 10000.0, False)
    assert rel(y[0], c1) and rel(y[1], s1) and rel(y[2], c2) and rel(y[3], s2)
    y = oracle.rope(x, 1, 4, 1, 10000.0, True)
    assert rel(y[0], c1 - s1) and rel(y[1], 0) and rel(y[2], s1 + c1) and rel(y[3], 0)
    y = oracle.rope(x, 1, 4, 0, 10000.0, False)
    assert np.array_equal(y, x)  # position 0 is the identity
    y = oracle.rope(x, 1, 4, 1, 10000.0, False, np.array([1.0, 2.0], np.float32))
    assert rel(y[2], math.cos(0.005)) and rel(y[3], math.sin(0.005))


def test_attention_known_answer():
    qkv = np.array([1, 0, 0, 1], np.float32)
    out = oracle.attention(qkv, qkv, qkv, 2, 0, 1, 1, 2).ravel()
    assert rel(out[0], 1) and rel(out[1], 0)
    e = math.exp(1.0 / math.sqrt(2.0))
    assert rel(out[2], 1.0 / (1.0 + e)) and rel(out[3], e / (1.0 + e))


def test_attention_gqa_mapping():
    H, KV, D, N = 4, 2, 2, 3
    q = np.ones((1, H, D), np.float32)
    k = np.zeros((N, KV, D), np.float32)
    v = np.zeros((N, KV, D), np.float32)
    for j in range(N):
        for g in range(KV):
            for d in range(D):
                v[j, g, d] = 10 * g + j + d
    out = oracle.attention(q, k, v, 1, N - 1, H, KV, D)
    for h in range(H):
        for d in range(D):
            assert rel(out[0, h, d], 10 * (h // 2) + 1 + d)


def test_softmax_overflow_safe():
    y = oracle.softmax(np.array([1000.0, 1000.0], np.float32))
    assert rel(y[0], 0.5) and rel(y[1], 0.5)


def test_lse_merge_reproduces_full_softmax():
    rng = np.random.default_rng(0)
    H, KV, D, ctx = 4, 2, 16, 97
    q = rng.standard_normal((1, H, D)).astype(np.float32)
    k = rng.standard_normal((ctx, KV, D)).astype(np.float32)
    v = rng.standard_normal((ctx, KV, D)).astype(np.float32)
    full = oracle.attention(q, k, v, 1, ctx - 1, H, KV, D)[0]
    cuts = [0, 10, 40, 41, 97]
    parts_o, parts_lse = [], []
    scale = 1.0 / math.sqrt(D)
    for a, b in zip(cuts[:-1], cuts[1:]):
        kk, vv = k[a:b].astype(np.float64), v[a:b].astype(np.float64)
        s = np.einsum("hd,jhd->hj", np.repeat(q[0].astype(np.float64), 1, 0), np.repeat(kk, H // KV, 1)) * scale
        m = s.max(1, keepdims=True)
        p = np.exp(s - m)
        parts_o.append((np.einsum("hj,jhd->hd", p, np.repeat(vv, H // KV, 1)) / p.sum(1, keepdims=True)))
        parts_lse.append((m[:, 0] + np.log(p.sum(1))))
    parts_o.append(np.zeros((H, D)))  # an empty part (lse = -inf) must not contribute
    parts_lse.append(np.full(H, -np.inf))
    out, lse = oracle.lse_merge(np.array(parts_o, np.float32), np.array(parts_lse, np.float32))
    np.testing.assert_allclose(out, full, atol=2e-6, rtol=0)


# ---------------------------------------------------------------- golden fixtures (nibble's own outputs)
@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "attention_*.npz"))),
                         ids=lambda p: os.path.basename(p)[10:-4])
def test_attention_matches_golden(path):
    f = np.load(path)
    n, pos0, H, KV, D = (int(x) for x in f["meta"])
    out = oracle.attention(f["q"], f["k"], f["v"], n, pos0, H, KV, D)
    assert np.array_equal(out, f["out_scalar"]), "scalar restatement must be bit-identical to cpu::attention_heads"
    qscale = max(1.0, float(np.abs(f["q"]).max()) / 4.0)
    assert np.abs(out - f["out_backend"]).max() <= 2e-6 * max(1.0, qscale)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "rope_*.npz"))),
                         ids=lambda p: os.path.basename(p)[5:-4])
def test_rope_matches_golden(path):
    f = np.load(path)
    n, H, D, pos0, neox = (int(x) for x in f["meta"])
    ff = f["ff"] if f["ff"].size else None
    out = oracle.rope(f["x"], H, D, pos0, float(f["base"]), bool(neox), ff)
    assert np.array_equal(out, f["out"])


def test_softmax_matches_golden():
    f = np.load(os.path.join(GOLD, "softmax.npz"))
    assert np.array_equal(oracle.softmax(f["x"]), f["out"])


def test_fp16_matches_golden():
    f = np.load(os.path.join(GOLD, "fp16.npz"))
    widened = oracle.fp16_bits_to_f32(np.arange(65536, dtype=np.uint16))
    same = (widened.view(np.uint32) == f["widened"].view(np.uint32))
    assert same.all(), "every fp16 bit pattern (NaN payloads included) widens like src/fp16.h"
    assert np.array_equal(oracle.f32_to_fp16_bits(f["sample"]), f["narrowed"])
    # numpy's IEEE conversion agrees with the reference on finite values (round to nearest even)
    fin = np.isfinite(f["sample"]) & (np.abs(f["sample"]) < 65520)
    assert np.array_equal(f["sample"][fin].astype(np.float16).view(np.uint16), f["narrowed"][fin])


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.1415927, 1e-40, np.inf], np.float32)
    bits = oracle.f32_to_bf16_bits(x)
    back = oracle.bf16_bits_to_f32(bits)
    assert back[0] == 1.0 and back[1] == 1.0 and back[2] == np.float32(1.0078125)
    assert back[5] == np.inf
    assert np.all(np.abs(back[:4] - x[:4]) <= np.abs(x[:4]) * 2.0 ** -8)


def test_gather_pages_layout():
    KV, D, P = 2, 4, 16
    n_pages, length = 5, 37
    rng = np.random.default_rng(1)
    pool = rng.integers(0, 2 ** 14, size=(n_pages, 2, KV, P, D), dtype=np.uint16)  # finite fp16 patterns
    table = np.array([3, 0, 4], np.int32)
    k, v = oracle.gather_pages(pool, table, length, KV, D, P)
    for j in (0, 15, 16, 36):
        page, slot = table[j // P], j % P
        np.testing.assert_array_equal(k[j], oracle.fp16_bits_to_f32(pool[page, 0, :, slot, :]))
        np.testing.assert_array_equal(v[j], oracle.fp16_bits_to_f32(pool[page, 1, :, slot, :]))


# ---------------------------------------------------------------- live reference (where it was built)
needs_ref = pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (no reference tree)")


@needs_ref
@pytest.mark.parametrize("shape", [(1, 0, 14, 2, 64), (9, 31, 32, 8, 64), (3, 100, 32, 4, 64), (2, 5, 6, 3, 10)])
def test_oracle_bit_identical_to_reference(shape):
    n, pos0, H, KV, D = shape
    rng = np.random.default_rng(sum(shape))
    q = rng.standard_normal((n, H, D)).astype(np.float32)
    k = rng.standard_normal((pos0 + n, KV, D)).astype(np.float32)
    v = rng.standard_normal((pos0 + n, KV, D)).astype(np.float32)
    assert np.array_equal(oracle.attention(q, k, v, n, pos0, H, KV, D),
                          oracle.ref_attention_scalar(q, k, v, n, pos0, H, KV, D))
    x = rng.standard_normal((n, H, D)).astype(np.float32)
    for neox in (False, True):
        assert np.array_equal(oracle.rope(x, H, D, pos0 + 70000, 5e5, neox),
                              oracle.ref_rope(x, H, D, pos0 + 70000, 5e5, neox))


# ---------------------------------------------------------------- the model's other ops (backend.h:54-70)
# Known answers restated from the reference's own tests (tests/test_ref_ops.cpp:33-37, :98-103, :106-127).
def test_rmsnorm_known_answer():
    x = np.array([1, 2, 3, 4], np.float32)
    y = oracle.rmsnorm(x, np.ones(4, np.float32), 1, 0.0)[0]
    assert np.allclose(y, x / np.sqrt(7.5), rtol=1e-6, atol=1e-7)


def test_silu_mul_known_answer():
    g = oracle.silu_mul(np.array([0, 1], np.float32), np.array([2, 3], np.float32))
    assert np.allclose(g, [0.0, 3.0 / (1.0 + np.exp(-1.0))], rtol=1e-6, atol=1e-7)


def test_matmul_and_embed_known_answer():
    w = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    x = np.ones((1, 3), np.float32)
    y = oracle.matmul(w, x, 1)[0]
    assert np.allclose(y, [6, 15], rtol=1e-6)
    wh = oracle.f32_to_fp16_bits(w)
    assert np.array_equal(oracle.matmul(wh, x, 1)[0], y)
    assert np.array_equal(oracle.embed(wh, np.array([1], np.int32))[0], [4, 5, 6])


@pytest.mark.parametrize("dt", ["f32", "f16"])
@pytest.mark.parametrize("shape", [(1, 3, 5), (5, 37, 72), (9, 64, 130), (3, 1, 1)])
def test_model_ops_bit_identical_to_reference(dt, shape):
    if not oracle.have_ref():
        pytest.skip("oracle/_ref (nibble's own code) is not built here")
    n, ne1, ne0 = shape
    rng = np.random.default_rng(n * 1000 + ne1 + ne0)
    w = (rng.standard_normal((ne1, ne0)) * 0.2).astype(np.float32)
    if dt == "f16":
        w = oracle.f32_to_fp16_bits(w)
    x = rng.standard_normal((n, ne0)).astype(np.float32)
    assert np.array_equal(oracle.matmul(w, x, n).view(np.uint32), oracle.ref_matmul(w, x, n).view(np.uint32))
    ids = rng.integers(0, ne1, n).astype(np.int32)
    assert np.array_equal(oracle.embed(w, ids).view(np.uint32), oracle.ref_embed(w, ids).view(np.uint32))
    norm_w = rng.standard_normal(ne0).astype(np.float32)
    for eps in (1e-6, 1e-5, 0.0):
        assert np.array_equal(oracle.rmsnorm(x * 3, norm_w, n, eps).view(np.uint32),
                              oracle.ref_rmsnorm(x * 3, norm_w, n, eps).view(np.uint32))
    g = (rng.standard_normal(n * ne0) * 6).astype(np.float32)
    u = rng.standard_normal(n * ne0).astype(np.float32)
    assert np.array_equal(oracle.silu_mul(g, u).view(np.uint32), oracle.ref_silu_mul(g, u).view(np.uint32))
    assert np.array_equal(oracle.add(g, u).view(np.uint32), oracle.ref_add(g, u).view(np.uint32))


def test_embed_out_of_range_matches_reference_error():
    w = np.zeros((7, 4), np.float32)
    with pytest.raises(ValueError):
        oracle.embed(w, np.array([7], np.int32))
    if oracle.have_ref():
        with pytest.raises(ValueError, match=r"embed: token id 7 out of range \(n_vocab 7\)"):
            oracle.ref_embed(w, np.array([7], np.int32))


# ---------------------------------------------------------------- quantized weights (Q8_0-activation family)
@pytest.mark.parametrize("dtype", [oracle.Q4_0, oracle.Q5_0, oracle.Q8_0])
def test_quant_oracle_bit_identical_to_reference(dtype):
    """Activation quantizer, row dequantization and the quantized matmul against nibble's own scalar code
    (src/quant.cpp via oracle/_ref), including an all-zero block and one of tiny magnitude."""
    if not oracle.have_ref():
        pytest.skip("oracle/_ref (nibble's own code) is not built here")
    rng = np.random.default_rng(dtype)
    x = (rng.standard_normal(32 * 9) * 3).astype(np.float32)
    x[:32] = 0.0
    x[32:64] *= 1e-30
    assert np.array_equal(oracle.quantize_q8_0(x), oracle.ref_quantize_q8_0(x))
    w = oracle.random_q_blocks(rng, dtype, 23, 160)
    a = oracle.dequantize_rows(w, dtype, 160, 23)
    b = oracle.ref_dequantize_rows(w, dtype, 160, 23)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    xs = x[:160 * 1].reshape(1, 160).repeat(3, axis=0) * np.array([[1.0], [0.5], [-2.0]], np.float32)
    y = oracle.matmul_q(w, dtype, 160, 23, xs, 3)
    yr = oracle.ref_matmul_q(w, dtype, 160, 23, xs, 3)
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


def test_quantize_q8_0_known_answer():
    """One block: d = max|x| / 127 and q = round(x / d), half away from zero (src/quant.cpp:37-51)."""
    x = np.zeros(32, np.float32)
    x[0], x[1], x[2], x[3] = 127.0, -63.5, 0.4, -127.0
    blk = oracle.quantize_q8_0(x)
    d = oracle.fp16_bits_to_f32(np.array([int(blk[0]) | (int(blk[1]) << 8)], np.uint16))[0]
    q = blk[2:].view(np.int8)
    assert d == 1.0 and list(q[:4]) == [127, -64, 0, -127] and not q[4:].any()


# ---------------------------------------------------------------- Q5_1 (Q8_1 activations) and the k-quants (Q8_K)
def _activation_edge_rows(rng, n):
    """n floats: random rows plus an all-zero 256-block, one of tiny magnitude, one whose largest magnitude is
    tied between a negative and a positive element (the first one wins), and one with a NaN."""
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    x[:256] = 0.0
    x[256:512] *= 1e-30
    x[512:768] = np.clip(x[512:768], -2.0, 2.0)
    x[512 + 7], x[512 + 9] = -5.0, 5.0
    return x


def test_q8_1_and_q8_K_quantizers_bit_identical_to_reference():
    if not oracle.have_ref():
        pytest.skip("oracle/_ref (nibble's own code) is not built here")
    rng = np.random.default_rng(17)
    x = _activation_edge_rows(rng, 256 * 6)
    x[1024 + 100] = np.nan
    assert np.array_equal(oracle.quantize_q8_1(x), oracle.ref_quantize_q8_1(x))
    assert np.array_equal(oracle.quantize_q8_K(x), oracle.ref_quantize_q8_K(x))
    # the tie: max = x[7] = -5 gives iscale = 127 / 5 > 0, so x[9] = 5 quantizes to +127
    blk = oracle.quantize_q8_K(x[512:768])
    q = blk[4:260].view(np.int8)
    assert q[7] == -127 and q[9] == 127
    assert oracle.quantize_q8_K(x[:256]).view(np.uint8).sum() == 0  # all-zero block: d, qs and sums zero


@pytest.mark.parametrize("dtype", [oracle.Q5_1, oracle.Q4_K, oracle.Q5_K, oracle.Q6_K])
def test_block_quant_oracle_bit_identical_to_reference(dtype):
    """Row dequantization and the quantized matmul (activations quantized to Q8_1 / Q8_K, the reference's block
    dots) against nibble's own scalar code (src/quant.cpp via oracle/_ref), over random blocks whose packed scale
    bytes, high bits and fp16 scales take arbitrary values."""
    if not oracle.have_ref():
        pytest.skip("oracle/_ref (nibble's own code) is not built here")
    rng = np.random.default_rng(dtype + 100)
    ne0, ne1 = 768, 29
    w = oracle.random_q_blocks(rng, dtype, ne1, ne0)
    a = oracle.dequantize_rows(w, dtype, ne0, ne1)
    b = oracle.ref_dequantize_rows(w, dtype, ne0, ne1)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    x = _activation_edge_rows(rng, ne0 * 4).reshape(4, ne0)
    y = oracle.matmul_q(w, dtype, ne0, ne1, x, 4)
    yr = oracle.ref_matmul_q(w, dtype, ne0, ne1, x, 4)
    assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
    # the same weights through CpuBackend (the SIMD tier the reference runs) agree bit for bit too
    be = oracle.RefBackend(2)
    try:
        yb = be.matmul(w, dtype, ne0, ne1, x, 4)
    finally:
        be.close()
    assert np.array_equal(yb.view(np.uint32), yr.view(np.uint32))


def test_quant_oracle_matches_reference_golden_vectors():
    """The oracle's Q8_0 / Q8_1 / Q8_K quantizers, every block dot and every dequantization against the golden
    vectors nibble ships (llama.cpp's outputs on inputs regenerated by nibble's own generators and checked by hash):
    oracle/golden_quant.cpp, built from the reference tree where it is present."""
    import subprocess
    if not os.path.exists(oracle.GOLDEN_CHECK):
        pytest.skip("oracle/_ref/nbl_golden_check is built only where the reference tree is present")
    r = subprocess.run([oracle.GOLDEN_CHECK], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "golden checks passed" in r.stdout


def test_activation_quantizers_on_hostile_rows_bit_identical_to_reference():
    """Rows a corrupt or overflowing model can produce -- +-Inf, NaN, a subnormal largest magnitude (an infinite
    inverse scale), values near the float maximum -- quantize to the same bytes as nibble's own Q8_0 / Q8_1 / Q8_K
    quantizers (src/quant.cpp:37-51, :250-307 define every one of these cases)."""
    if not oracle.have_ref():
        pytest.skip("oracle/_ref (nibble's own code) is not built here")
    rng = np.random.default_rng(23)
    rows = []
    for fill in ("inf", "ninf", "nan", "subnormal", "huge", "mixed"):
        x = (rng.standard_normal(256) * 3).astype(np.float32)
        if fill == "inf":
            x[17] = np.inf
        elif fill == "ninf":
            x[200] = -np.inf
        elif fill == "nan":
            x[5] = np.nan
        elif fill == "subnormal":
            x = (rng.standard_normal(256) * 1e-42).astype(np.float32)
        elif fill == "huge":
            x = (np.clip(rng.standard_normal(256), -3.0, 3.0) * 1e38).astype(np.float32)
        else:
            x[::7] = 0.0
            x[3], x[4] = np.inf, np.nan
        rows.append(x)
    x = np.concatenate(rows)
    with np.errstate(all="ignore"):
        assert np.array_equal(oracle.quantize_q8_0(x), oracle.ref_quantize_q8_0(x))
        assert np.array_equal(oracle.quantize_q8_1(x), oracle.ref_quantize_q8_1(x))
        assert np.array_equal(oracle.quantize_q8_K(x), oracle.ref_quantize_q8_K(x))


# ---------------------------------------------------------------- known answers for Q5_1 / Q8_1 / Q8_K / k-quants
# Hand-built blocks whose values follow from the formats (src/quant.h:50-99); the cases restate the reference's own
# known-answer tests (tests/test_quant.cpp:286-327, :466-496, :612-655) with the expected values derived here.
def _f16(v):
    return int(oracle.f32_to_fp16_bits(np.array([v], np.float32))[0])


def _put16(blk, off, v):
    h = _f16(v)
    blk[off], blk[off + 1] = h & 0xFF, h >> 8


def test_q5_1_known_answer():
    blk = np.zeros(24, np.uint8)
    _put16(blk, 0, 0.5)    # d
    _put16(blk, 2, -1.0)   # m
    blk[4 + 2] = 0x01      # qh bit 16: element 16's fifth bit
    blk[8] = 0x10          # qs[0]: element 0 = 0, element 16 = 1
    y = oracle.dequantize_rows(blk, oracle.Q5_1, 32, 1)[0]
    assert y[0] == -1.0            # 0 * 0.5 - 1
    assert y[16] == 7.5            # (1 + 16) * 0.5 - 1
    assert y[17] == -1.0


def test_q8_1_known_answer():
    blk = oracle.quantize_q8_1(np.full(32, 127.0, np.float32))
    h = blk[:4].view(np.uint16)
    assert h[0] == _f16(1.0)        # d = 127 / 127
    assert h[1] == _f16(4064.0)     # s = 32 * 127 * d
    assert np.all(blk[4:].view(np.int8) == 127)
    assert not oracle.quantize_q8_1(np.zeros(32, np.float32)).any()


def test_q8_K_known_answer():
    x = np.zeros(256, np.float32)
    x[:4] = [-127.0, 2.5, 3.5, -2.5]
    blk = oracle.quantize_q8_K(x)
    q = blk[4:260].view(np.int8)
    assert blk[:4].view(np.float32)[0] == 1.0          # iscale = -127 / -127, d = 1 / iscale
    assert list(q[:4]) == [-127, 2, 4, -2]             # half to even, not half away from zero
    sums = blk[260:292].view(np.int16)
    assert sums[0] == -123 and not sums[1:].any()
    x = np.zeros(256, np.float32)
    x[0] = 127.0
    blk = oracle.quantize_q8_K(x)
    assert blk[:4].view(np.float32)[0] == -1.0 and blk[4:260].view(np.int8)[0] == -127  # the sign flips into d


def _k_scales():
    """Packed 6-bit scales / minimums with sub-block 0 = (2, 3), 1 = (1, 1), 4 = (17, 18): sub-blocks 4-7 keep their
    low four bits in the nibbles of bytes 8-11 and their top two bits in bits 6-7 of bytes 0-3 (scale) / 4-7 (min)."""
    s = np.zeros(12, np.uint8)
    s[0] = 2 | (17 >> 4) << 6
    s[4] = 3 | (18 >> 4) << 6
    s[1], s[5] = 1, 1
    s[8] = (17 & 15) | (18 & 15) << 4
    return s


@pytest.mark.parametrize("dtype", [oracle.Q4_K, oracle.Q5_K])
def test_q4_K_q5_K_known_answer(dtype):
    blk = np.zeros(oracle.BLOCK_BYTES[dtype], np.uint8)
    _put16(blk, 0, 1.0)    # d
    _put16(blk, 2, 0.5)    # dmin
    blk[4:16] = _k_scales()
    qs = 48 if dtype == oracle.Q5_K else 16
    blk[qs + 0] = 0x5A     # element 0 = 10 (sub-block 0), element 32 = 5 (sub-block 1)
    blk[qs + 64] = 0x03    # element 128 = 3 (sub-block 4)
    if dtype == oracle.Q5_K:
        blk[16] = 0x01     # element 0's fifth bit
    y = oracle.dequantize_rows(blk, dtype, 256, 1)[0]
    assert y[0] == (2 * 26 - 0.5 * 3 if dtype == oracle.Q5_K else 2 * 10 - 0.5 * 3)
    assert y[32] == 1 * 5 - 0.5 * 1
    assert y[128] == 17 * 3 - 0.5 * 18


def test_q6_K_known_answer():
    blk = np.zeros(210, np.uint8)
    _put16(blk, 208, 0.5)
    blk[192] = 2                      # scale of elements 0-15
    blk[192 + 4] = np.uint8(0xFF)     # scale -1 for elements 64-79
    blk[0] = 0x21                     # element 0 low bits 1, element 64 low bits 2
    blk[128] = 0x03                   # element 0 high bits 3
    y = oracle.dequantize_rows(blk, oracle.Q6_K, 256, 1)[0]
    assert y[0] == 0.5 * 2 * ((1 | 3 << 4) - 32)
    assert y[64] == 0.5 * -1 * (2 - 32)


@pytest.mark.parametrize("dtype", [oracle.Q4_K, oracle.Q5_K, oracle.Q6_K])
def test_k_dot_against_zero_activations_is_zero(dtype):
    rng = np.random.default_rng(dtype)
    w = oracle.random_q_blocks(rng, dtype, 1, 256)
    act = oracle.quantize_q8_K(np.zeros(256, np.float32))
    assert oracle.vec_dot(dtype, w[0], act, 1) == 0.0
