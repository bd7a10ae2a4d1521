"""The arithmetic identities the tensor-core matmuls rely on, checked on the CPU with numpy (no GPU, no library):

* quant_gemm.cu turns an int32 block dot s into a float exactly as (float with bits 0x4B400000 + s) - 1.5 * 2^23,
  valid for |s| < 2^22; a Q8_0 block dot is at most 32 * 128 * 127 in magnitude.
* f32_gemm.cu splits an activation row for the fp16 MMAs: scale by 2^-s so the row's largest magnitude lies in
  [2^13, 2^14), t1 = fp16(x'), t2 = fp16(x' - t1); the remainder is below 2^-22 of the element (or, where t2 is
  subnormal, 2^-38 of the row's largest magnitude), products of fp16 terms and F16 weights are exact in fp32, and
  scaling back by 2^s is exact.
* For F32 weights it splits both operands into tf32 terms (round to nearest, ties away from zero, to 10 stored
  mantissa bits); hi + lo carries all but 2^-22 of the value.
* quant_blocks.cu's k-quant decode kernel regroups the reference's eight per-super-block integer accumulators by
  lane and carries the nine float chains through chunks of super-blocks; restated in numpy it equals the
  reference's dot bit for bit.
"""
import numpy as np

import oracle


def test_exact_int_to_float_trick():
    s = np.concatenate([np.arange(-70000, 70000, dtype=np.int64),
                        np.array([-(2 ** 22) + 1, 2 ** 22 - 1, 32 * 128 * 127, -32 * 128 * 127])])
    bits = (np.uint32(0x4B400000) + s.astype(np.uint32)).astype(np.uint32)  # wraps like the device's 32-bit add
    f = bits.view(np.float32) - np.float32(12582912.0)
    assert np.array_equal(f.astype(np.int64), s)
    assert np.array_equal(f, s.astype(np.float32))


def _fp16_split(row):
    """The device's split of one activation row (split_f16_rows_kernel)."""
    m = np.max(np.abs(row))
    sh = int(np.frexp(m)[1]) - 14 if m > 0 else 0
    down = np.float32(np.ldexp(1.0, -sh))
    v = (row * down).astype(np.float32)
    t1 = v.astype(np.float16)
    t2 = (v - t1.astype(np.float32)).astype(np.float16)
    return t1, t2, np.float32(np.ldexp(1.0, sh)), v


def test_fp16_split_of_scaled_rows():
    rng = np.random.default_rng(0)
    for scale in (1e-6, 1e-2, 1.0, 37.0, 1e4, 3e7):
        row = (rng.standard_normal(4096) * scale).astype(np.float32)
        row[:5] = [0.0, -0.0, scale * 1e-9, -scale * 3e-12, scale * 200]  # tiny and large elements in one row
        t1, t2, up, v = _fp16_split(row)
        assert np.all(np.isfinite(t1)) and np.all(np.isfinite(t2))
        assert np.max(np.abs(v)) < 2.0 ** 14
        rem = v.astype(np.float64) - t1.astype(np.float64) - t2.astype(np.float64)
        bound = np.maximum(2.0 ** -22 * np.abs(v.astype(np.float64)), 2.0 ** -38 * np.max(np.abs(v)))
        assert np.all(np.abs(rem) <= bound)
        # scaling back by a power of two is exact
        assert np.array_equal((v * up).astype(np.float32), row)


def test_fp16_products_are_exact_in_fp32():
    rng = np.random.default_rng(1)
    a = rng.standard_normal(10000).astype(np.float16)
    b = (rng.standard_normal(10000) * 1000).astype(np.float16)
    exact = a.astype(np.float64) * b.astype(np.float64)
    assert np.array_equal(exact.astype(np.float32).astype(np.float64), exact)


def _tf32(x):
    """Round fp32 to tf32 (10 stored mantissa bits), to nearest with ties away from zero (cvt.rna)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x1000) & 0xFFFFE000
    return u.astype(np.uint32).view(np.float32)


def test_tf32_split_carries_all_but_2_pow_minus_22():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    hi = _tf32(x)
    lo = _tf32((x - hi).astype(np.float32))
    assert np.array_equal((x.astype(np.float64) - hi), (x - hi).astype(np.float64))  # the difference is exact
    rem = x.astype(np.float64) - hi.astype(np.float64) - lo.astype(np.float64)
    assert np.all(np.abs(rem) <= 2.0 ** -22 * np.abs(x.astype(np.float64)))
    # the low 13 bits of every term are zero (what the tensor core reads of a tf32 operand)
    assert not np.any(hi.view(np.uint32) & 0x1FFF) and not np.any(lo.view(np.uint32) & 0x1FFF)


# ---------------------------------------------------------------- the k-quant decode kernel's decomposition
def _k_values_and_scales(dtype, blk):
    """A k-quant super-block's 256 integer values and each element's sub-block scale (src/quant.cpp:67-96), plus
    the eight Q4_K / Q5_K minimums."""
    v = np.zeros(256, np.int64)
    if dtype == oracle.Q6_K:
        for h in range(2):
            ql, qh = blk[64 * h:64 * h + 64].astype(np.int64), blk[128 + 32 * h:160 + 32 * h].astype(np.int64)
            v[128 * h:128 * h + 32] = (ql[:32] & 15) | ((qh & 3) << 4)
            v[128 * h + 32:128 * h + 64] = (ql[32:] & 15) | (((qh >> 2) & 3) << 4)
            v[128 * h + 64:128 * h + 96] = (ql[:32] >> 4) | (((qh >> 4) & 3) << 4)
            v[128 * h + 96:128 * h + 128] = (ql[32:] >> 4) | (((qh >> 6) & 3) << 4)
        return v - 32, np.repeat(blk[192:208].view(np.int8).astype(np.int64), 16), None
    q = blk[4:16].astype(np.int64)
    sc = [q[j] & 63 if j < 4 else (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4) for j in range(8)]
    mn = [q[j + 4] & 63 if j < 4 else (q[j + 4] >> 4) | ((q[j] >> 6) << 4) for j in range(8)]
    qs = blk[48:176] if dtype == oracle.Q5_K else blk[16:144]
    qh = blk[16:48].astype(np.int64)
    for c in range(4):
        b = qs[32 * c:32 * c + 32].astype(np.int64)
        v[64 * c:64 * c + 32], v[64 * c + 32:64 * c + 64] = b & 15, b >> 4
        if dtype == oracle.Q5_K:
            v[64 * c:64 * c + 32] += ((qh >> (2 * c)) & 1) << 4
            v[64 * c + 32:64 * c + 64] += ((qh >> (2 * c + 1)) & 1) << 4
    return v, np.repeat(np.array(sc, np.int64), 32), np.array(mn, np.int64)


def _decode_kernel_dot(dtype, wrow, act, nb, chunk=16):
    """kquant_gemv_kernel's arithmetic for one (weight row, activation row): the activation block relaid lane-major
    (lane i holds elements i + 32 j) with eight 32-element sums, lane i's share of accumulator lane i % 8, the four
    lanes i, i^8, i^16, i^24 added, then the float chains carried through chunks of `chunk` super-blocks."""
    bb = oracle.BLOCK_BYTES[dtype]
    st = np.zeros(8, np.float32)
    tot = np.float32(0.0)
    for b0 in range(0, nb, chunk):
        parts = []
        for b in range(b0, min(nb, b0 + chunk)):
            blk = wrow[b * bb:(b + 1) * bb]
            a = act[b * 292:(b + 1) * 292]
            da = a[:4].view(np.float32)[0]
            aq = a[4:260].view(np.int8).astype(np.int64)
            lane_major = aq.reshape(8, 32).T            # [lane][j] = element lane + 32 j
            pair_sums = aq.reshape(8, 32).sum(axis=1)   # bsums[2k] + bsums[2k + 1]
            v, sc, mn = _k_values_and_scales(dtype, blk)
            share = (sc.reshape(8, 32).T * lane_major * v.reshape(8, 32).T).sum(axis=1)  # per lane
            acc = np.array([share[l] + share[l ^ 8] + share[l ^ 16] + share[l ^ 24] for l in range(8)])
            sumi = int((pair_sums * mn).sum()) if mn is not None else 0
            parts.append((blk, da, acc, sumi))
        for blk, da, acc, sumi in parts:  # phase 2, in super-block order
            dw = oracle.fp16_bits_to_f32(blk[208:210].view(np.uint16) if dtype == oracle.Q6_K else blk[0:2].view(np.uint16))[0]
            d = np.float32(dw * da)
            st = (st + (d * acc.astype(np.float32)).astype(np.float32)).astype(np.float32)
            if mn is not None:
                dmin = np.float32(oracle.fp16_bits_to_f32(blk[2:4].view(np.uint16))[0] * da)
                tot = np.float32(tot - np.float32(dmin * np.float32(sumi)))
    res = tot
    for l in range(8):
        res = np.float32(res + st[l])
    return res


def test_kquant_decode_decomposition_equals_reference_dot():
    """The decode kernel regroups the reference's eight integer accumulators by lane and runs its nine float chains
    in chunks of 16 super-blocks; restated here in numpy, that equals nibble's dot (through the oracle, pinned to
    it and to llama.cpp's golden vectors) bit for bit, across a chunk boundary (20 super-blocks)."""
    rng = np.random.default_rng(9)
    nb = 20
    for dtype in (oracle.Q4_K, oracle.Q5_K, oracle.Q6_K):
        w = oracle.random_q_blocks(rng, dtype, 4, 256 * nb)
        for r in range(4):
            act = oracle.quantize_q8_K((rng.standard_normal(256 * nb) * 2).astype(np.float32))
            got = _decode_kernel_dot(dtype, w[r], act, nb)
            ref = oracle.vec_dot(dtype, w[r], act, nb)
            assert np.float32(got).view(np.uint32) == np.float32(ref).view(np.uint32), (dtype, r, got, ref)
