"""The arithmetic identities the tensor-core matmuls rely on, checked on the CPU with numpy (no GPU, no library):

* quant_gemm.cu turns an int32 block dot s into a float exactly as (float with bits 0x4B400000 + s) - 1.5 * 2^23,
  valid for |s| < 2^22; a Q8_0 block dot is at most 32 * 128 * 127 in magnitude.
* f32_gemm.cu splits an activation row for the fp16 MMAs: scale by 2^-s so the row's largest magnitude lies in
  [2^13, 2^14), t1 = fp16(x'), t2 = fp16(x' - t1); the remainder is below 2^-22 of the element (or, where t2 is
  subnormal, 2^-38 of the row's largest magnitude), products of fp16 terms and F16 weights are exact in fp32, and
  scaling back by 2^s is exact.
* For F32 weights it splits both operands into tf32 terms (round to nearest, ties away from zero, to 10 stored
  mantissa bits); hi + lo carries all but 2^-22 of the value.
"""
import numpy as np


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
