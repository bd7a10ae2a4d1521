"""The drop-in Backend ops served from fp16 pages (nbl_ctx_set_paged_kv), driven through the C ABI in exactly the
order nibble's Transformer calls them for one layer (src/model/transformer.cpp:171-202):

    matmul_multi([wq, wk, wv], h, [q, k + pos0*kvw, v + pos0*kvw], n)      K/V projected into the cache rows
    add_bias(q, bq), add_bias(kc, bk), add_bias(vc, bv)                     (qwen2 only)
    rope(q, n, H, 64, pos0), rope(kc, n, KVH, 64, pos0)
    attention(q, k, v, out, n, pos0, H, KVH, 64)

over a sequence of chunks (prefill chunks of more than 8 rows, short chunks, single-token decode steps). A second
context runs the same calls with the route off (the reference's flat fp32 cache); its matmuls are the same kernels,
so its K/V rows and roped queries are the exact fp32 values the paged context rounds.

Checked:
  * the cache: reading the paged context's K/V blocks back gives the flat context's rows rounded to fp16 (RNE),
    bit for bit (the fused bias + RoPE + append equals add_bias, cpu::rope and narrowing);
  * the roped queries: bit-identical to the flat context's;
  * every attention output against the C oracle (nibble's scalar attention restated, pinned bit-exactly to the
    reference by test_oracle.py) on the fp16 cache: decode chunks (up to 8 rows, split-K decode kernel, fp32
    accumulate) max relative error per head <= 1e-4; prefill chunks (tcgen05, fp16 queries) max abs error <= 2e-2
    and cosine >= 0.9999 per head, the queries rounded to fp16 for the oracle as the kernel consumes them;
  * reading the cache back between chunks (pages turned back into flat rows, converted again at the next attention)
    changes no output bit.
"""
import numpy as np
import pytest

import oracle
from helpers import max_rel_err_per_head, min_cosine_per_head

pytestmark = pytest.mark.gpu
D = 64
CHUNKS = [37, 1, 1, 5, 20, 1, 8, 9, 1, 130, 1]  # prefill, decode steps, short chunks, a long chunk over a prefix
N_CTX = 256
E = 128


class Layer:
    """One attention layer's weights and buffers in one context, driven like run_chunk."""

    def __init__(self, ctx, H, KV, bias, spec, w, n_ctx, max_rows, wdtype=np.float32):
        import torch
        self.ctx, self.H, self.KV, self.spec = ctx, H, KV, spec
        self.kvw = KV * D
        ctx.reserve(n_ctx, H, max_rows, max(E, H * D))
        self.k = ctx.alloc(n_ctx * self.kvw)
        self.v = ctx.alloc(n_ctx * self.kvw)
        self.h = ctx.alloc(max_rows * E)
        self.q = ctx.alloc(max_rows * H * D)
        self.out = ctx.alloc(max_rows * H * D)
        if isinstance(wdtype, str):  # GGUF blocks of a quantized type, made by run_case
            import nibble_b200 as nb
            code = getattr(nb._abi, wdtype)
            self.wq, self.wk, self.wv = (ctx.weight(a, code, E) for a in w[:3])
        else:
            self.wq, self.wk, self.wv = (ctx.weight(a.astype(wdtype)) for a in w[:3])
        self.b = [ctx.weight(a) for a in w[3:]] if bias else None
        self.bdev = None
        if bias:
            from nibble_b200 import _abi
            import ctypes as C
            self.bdev = []
            for wt in self.b:
                p = C.c_void_p()
                _abi.check(_abi.lib.nbl_weight_data(wt.handle, C.byref(p), None, None, None))
                self.bdev.append(p.value)
        del torch

    def chunk(self, x, pos0):
        n = x.shape[0]
        ctx, H, KV, kvw = self.ctx, self.H, self.KV, self.kvw
        ctx.write(self.h, np.ascontiguousarray(x, np.float32), n * E)
        kc, vc = self.k + pos0 * kvw * 4, self.v + pos0 * kvw * 4
        ctx.matmul_multi([self.wq, self.wk, self.wv], self.h, [self.q, kc, vc], n)
        if self.bdev:
            ctx.add_bias(self.q, self.bdev[0], H * D, n)
            ctx.add_bias(kc, self.bdev[1], kvw, n)
            ctx.add_bias(vc, self.bdev[2], kvw, n)
        ctx.rope(self.q, n, H, D, pos0, self.spec)
        ctx.rope(kc, n, KV, D, pos0, self.spec)
        ctx.attention(self.q, self.k, self.v, self.out, n, pos0, H, KV, D)

    def read(self, ptr, count):
        a = np.empty(count, np.float32)
        self.ctx.read(a, ptr, count)
        return a


def run_case(H, KV, bias, spec, seed, read_between, wdtype=np.float32):
    import nibble_b200 as nb
    rng = np.random.default_rng(seed)
    w = [(rng.standard_normal((H * D, E)) / np.sqrt(E)).astype(np.float32),
         (rng.standard_normal((KV * D, E)) / np.sqrt(E)).astype(np.float32),
         (rng.standard_normal((KV * D, E)) / np.sqrt(E)).astype(np.float32),
         (rng.standard_normal(H * D) * 0.5).astype(np.float32),
         (rng.standard_normal(KV * D) * 0.5).astype(np.float32),
         (rng.standard_normal(KV * D) * 0.5).astype(np.float32)]
    xs = [rng.standard_normal((n, E)).astype(np.float32) for n in CHUNKS]
    if isinstance(wdtype, str):
        w[:3] = [oracle.random_q_blocks(rng, getattr(oracle, wdtype), rows, E, scale=0.01)
                 for rows in (H * D, KV * D, KV * D)]
    cp, cf = nb.Context(0), nb.Context(0)
    cp.set_paged_kv(True)
    lp = Layer(cp, H, KV, bias, spec, w, N_CTX, 160, wdtype)
    lf = Layer(cf, H, KV, bias, spec, w, N_CTX, 160, wdtype)
    outs, queries = [], []
    pos0 = 0
    for x in xs:
        n = x.shape[0]
        lp.chunk(x, pos0)
        lf.chunk(x, pos0)
        out = lp.read(lp.out, n * H * D).reshape(n, H, D)
        qp = lp.read(lp.q, n * H * D).reshape(n, H, D)  # applies the recorded rope of q where it is still pending
        qf = lf.read(lf.q, n * H * D).reshape(n, H, D)
        assert np.array_equal(qp.view(np.uint32), qf.view(np.uint32)), f"roped queries differ at pos0 {pos0}"
        L = pos0 + n
        kf = lf.read(lf.k, L * KV * D).reshape(L, KV, D)
        vf = lf.read(lf.v, L * KV * D).reshape(L, KV, D)
        k16 = oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(kf))
        v16 = oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(vf))
        if read_between:
            kp = lp.read(lp.k, L * KV * D).reshape(L, KV, D)
            vp = lp.read(lp.v, L * KV * D).reshape(L, KV, D)
            assert np.array_equal(kp.view(np.uint32), k16.view(np.uint32)), f"K cache differs at pos0 {pos0}"
            assert np.array_equal(vp.view(np.uint32), v16.view(np.uint32)), f"V cache differs at pos0 {pos0}"
        q_or = qf if n <= 8 else oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(qf))
        ref = oracle.attention(q_or, k16, v16, n, pos0, H, KV, D)
        if n <= 8:
            err = max_rel_err_per_head(out, ref)
            assert err <= 1e-4, f"decode chunk at {pos0} (n={n}): rel err {err}"
        else:
            err = float(np.abs(out - ref).max())
            cos = min_cosine_per_head(out, ref)
            assert err <= 2e-2 and cos >= 0.9999, f"prefill chunk at {pos0} (n={n}): abs {err} cos {cos}"
        outs.append(out)
        queries.append(qp)
        pos0 += n
    # at the end the whole paged cache is the flat one rounded to fp16
    kp = lp.read(lp.k, pos0 * KV * D)
    kf = lf.read(lf.k, pos0 * KV * D)
    assert np.array_equal(kp.view(np.uint32), oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(kf)).view(np.uint32))
    cp.check()
    cf.check()
    cp.close()
    cf.close()
    return outs


CASES = {
    "qwen_g7_neox_bias": (14, 2, True, dict(freq_base=1e6, neox=True)),
    "llama_g4_interleaved_factors": (32, 8, False, dict(freq_base=5e5, neox=False,
                                                        freq_factors=tuple(float(x) for x in np.linspace(1, 8, 32)))),
}


@pytest.mark.parametrize("wdtype", [np.float32, np.float16, "Q4_0", "Q8_0"], ids=["F32", "F16", "Q4_0", "Q8_0"])
@pytest.mark.parametrize("name", list(CASES))
def test_transformer_layer_sequence_on_pages(name, wdtype):
    """Chunks of up to 8 rows run the recorded Q/K/V projection with bias + RoPE + page write in its epilogue (one
    launch: the float GEMV, or the quantized GEMV after its activation quantizer); longer chunks the projection,
    then one append launch. Both must reproduce the flat context's rows."""
    import nibble_b200 as nb
    H, KV, bias, sp = CASES[name]
    spec = nb.RopeSpec(**sp)
    plain = run_case(H, KV, bias, spec, seed=len(name), read_between=False, wdtype=wdtype)
    checked = run_case(H, KV, bias, spec, seed=len(name), read_between=True, wdtype=wdtype)
    for a, b in zip(plain, checked):  # converting the cache back and forth changes no bit
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_other_ops_on_paged_blocks_keep_backend_meaning():
    """Ops the Transformer never issues on cache rows still mean what they mean on CpuBackend: a read of the cache
    between the projection and attention, a copy into cache rows, and freeing one block of a bound pair."""
    import nibble_b200 as nb
    H, KV = 8, 2
    kvw = KV * D
    rng = np.random.default_rng(5)
    ctx = nb.Context(0)
    ctx.set_paged_kv(True)
    ctx.reserve(64, H, 16, H * D)
    k, v = ctx.alloc(64 * kvw), ctx.alloc(64 * kvw)
    q, out = ctx.alloc(16 * H * D), ctx.alloc(16 * H * D)
    kh = rng.standard_normal((64, KV, D)).astype(np.float32)
    vh = rng.standard_normal((64, KV, D)).astype(np.float32)
    qh = rng.standard_normal((16, H, D)).astype(np.float32)
    ctx.write(k, kh, 64 * kvw)
    ctx.write(v, vh, 64 * kvw)
    ctx.write(q, qh, 16 * H * D)
    ctx.attention(q, k, v, out, 12, 0, H, KV, D)  # binds the pair: pages from here on
    kr = np.empty(64 * kvw, np.float32)
    ctx.read(kr, k, 64 * kvw)  # back to flat rows: the values rounded to fp16
    assert np.array_equal(kr.view(np.uint32), oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(kh.ravel())).view(np.uint32))
    # a copy into rows 12..15 of k from rows 0..3 of v, then attention over 16 rows
    ctx.copy(k + 12 * kvw * 4, v, 4 * kvw)
    kh2 = oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(kh)).copy()
    kh2[12:16] = oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(vh[0:4]))
    vh16 = oracle.fp16_bits_to_f32(oracle.f32_to_fp16_bits(vh))
    ctx.attention(q, k, v, out, 1, 15, H, KV, D)
    got = np.empty(H * D, np.float32)
    ctx.read(got, out, H * D)
    ref = oracle.attention(qh[:1], kh2[:16], vh16[:16], 1, 15, H, KV, D)[0]
    assert max_rel_err_per_head(got.reshape(H, D), ref) <= 1e-4
    # freeing k leaves v as flat rows with its (fp16-rounded) values
    ctx.free(k)
    vr = np.empty(64 * kvw, np.float32)
    ctx.read(vr, v, 64 * kvw)
    assert np.array_equal(vr.view(np.uint32), vh16.ravel().view(np.uint32))
    ctx.check()
    ctx.close()


def test_route_off_and_other_head_dims_use_the_flat_kernels():
    """head_dim 32 stays on the flat fp32 path with the route on: results equal a route-off context bit for bit."""
    import nibble_b200 as nb
    H, KV, d = 6, 2, 32
    rng = np.random.default_rng(6)
    res = []
    for paged in (False, True):
        ctx = nb.Context(0)
        ctx.set_paged_kv(paged)
        ctx.reserve(40, H, 8, H * d)
        k, v, q, out = (ctx.alloc(40 * KV * d), ctx.alloc(40 * KV * d), ctx.alloc(8 * H * d), ctx.alloc(8 * H * d))
        r2 = np.random.default_rng(6)
        ctx.write(k, r2.standard_normal(40 * KV * d).astype(np.float32), 40 * KV * d)
        ctx.write(v, r2.standard_normal(40 * KV * d).astype(np.float32), 40 * KV * d)
        ctx.write(q, r2.standard_normal(8 * H * d).astype(np.float32), 8 * H * d)
        ctx.rope(q, 8, H, d, 30, nb.RopeSpec(1e4, False))
        ctx.attention(q, k, v, out, 8, 30, H, KV, d)
        o = np.empty(8 * H * d, np.float32)
        ctx.read(o, out, 8 * H * d)
        res.append(o)
        ctx.close()
    del rng
    assert np.array_equal(res[0].view(np.uint32), res[1].view(np.uint32))
