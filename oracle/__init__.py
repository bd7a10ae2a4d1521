"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference leg import this package, and
only as the checker or the timed CPU baseline. The product (``nibble_b200`` and ``libnibble_cuda.so``) never
imports it and has no CPU fallback.

Two libraries are wrapped:

* ``liboracle.so`` -- the plain-C restatement of nibble's scalar attention path (``nbl_oracle.c``; each
  function cites the reference function it restates).
* ``_ref/libnibble_ref.so`` -- nibble's own sources (``src/backend/cpu/ref_ops.cpp``, the AVX2 tiers,
  ``CpuBackend``, ``ThreadPool``) compiled by ``oracle/Makefile`` behind ``ref_shim.cpp``. It exists only where
  the reference tree was available at build time; ``have_ref()`` says whether it loaded.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libnibble_ref.so")
# The nibble source tree the _ref targets compile from: NIBBLE_REFERENCE_TREE, else a checkout named "reference"
# beside this repository. Without one, only liboracle.so is built (the prebuilt _ref files are used as they are).
REF_TREE = os.environ.get("NIBBLE_REFERENCE_TREE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64

_lib = None
_ref = None


MODEL_CHECK = os.path.join(HERE, "_ref", "nbl_model_check")
MODEL_BENCH = os.path.join(HERE, "_ref", "nbl_model_bench")
BATCHED_CHECK = os.path.join(HERE, "_ref", "nbl_batched_check")
BATCHED_BENCH = os.path.join(HERE, "_ref", "nbl_batched_bench")
GOLDEN_CHECK = os.path.join(HERE, "_ref", "nbl_golden_check")


def build(with_ref: bool | None = None) -> None:
    """Compiles liboracle.so, and oracle/_ref when the reference tree is present (or with_ref is True): nibble's own
    code, the golden-vector check of the quantized arithmetic, and -- once nibble_b200/libnibble_cuda.so exists -- the
    Transformer drop-in check and bench binaries and the multi-sequence decoder's check and bench."""
    targets = ["oracle"]
    if with_ref or (with_ref is None and os.path.isdir(os.path.join(REF_TREE, "src"))):
        targets += ["ref", "golden-check"]
        if os.path.exists(os.path.join(os.path.dirname(HERE), "nibble_b200", "libnibble_cuda.so")):
            targets += ["model-check", "model-bench", "batched-check", "batched-bench"]
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REF_TREE}", "-j8", *targets], check=True)


def _load_oracle():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(ORACLE_SO):
        build(with_ref=False)
    lib = C.CDLL(ORACLE_SO)
    lib.orc_fp16_to_fp32.argtypes = [C.c_uint16]
    lib.orc_fp16_to_fp32.restype = C.c_float
    lib.orc_fp32_to_fp16.argtypes = [C.c_float]
    lib.orc_fp32_to_fp16.restype = C.c_uint16
    for name, a, b in (("orc_fp16_to_fp32_n", _u16p, _f32p), ("orc_fp32_to_fp16_n", _f32p, _u16p),
                       ("orc_bf16_to_fp32_n", _u16p, _f32p), ("orc_fp32_to_bf16_n", _f32p, _u16p)):
        getattr(lib, name).argtypes = [a, b, _i64]
        getattr(lib, name).restype = None
    lib.orc_softmax_inplace.argtypes = [_f32p, _i64]
    lib.orc_rope.argtypes = [_f32p, _i64, _i64, _i64, _i64, C.c_float, C.c_int, C.c_void_p]
    lib.orc_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]
    lib.orc_attention.restype = C.c_int
    lib.orc_add_bias.argtypes = [_f32p, _f32p, _i64, _i64]
    lib.orc_gather_pages.argtypes = [_u16p, _i32p, _i64, _i64, _i64, _i64, C.c_int, _f32p, _f32p]
    lib.orc_lse_merge.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p, C.c_void_p]
    lib.orc_embed.argtypes = [C.c_void_p, C.c_int, _i64, _i64, _i32p, _i64, _f32p]
    lib.orc_embed.restype = C.c_int
    lib.orc_matmul.argtypes = [C.c_void_p, C.c_int, _i64, _i64, _f32p, _f32p, _i64]
    lib.orc_rmsnorm.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_float]
    lib.orc_add.argtypes = [_f32p, _f32p, _i64]
    lib.orc_silu_mul.argtypes = [_f32p, _f32p, _i64]
    lib.orc_quantize_q8_0.argtypes = [_f32p, C.c_void_p, _i64]
    lib.orc_quantize_q8_1.argtypes = [_f32p, C.c_void_p, _i64]
    lib.orc_quantize_q8_K.argtypes = [_f32p, C.c_void_p, _i64]
    lib.orc_dequantize_row.argtypes = [C.c_int, C.c_void_p, _f32p, _i64]
    lib.orc_dequantize_row.restype = C.c_int
    lib.orc_matmul_q.argtypes = [C.c_void_p, C.c_int, _i64, _i64, _f32p, _f32p, _i64]
    lib.orc_matmul_q.restype = C.c_int
    lib.orc_vec_dot.argtypes = [C.c_int, C.c_void_p, C.c_void_p, _i64]
    lib.orc_vec_dot.restype = C.c_float
    _lib = lib
    return lib


def have_ref() -> bool:
    """True when oracle/_ref/libnibble_ref.so (nibble's own code) is built and loads."""
    try:
        _load_ref()
        return True
    except OSError:
        return False


def _load_ref():
    global _ref
    if _ref is not None:
        return _ref
    if not os.path.exists(REF_SO) and os.path.isdir(os.path.join(REF_TREE, "src")):
        build(with_ref=True)
    lib = C.CDLL(REF_SO)
    lib.nref_last_error.restype = C.c_char_p
    lib.nref_attention_scalar.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _f32p]
    lib.nref_rope.argtypes = [_f32p, _i64, _i64, _i64, _i64, C.c_float, C.c_int, C.c_void_p]
    lib.nref_softmax.argtypes = [_f32p, _i64]
    lib.nref_fp16_to_fp32.argtypes = [C.c_uint16]
    lib.nref_fp16_to_fp32.restype = C.c_float
    lib.nref_fp32_to_fp16.argtypes = [C.c_float]
    lib.nref_fp32_to_fp16.restype = C.c_uint16
    lib.nref_fp16_to_fp32_n.argtypes = [_u16p, _f32p, _i64]
    lib.nref_fp32_to_fp16_n.argtypes = [_f32p, _u16p, _i64]
    lib.nref_kernels_name.restype = C.c_char_p
    lib.nref_backend_create.argtypes = [C.c_int]
    lib.nref_backend_create.restype = C.c_void_p
    lib.nref_backend_destroy.argtypes = [C.c_void_p]
    lib.nref_backend_threads.argtypes = [C.c_void_p]
    lib.nref_backend_reserve.argtypes = [C.c_void_p, _i64, _i64, _i64, _i64]
    lib.nref_backend_attention.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           _i64, _i64, _i64, _i64, _i64]
    lib.nref_backend_rope.argtypes = [C.c_void_p, _f32p, _i64, _i64, _i64, _i64, C.c_float, C.c_int, C.c_void_p]
    lib.nref_embed.argtypes = [C.c_void_p, C.c_int, _i64, _i64, _i32p, _i64, _f32p]
    lib.nref_matmul.argtypes = [C.c_void_p, C.c_int, _i64, _i64, _f32p, _f32p, _i64]
    lib.nref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_float]
    lib.nref_add.argtypes = [_f32p, _f32p, _i64]
    lib.nref_silu_mul.argtypes = [_f32p, _f32p, _i64]
    lib.nref_backend_matmul.argtypes = [C.c_void_p, C.c_void_p, C.c_int, _i64, _i64, _f32p, _f32p, _i64]
    lib.nref_backend_rmsnorm.argtypes = [C.c_void_p, _f32p, _f32p, _f32p, _i64, _i64, C.c_float]
    lib.nref_backend_silu_mul.argtypes = [C.c_void_p, _f32p, _f32p, _i64]
    lib.nref_quantize_q8_0.argtypes = [_f32p, C.c_void_p, _i64]
    lib.nref_quantize_q8_1.argtypes = [_f32p, C.c_void_p, _i64]
    lib.nref_quantize_q8_K.argtypes = [_f32p, C.c_void_p, _i64]
    lib.nref_dequantize_row.argtypes = [C.c_int, C.c_void_p, _f32p, _i64]
    lib.nref_matmul_q.argtypes = [C.c_void_p, C.c_int, _i64, _i64, _f32p, _f32p, _i64]
    _ref = lib
    return lib


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- the C restatement
def fp16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    b = _c(bits, np.uint16).ravel()
    out = np.empty(b.size, np.float32)
    _load_oracle().orc_fp16_to_fp32_n(b, out, b.size)
    return out.reshape(np.shape(bits))


def f32_to_fp16_bits(x: np.ndarray) -> np.ndarray:
    a = _c(x).ravel()
    out = np.empty(a.size, np.uint16)
    _load_oracle().orc_fp32_to_fp16_n(a, out, a.size)
    return out.reshape(np.shape(x))


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    b = _c(bits, np.uint16).ravel()
    out = np.empty(b.size, np.float32)
    _load_oracle().orc_bf16_to_fp32_n(b, out, b.size)
    return out.reshape(np.shape(bits))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    a = _c(x).ravel()
    out = np.empty(a.size, np.uint16)
    _load_oracle().orc_fp32_to_bf16_n(a, out, a.size)
    return out.reshape(np.shape(x))


def softmax(x: np.ndarray) -> np.ndarray:
    y = _c(x).copy()
    _load_oracle().orc_softmax_inplace(y, y.size)
    return y


def _ff(freq_factors):
    if freq_factors is None:
        return None, None
    ff = _c(freq_factors)
    return ff, ff.ctypes.data_as(C.c_void_p)


def rope(x: np.ndarray, n_heads: int, head_dim: int, pos0: int, freq_base: float, neox: bool,
         freq_factors=None) -> np.ndarray:
    """Returns a roped copy of x viewed as [n, n_heads, head_dim] (nbl_oracle.c orc_rope)."""
    y = _c(x).copy()
    n = y.size // (n_heads * head_dim)
    ff, ffp = _ff(freq_factors)
    _load_oracle().orc_rope(y, n, n_heads, head_dim, pos0, freq_base, int(neox), ffp)
    return y


def attention(q, k, v, n, pos0, n_heads, n_kv_heads, head_dim) -> np.ndarray:
    """Scalar causal GQA attention (nbl_oracle.c orc_attention); returns out [n, n_heads, head_dim]."""
    q, k, v = _c(q), _c(k), _c(v)
    out = np.empty((n, n_heads, head_dim), np.float32)
    if _load_oracle().orc_attention(q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim) != 0:
        raise MemoryError("oracle attention scratch")
    return out


def add_bias(x, bias, n) -> np.ndarray:
    y = _c(x).copy()
    b = _c(bias)
    _load_oracle().orc_add_bias(y, b, b.size, n)
    return y


def gather_pages(pool_bits, page_table, length, n_kv_heads, head_dim, page_size, bf16=False):
    """Widens one sequence's paged K/V (uint16 bits) into contiguous fp32 [length, n_kv_heads, head_dim]."""
    k = np.empty((length, n_kv_heads, head_dim), np.float32)
    v = np.empty_like(k)
    _load_oracle().orc_gather_pages(_c(pool_bits, np.uint16).ravel(), _c(page_table, np.int32), length, n_kv_heads,
                                    head_dim, page_size, int(bf16), k, v)
    return k, v


def lse_merge(part_o, part_lse):
    """part_o [P, rows, D], part_lse [P, rows] -> (out [rows, D], lse [rows])."""
    part_o, part_lse = _c(part_o), _c(part_lse)
    p, rows, d = part_o.shape
    out = np.empty((rows, d), np.float32)
    lse = np.empty(rows, np.float32)
    _load_oracle().orc_lse_merge(part_o, part_lse, p, rows, d, out, lse.ctypes.data_as(C.c_void_p))
    return out, lse


# ---------------------------------------------------------------- the model's other ops (backend.h:54-70)
def _weight_arg(w):
    """(pointer, dtype code, array kept alive) for an F32 or F16 (float16 or uint16 bits) weight array."""
    w = np.ascontiguousarray(w)
    if w.dtype == np.float32:
        return w.ctypes.data, 0, w
    if w.dtype in (np.float16, np.uint16):
        return w.ctypes.data, 1, w
    raise ValueError(f"weight dtype {w.dtype}")


def embed(table, ids) -> np.ndarray:
    """Rows ids of table [n_rows, ne0] (F32 or F16), widened to fp32 (ref_ops.cpp:80-98)."""
    ptr, dt, keep = _weight_arg(table)
    ids = _c(ids, np.int32)
    out = np.empty((ids.size, keep.shape[-1]), np.float32)
    if _load_oracle().orc_embed(ptr, dt, keep.shape[-1], keep.shape[0], ids, ids.size, out) != 0:
        raise ValueError("embed: token id out of range")
    return out


def matmul(w, x, n) -> np.ndarray:
    """y[n, ne1] = x[n, ne0] . W^T, float accumulation left to right (ref_ops.cpp:109-136)."""
    ptr, dt, keep = _weight_arg(w)
    ne1, ne0 = keep.shape
    y = np.empty((n, ne1), np.float32)
    _load_oracle().orc_matmul(ptr, dt, ne0, ne1, _c(x), y, n)
    return y


def rmsnorm(x, weight, n, eps) -> np.ndarray:
    w = _c(weight)
    y = np.empty((n, w.size), np.float32)
    _load_oracle().orc_rmsnorm(_c(x), w, y, n, w.size, eps)
    return y


def add(x, y) -> np.ndarray:
    z = _c(x).copy()
    _load_oracle().orc_add(z, _c(y), z.size)
    return z


def silu_mul(gate, up) -> np.ndarray:
    g = _c(gate).copy()
    _load_oracle().orc_silu_mul(g, _c(up), g.size)
    return g


# ---------------------------------------------------------------- quantized weights (Q8_0-activation family)
Q4_0, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K = 2, 6, 7, 8, 12, 13, 14  # nibble DType ids (ggml's)
BLOCK_BYTES = {Q4_0: 18, Q5_0: 22, Q5_1: 24, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {Q4_0: 32, Q5_0: 32, Q5_1: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}


def row_bytes(dtype, ne0) -> int:
    return ne0 // BLOCK_ELEMS[dtype] * BLOCK_BYTES[dtype]


def quantize_q8_0(x) -> np.ndarray:
    """fp32 [n] (n % 32 == 0) -> uint8 [n / 32 * 34] Q8_0 blocks (src/quant.cpp:37-51, :250-257)."""
    x = _c(x).ravel()
    out = np.empty(x.size // 32 * 34, np.uint8)
    _load_oracle().orc_quantize_q8_0(x, out.ctypes.data, x.size)
    return out


def quantize_q8_1(x) -> np.ndarray:
    """fp32 [n] (n % 32 == 0) -> uint8 [n / 32 * 36] Q8_1 blocks (src/quant.cpp:260-273)."""
    x = _c(x).ravel()
    out = np.empty(x.size // 32 * 36, np.uint8)
    _load_oracle().orc_quantize_q8_1(x, out.ctypes.data, x.size)
    return out


def quantize_q8_K(x) -> np.ndarray:
    """fp32 [n] (n % 256 == 0) -> uint8 [n / 256 * 292] Q8_K blocks (src/quant.cpp:276-307)."""
    x = _c(x).ravel()
    out = np.empty(x.size // 256 * 292, np.uint8)
    _load_oracle().orc_quantize_q8_K(x, out.ctypes.data, x.size)
    return out


def dequantize_rows(blocks, dtype, ne0, ne1) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((ne1, ne0), np.float32)
    rb = row_bytes(dtype, ne0)
    for r in range(ne1):
        if _load_oracle().orc_dequantize_row(dtype, b.ctypes.data + r * rb, out[r], ne0) != 0:
            raise ValueError("dtype")
    return out


def matmul_q(blocks, dtype, ne0, ne1, x, n) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    y = np.empty((n, ne1), np.float32)
    if _load_oracle().orc_matmul_q(b.ctypes.data, dtype, ne0, ne1, _c(x), y, n) != 0:
        raise ValueError("dtype")
    return y


def vec_dot(dtype, w_row, act_blocks, n_blocks) -> np.float32:
    """One weight row's block dot with activation blocks already quantized (Q8_0 / Q8_1 / Q8_K bytes): nibble's
    dot_*_q8_* (src/quant.cpp:117-146, :310-418)."""
    w = np.ascontiguousarray(w_row, dtype=np.uint8)
    a = np.ascontiguousarray(act_blocks, dtype=np.uint8)
    return np.float32(_load_oracle().orc_vec_dot(dtype, w.ctypes.data, a.ctypes.data, n_blocks))


def random_q_blocks(rng, dtype, ne1, ne0, scale=0.02) -> np.ndarray:
    """Random but well-formed weight blocks: random value bytes (and random packed sub-block scales for the
    k-quants) with fp16 scales of about `scale` (Q5_1's minimum and Q4_K / Q5_K's dmin of about -8 / 4 scales)."""
    nb = ne0 // BLOCK_ELEMS[dtype]
    bb = BLOCK_BYTES[dtype]
    raw = rng.integers(0, 256, size=(ne1 * nb, bb), dtype=np.uint8)

    def put(off, vals):
        h = f32_to_fp16_bits(vals.astype(np.float32))
        raw[:, off] = h & 0xFF
        raw[:, off + 1] = h >> 8

    mag = scale * (0.5 + rng.random(ne1 * nb))
    if dtype in (Q4_K, Q5_K):
        put(0, mag / 32)
        put(2, mag / 16 * rng.random(ne1 * nb))
    elif dtype == Q6_K:
        put(208, mag / 64)
    else:
        put(0, mag)
        if dtype == Q5_1:
            put(2, -8 * mag * rng.random(ne1 * nb))
    return raw.reshape(ne1, nb * bb)


# ---------------------------------------------------------------- nibble's own code (oracle/_ref)
def ref_quantize_q8_0(x) -> np.ndarray:
    x = _c(x).ravel()
    out = np.empty(x.size // 32 * 34, np.uint8)
    _load_ref().nref_quantize_q8_0(x, out.ctypes.data, x.size)
    return out


def ref_quantize_q8_1(x) -> np.ndarray:
    x = _c(x).ravel()
    out = np.empty(x.size // 32 * 36, np.uint8)
    _load_ref().nref_quantize_q8_1(x, out.ctypes.data, x.size)
    return out


def ref_quantize_q8_K(x) -> np.ndarray:
    x = _c(x).ravel()
    out = np.empty(x.size // 256 * 292, np.uint8)
    _load_ref().nref_quantize_q8_K(x, out.ctypes.data, x.size)
    return out


def ref_dequantize_rows(blocks, dtype, ne0, ne1) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((ne1, ne0), np.float32)
    rb = row_bytes(dtype, ne0)
    lib = _load_ref()
    for r in range(ne1):
        if lib.nref_dequantize_row(dtype, b.ctypes.data + r * rb, out[r], ne0) != 0:
            raise ValueError(lib.nref_last_error().decode())
    return out


def ref_matmul_q(blocks, dtype, ne0, ne1, x, n) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    y = np.empty((n, ne1), np.float32)
    lib = _load_ref()
    if lib.nref_matmul_q(b.ctypes.data, dtype, ne0, ne1, _c(x), y, n) != 0:
        raise ValueError(lib.nref_last_error().decode())
    return y



def ref_embed(table, ids) -> np.ndarray:
    """nibble::cpu::embed (src/backend/cpu/ref_ops.cpp:80)."""
    ptr, dt, keep = _weight_arg(table)
    ids = _c(ids, np.int32)
    out = np.empty((ids.size, keep.shape[-1]), np.float32)
    lib = _load_ref()
    if lib.nref_embed(ptr, dt, keep.shape[-1], keep.shape[0], ids, ids.size, out) != 0:
        raise ValueError(lib.nref_last_error().decode())
    return out


def ref_matmul(w, x, n) -> np.ndarray:
    """nibble::cpu::matmul_rows, float weights (src/backend/cpu/ref_ops.cpp:109)."""
    ptr, dt, keep = _weight_arg(w)
    ne1, ne0 = keep.shape
    y = np.empty((n, ne1), np.float32)
    _load_ref().nref_matmul(ptr, dt, ne0, ne1, _c(x), y, n)
    return y


def ref_rmsnorm(x, weight, n, eps) -> np.ndarray:
    w = _c(weight)
    y = np.empty((n, w.size), np.float32)
    _load_ref().nref_rmsnorm(_c(x), w, y, n, w.size, eps)
    return y


def ref_add(x, y) -> np.ndarray:
    z = _c(x).copy()
    _load_ref().nref_add(z, _c(y), z.size)
    return z


def ref_silu_mul(gate, up) -> np.ndarray:
    g = _c(gate).copy()
    _load_ref().nref_silu_mul(g, _c(up), g.size)
    return g



def ref_attention_scalar(q, k, v, n, pos0, n_heads, n_kv_heads, head_dim) -> np.ndarray:
    """nibble::cpu::attention_heads over all heads (src/backend/cpu/ref_ops.cpp:188)."""
    q, k, v = _c(q), _c(k), _c(v)
    out = np.empty((n, n_heads, head_dim), np.float32)
    scratch = np.empty(pos0 + n, np.float32)
    _load_ref().nref_attention_scalar(q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, scratch)
    return out


def ref_rope(x, n_heads, head_dim, pos0, freq_base, neox, freq_factors=None) -> np.ndarray:
    """nibble::cpu::rope (src/backend/cpu/ref_ops.cpp:166)."""
    y = _c(x).copy()
    n = y.size // (n_heads * head_dim)
    ff, ffp = _ff(freq_factors)
    _load_ref().nref_rope(y, n, n_heads, head_dim, pos0, freq_base, int(neox), ffp)
    return y


def ref_softmax(x) -> np.ndarray:
    y = _c(x).copy()
    _load_ref().nref_softmax(y, y.size)
    return y


def ref_fp16_bits_to_f32(bits) -> np.ndarray:
    """nibble::fp16_to_fp32 over an array (src/fp16.h:18)."""
    b = _c(bits, np.uint16).ravel()
    out = np.empty(b.size, np.float32)
    _load_ref().nref_fp16_to_fp32_n(b, out, b.size)
    return out


def ref_f32_to_fp16_bits(x) -> np.ndarray:
    """nibble::fp32_to_fp16 over an array (src/fp16.h:46)."""
    a = _c(x).ravel()
    out = np.empty(a.size, np.uint16)
    _load_ref().nref_fp32_to_fp16_n(a, out, a.size)
    return out


def ref_kernels_name() -> str:
    name = _load_ref().nref_kernels_name()
    if name is None:
        raise RuntimeError(_load_ref().nref_last_error().decode())
    return name.decode()


class RefBackend:
    """nibble's CpuBackend on a ThreadPool of `threads` (the reference's timed AVX2 attention path)."""

    def __init__(self, threads: int):
        self._lib = _load_ref()
        self._h = self._lib.nref_backend_create(threads)
        if not self._h:
            raise RuntimeError(self._lib.nref_last_error().decode())

    @property
    def threads(self) -> int:
        return self._lib.nref_backend_threads(self._h)

    def reserve(self, n_ctx, n_heads, max_rows, max_width):
        if self._lib.nref_backend_reserve(self._h, n_ctx, n_heads, max_rows, max_width):
            raise RuntimeError(self._lib.nref_last_error().decode())

    def attention_into(self, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim):
        """CpuBackend::attention on preallocated float32 C-contiguous arrays (no copies: for timing)."""
        rc = self._lib.nref_backend_attention(self._h, q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data,
                                              n, pos0, n_heads, n_kv_heads, head_dim)
        if rc:
            raise RuntimeError(self._lib.nref_last_error().decode())

    def attention(self, q, k, v, n, pos0, n_heads, n_kv_heads, head_dim):
        q, k, v = _c(q), _c(k), _c(v)
        out = np.empty((n, n_heads, head_dim), np.float32)
        self.attention_into(q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim)
        return out

    def rope(self, x, n_heads, head_dim, pos0, freq_base, neox, freq_factors=None):
        y = _c(x).copy()
        n = y.size // (n_heads * head_dim)
        ff, ffp = _ff(freq_factors)
        if self._lib.nref_backend_rope(self._h, y, n, n_heads, head_dim, pos0, freq_base, int(neox), ffp):
            raise RuntimeError(self._lib.nref_last_error().decode())
        return y

    def matmul(self, blocks, dtype, ne0, ne1, x, n):
        """CpuBackend::matmul (src/backend/cpu/cpu_backend.cpp:134) of a weight given as GGUF bytes [ne1, row]."""
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        y = np.empty((n, ne1), np.float32)
        if self._lib.nref_backend_matmul(self._h, b.ctypes.data, dtype, ne0, ne1, _c(x), y, n):
            raise ValueError(self._lib.nref_last_error().decode())
        return y

    def close(self):
        if self._h:
            self._lib.nref_backend_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
