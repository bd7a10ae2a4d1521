"""nibble_b200: a B200 (sm_100a) attention backend for nibble, behind a C ABI (include/nibble_cuda.h).

The product is ``libnibble_cuda.so``: hand-written CUDA kernels for grouped-query attention (tcgen05/TMEM prefill,
split-K flash-decode over a paged fp16 K/V pool, fused bias+RoPE+append, LSE merge) and the drop-in fp32
operations of nibble's ``Backend`` interface. This package is the Python view of that ABI, used by the tests, the
benchmark and multi-GPU drivers; ``csrc/host/cuda_backend.h`` is the C++ view, mirroring ``nibble::Backend``.

Tensors passed here are torch CUDA tensors (torch is only the device-memory and stream plumbing); every compute
call goes through the C ABI. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _abi
from ._abi import BF16, F16, F32, Q4_0, Q4_K, Q5_0, Q5_1, Q5_K, Q6_K, Q8_0, NibbleError, check

__all__ = ["Context", "KVPool", "Weight", "NibbleError", "RopeSpec", "F32", "F16", "BF16", "Q4_0", "Q5_0", "Q8_0", "Q5_1",
           "Q4_K", "Q5_K", "Q6_K",
           "abi_version"]


def abi_version() -> int:
    return _abi.lib.nbl_abi_version()


@dataclass(frozen=True)
class RopeSpec:
    """nibble's RopeParams (src/backend/backend.h:16-20): base, NeoX pairing, optional per-pair factors."""
    freq_base: float
    neox: bool
    freq_factors: tuple | None = None

    def _c(self):
        ff = None
        ptr = None
        if self.freq_factors is not None:
            ff = (C.c_float * len(self.freq_factors))(*self.freq_factors)
            ptr = C.cast(ff, C.c_void_p)
        return _abi.RopeParams(self.freq_base, int(self.neox), ptr), ff


_DT = {"float32": F32, "float16": F16, "bfloat16": BF16}


def torch_float32():
    import torch
    return torch.float32


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def _dtype(t) -> int:
    name = str(t.dtype).replace("torch.", "")
    if name not in _DT:
        raise ValueError(f"unsupported dtype {t.dtype}")
    return _DT[name]


class KVPool:
    """A paged K/V pool: pool[page][2][n_kv_heads][page_size][head_dim] (fp16 or bf16)."""

    def __init__(self, ctx: "Context", n_pages: int, n_kv_heads: int, head_dim: int = 64, page_size: int = 16,
                 dtype: int = F16):
        self.ctx = ctx
        cfg = _abi.KvConfig(n_pages, n_kv_heads, head_dim, page_size, dtype)
        h = C.c_void_p()
        check(_abi.lib.nbl_kv_create(ctx.handle, C.byref(cfg), C.byref(h)))
        self.handle = h
        self.n_pages, self.n_kv_heads, self.head_dim, self.page_size, self.dtype = (n_pages, n_kv_heads, head_dim,
                                                                                    page_size, dtype)
        base, nbytes = C.c_void_p(), C.c_int64()
        check(_abi.lib.nbl_kv_pool(h, C.byref(base), C.byref(nbytes)))
        self.base, self.nbytes = base.value, nbytes.value

    def tensor(self):
        """The pool's raw 16-bit elements as a torch int16 view [n_pages, 2, n_kv_heads, page_size, head_dim]
        (aliases the pool; no copy). Reinterpret with .view(torch.float16 / torch.bfloat16)."""
        import torch
        t = _wrap_device_memory(self.base, self.nbytes // 2, torch.int16, self.ctx.device)
        return t.view(self.n_pages, 2, self.n_kv_heads, self.page_size, self.head_dim)

    def close(self):
        if self.handle:
            check(_abi.lib.nbl_kv_destroy(self.handle))
            self.handle = None


class Weight:
    """A weight tensor uploaded to the device (nbl_weight): ne1 rows of ne0 elements, F32 or F16 -- the device form
    of nibble's Tensor view (src/tensor.h:57-70)."""

    def __init__(self, ctx: "Context", host, dtype: int | None = None, ne0: int | None = None):
        """host: a C-contiguous numpy float32 / float16 array, 1-D (a vector) or 2-D [ne1, ne0]; or, with dtype
        a quantized type (Q4_0 / Q5_0 / Q8_0 / Q5_1 / Q4_K / Q5_K / Q6_K) and ne0 given, the GGUF block bytes as
        uint8 [ne1, row bytes]."""
        import numpy as np
        a = np.ascontiguousarray(host)
        if dtype is None:
            dtype = {np.dtype(np.float32): F32, np.dtype(np.float16): F16}.get(a.dtype)
            if dtype is None:
                raise ValueError(f"weights must be float32 or float16, got {a.dtype}")
        if dtype in (Q4_0, Q5_0, Q8_0, Q5_1, Q4_K, Q5_K, Q6_K):
            if ne0 is None or a.ndim != 2:
                raise ValueError("quantized weights take uint8 blocks [ne1, row bytes] and ne0")
            ne1 = a.shape[0]
        else:
            ne1, ne0 = (1, a.shape[0]) if a.ndim == 1 else a.shape
        h = C.c_void_p()
        check(_abi.lib.nbl_weight_create(ctx.handle, a.ctypes.data, dtype, ne0, ne1, C.byref(h)))
        self.ctx, self.handle, self.ne0, self.ne1, self.dtype = ctx, h, ne0, ne1, dtype

    def close(self):
        if self.handle:
            check(_abi.lib.nbl_weight_destroy(self.handle))
            self.handle = None


def _wrap_device_memory(ptr: int, numel: int, dtype, device: int):
    """A torch tensor aliasing `numel` elements of device memory at `ptr` (owned elsewhere)."""
    import torch

    class _Holder:
        def __init__(self):
            elsize = torch.empty((), dtype=dtype).element_size()
            self.__cuda_array_interface__ = {
                "shape": (numel,), "typestr": {torch.int16: "<i2", torch.float32: "<f4"}[dtype],
                "data": (ptr, False), "version": 3, "strides": (elsize,)}

    with torch.cuda.device(device):
        return torch.as_tensor(_Holder(), device=f"cuda:{device}")


class Context:
    """An nbl_ctx on one device. By default its kernels run on torch's current stream for that device, so they
    order correctly with the torch ops that prepare inputs."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        h = C.c_void_p()
        check(_abi.lib.nbl_ctx_create(device, C.byref(h)))
        self.handle = h
        self.device = device
        if use_torch_stream:
            import torch
            self.set_stream(torch.cuda.current_stream(device).cuda_stream)

    # ---- context
    def set_stream(self, stream: int | None):
        """Runs later kernels on this cudaStream_t (0 / None = CUDA's default stream)."""
        check(_abi.lib.nbl_ctx_set_stream(self.handle, stream))

    def set_paged_kv(self, on: bool = True):
        """Backend-level K/V blocks as fp16 pages with the fused append and the paged kernels (nbl_ctx_set_paged_kv);
        call before reserve() and before allocating the blocks."""
        check(_abi.lib.nbl_ctx_set_paged_kv(self.handle, 1 if on else 0))

    def sync(self):
        check(_abi.lib.nbl_ctx_sync(self.handle))

    def check(self):
        """Raises NibbleError(NBL_E_DEVICE) if a kernel flagged an out-of-range device-side index."""
        check(_abi.lib.nbl_ctx_check(self.handle))

    def close(self):
        if self.handle:
            check(_abi.lib.nbl_ctx_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- Backend memory (backend.h:45-53)
    def reserve(self, n_ctx: int, n_heads: int, max_rows: int = 1, max_width: int = 0):
        check(_abi.lib.nbl_reserve(self.handle, n_ctx, n_heads, max_rows, max_width))

    def alloc(self, n_floats: int) -> int:
        p = C.c_void_p()
        check(_abi.lib.nbl_alloc(self.handle, n_floats, C.byref(p)))
        return p.value

    def free(self, p: int | None):
        check(_abi.lib.nbl_free(self.handle, p))

    def read(self, host_dst, src: int, n: int):
        """Backend::read into a float32 numpy array (or anything exposing a ctypes data pointer)."""
        check(_abi.lib.nbl_read(self.handle, host_dst.ctypes.data, src, n))

    def write(self, dst: int, host_src, n: int):
        check(_abi.lib.nbl_write(self.handle, dst, host_src.ctypes.data, n))

    # ---- Backend ops on fp32 device buffers (pointers or CUDA tensors)
    def add_bias(self, x, bias, width: int, n: int):
        check(_abi.lib.nbl_add_bias(self.handle, _ptr(x), _ptr(bias), width, n))

    def rope(self, x, n: int, n_heads: int, head_dim: int, pos0: int, rope: RopeSpec):
        p, keep = rope._c()
        check(_abi.lib.nbl_rope(self.handle, _ptr(x), n, n_heads, head_dim, pos0, C.byref(p)))

    def attention(self, q, k, v, out, n: int, pos0: int, n_heads: int, n_kv_heads: int, head_dim: int):
        check(_abi.lib.nbl_attention(self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(out), n, pos0, n_heads, n_kv_heads,
                                     head_dim))

    # ---- the model's other Backend ops (backend.h:54-70) on fp32 device buffers
    def weight(self, host, dtype: int | None = None, ne0: int | None = None) -> Weight:
        return Weight(self, host, dtype, ne0)

    def embed(self, table: Weight, ids, out):
        """ids: host int32 array (a std::span in the reference); out [n, ne0] fp32."""
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        check(_abi.lib.nbl_embed(self.handle, table.handle, ids.ctypes.data, ids.shape[0], _ptr(out)))

    def matmul(self, w: Weight, x, y, n: int):
        """y[n, ne1] = x[n, ne0] . W^T"""
        check(_abi.lib.nbl_matmul(self.handle, w.handle, _ptr(x), _ptr(y), n))

    def matmul_multi(self, ws, x, ys, n: int):
        """ys[i][n, ws[i].ne1] = x[n, ne0] . ws[i]^T for weights sharing one input (one launch for n <= 8)."""
        count = len(ws)
        warr = (C.c_void_p * count)(*[w.handle.value for w in ws])
        yarr = (C.c_void_p * count)(*[_ptr(y) for y in ys])
        check(_abi.lib.nbl_matmul_multi(self.handle, warr, count, _ptr(x), yarr, n))

    def rmsnorm(self, x, weight: Weight, y, n: int, eps: float):
        check(_abi.lib.nbl_rmsnorm(self.handle, _ptr(x), weight.handle, _ptr(y), n, eps))

    def add(self, x, y, count: int):
        check(_abi.lib.nbl_add(self.handle, _ptr(x), _ptr(y), count))

    def copy(self, dst, src, count: int):
        check(_abi.lib.nbl_copy(self.handle, _ptr(dst), _ptr(src), count))

    def silu_mul(self, gate, up, count: int):
        check(_abi.lib.nbl_silu_mul(self.handle, _ptr(gate), _ptr(up), count))

    # ---- paged path
    def kv_pool(self, n_pages: int, n_kv_heads: int, head_dim: int = 64, page_size: int = 16,
                dtype: int = F16) -> KVPool:
        return KVPool(self, n_pages, n_kv_heads, head_dim, page_size, dtype)

    def rope_kv_append(self, kv: KVPool, q_in, k_in, v_in, q_out, tok_row, tok_pos, page_table, n_heads: int,
                       rope: RopeSpec, bq=None, bk=None, bv=None):
        """Fused bias -> RoPE -> narrowing -> page write for q_in.shape[0] tokens (see nbl_rope_kv_append)."""
        p, keep = rope._c()
        in_dt = _dtype(q_in)
        if _dtype(k_in) != in_dt or _dtype(v_in) != in_dt:
            raise ValueError("q_in, k_in, v_in must share a dtype")
        check(_abi.lib.nbl_rope_kv_append(
            self.handle, kv.handle, _ptr(q_in), _ptr(k_in), _ptr(v_in), in_dt, _ptr(bq), _ptr(bk), _ptr(bv),
            _ptr(q_out), _dtype(q_out), _ptr(tok_row), _ptr(tok_pos), _ptr(page_table), page_table.shape[-1],
            q_in.shape[0], n_heads, C.byref(p)))

    def attn_decode(self, kv: KVPool, q, page_table, seq_lens, max_seq_len: int, out, lse=None, n_splits: int = 0):
        """One query token per row: q/out [rows, n_heads, head_dim] fp32, page_table [rows, stride] int32."""
        check(_abi.lib.nbl_attn_decode(self.handle, kv.handle, _ptr(q), _ptr(page_table), page_table.shape[-1],
                                       _ptr(seq_lens), max_seq_len, q.shape[0], q.shape[1], _ptr(out), _ptr(lse),
                                       n_splits))

    def decode_step_host(self, kv: KVPool, q_in_h, k_in_h, v_in_h, page_table, seq_lens, max_seq_len: int,
                         rope: RopeSpec, out_h, bq=None, bk=None, bv=None, n_chunks: int = 0):
        """One decode step from host memory (see nbl_decode_step_host): q_in_h [rows, H, D], k_in_h/v_in_h
        [rows, KVH, D] and out_h [rows, H, D] are fp32 host tensors (pinned for overlapped copies); page_table
        and seq_lens (counting the new token) are device tensors."""
        for t in (q_in_h, k_in_h, v_in_h, out_h):
            if t.is_cuda or not t.is_contiguous() or t.dtype != torch_float32():
                raise ValueError("host tensors must be contiguous float32 CPU tensors")
        p, keep = rope._c()
        check(_abi.lib.nbl_decode_step_host(
            self.handle, kv.handle, q_in_h.data_ptr(), k_in_h.data_ptr(), v_in_h.data_ptr(), _ptr(bq), _ptr(bk),
            _ptr(bv), _ptr(page_table), page_table.shape[-1], _ptr(seq_lens), max_seq_len, q_in_h.shape[0],
            q_in_h.shape[1], C.byref(p), out_h.data_ptr(), n_chunks))

    def attn_prefill(self, kv: KVPool, q, q_start, q_len, kv_pos0, page_table, max_q_len: int, out):
        """Causal prefill: q [rows, n_heads, head_dim] (pool dtype), out [rows, n_heads, head_dim] fp32/pool dtype."""
        check(_abi.lib.nbl_attn_prefill(self.handle, kv.handle, _ptr(q), _dtype(q), q.shape[0], _ptr(q_start),
                                        _ptr(q_len), _ptr(kv_pos0), _ptr(page_table), page_table.shape[-1],
                                        q_start.shape[0], q.shape[1], max_q_len, _ptr(out), _dtype(out)))

    def lse_merge_packed(self, packed, n_parts: int, rows: int, head_dim: int, out, lse=None):
        """packed [n_parts, rows * (head_dim + 1)] fp32 (per part: outputs then lse) -> out [rows, head_dim]."""
        check(_abi.lib.nbl_lse_merge_packed(self.handle, _ptr(packed), n_parts, rows, head_dim, _ptr(out), _ptr(lse)))

    def lse_merge(self, part_o, part_lse, out, lse=None):
        """part_o [P, rows, D], part_lse [P, rows] fp32 -> out [rows, D] (+ lse [rows])."""
        n_parts, rows, d = part_o.shape
        check(_abi.lib.nbl_lse_merge(self.handle, _ptr(part_o), _ptr(part_lse), n_parts, rows, d, _ptr(out),
                                     _ptr(lse)))
