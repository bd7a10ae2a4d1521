"""Cross-rank exchange for long-context decode split along the KV sequence.

Each rank attends its contiguous chunk of the KV sequence (workloads.kv_split) and holds, per (row, head), the
chunk's normalised output O and its natural-log sum of exponentials lse. One all-gather moves every rank's
packed [O | lse] block to every rank (one call for all rows and layers: the messages are latency-bound, a few
KB per rank); the log-sum-exp merge then gives the exact full-context result. With NCCL this is the only
collective in the package; the sequence-sharded workloads exchange nothing.

The packing and the gather work on any torch.distributed backend: NCCL over NVLink for the GPUs, gloo for the
CPU tests of this protocol.
"""
from __future__ import annotations


def pack_partials(o, lse):
    """o [rows, H, D] float32, lse [rows, H] float32 -> one flat float32 tensor [rows*H*D + rows*H]."""
    import torch
    return torch.cat([o.reshape(-1), lse.reshape(-1)])


def partials_buffer(rows: int, heads: int, head_dim: int, device="cuda"):
    """A send buffer in the packed layout plus views a decode can write into directly: returns (send, o, lse)
    with send [rows*H*D + rows*H] fp32, o = send's first rows*H*D floats as [rows, H, D], lse the rest as
    [rows, H]. After all_gather_partials(send), Context.lse_merge_packed merges the gathered buffer in place."""
    import torch
    n_o = rows * heads * head_dim
    send = torch.empty(n_o + rows * heads, dtype=torch.float32, device=device)
    return send, send[:n_o].view(rows, heads, head_dim), send[n_o:].view(rows, heads)


def unpack_partials(gathered, rows: int, heads: int, head_dim: int):
    """gathered [world, rows*H*D + rows*H] -> part_o [world, rows*H, D], part_lse [world, rows*H]."""
    world = gathered.shape[0]
    n_o = rows * heads * head_dim
    part_o = gathered[:, :n_o].reshape(world, rows * heads, head_dim)
    part_lse = gathered[:, n_o:].reshape(world, rows * heads)
    return part_o.contiguous(), part_lse.contiguous()


def all_gather_partials(packed, group=None):
    """All-gathers each rank's packed partials; returns [world, n]. One collective call."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = torch.empty((world, packed.numel()), dtype=packed.dtype, device=packed.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, packed, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), packed, group=group)
    return out


class PeerExchange:
    """The same exchange without a collective library (nbl_lse_exchange_peers): each rank stores its packed partials
    straight into every other rank's receive buffer over NVLink and raises one flag word per peer; each rank merges
    as soon as all flags show the step. The buffers are symmetric-memory allocations from torch.distributed (the
    same size on every rank, each rank's mapped into every other's address space), used here only for that mapping.
    All ranks must construct it together and call exchange() the same number of times."""

    def __init__(self, ctx, rows: int, head_dim: int, group=None):
        import ctypes as C
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.ctx, self.rows, self.head_dim = ctx, rows, head_dim
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer exchange takes at most 8 ranks")
        group = group if group is not None else dist.group.WORLD
        dev = torch.device("cuda", torch.cuda.current_device())
        part = rows * (head_dim + 1)
        self.recv = symm.empty(2 * self.world * part, dtype=torch.float32, device=dev)
        self.flags = symm.empty(max(self.world, 4), dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.sync = torch.zeros(2, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        hr = symm.rendezvous(self.recv, group)
        hf = symm.rendezvous(self.flags, group)

        def peers(h, t):  # every rank's address of this tensor, mapped in this process
            off = t.data_ptr() - int(h.buffer_ptrs[self.rank])
            if len(h.buffer_ptrs) != self.world or off < 0 or off + t.numel() * t.element_size() > int(h.buffer_size):
                raise RuntimeError("symmetric-memory buffer does not cover the tensor on every rank")
            return (C.c_void_p * self.world)(*[int(p) + off for p in h.buffer_ptrs])

        self._recv_ptrs, self._flag_ptrs = peers(hr, self.recv), peers(hf, self.flags)
        self._handles = (hr, hf)
        dist.barrier(group)

    def exchange(self, send, out, lse=None):
        """send: this rank's packed partials [rows * head_dim + rows] fp32; out [rows, head_dim] (+ lse [rows])."""
        from . import _abi, _ptr
        _abi.check(_abi.lib.nbl_lse_exchange_peers(
            self.ctx.handle, _ptr(send), self.rows, self.head_dim, self.world, self.rank, self._recv_ptrs,
            self._flag_ptrs, _ptr(self.sync), _ptr(out), _ptr(lse)))

    def decode_exchange(self, kv, q, page_table, seq_lens, max_seq_len: int, out, lse=None):
        """The decode of this rank's KV chunk with the exchange fused in (nbl_attn_decode_peers): q [rows, H, 64] fp32
        with rows * H equal to this exchange's rows; out [rows, H, 64] (+ lse [rows, H]) receive the merged result of
        all ranks' chunks. No send buffer: the decode kernel stores each finished row into every rank's buffer."""
        from . import _abi, _ptr
        if q.shape[0] * q.shape[1] != self.rows or self.head_dim != 64:
            raise ValueError("q must hold this exchange's rows of head_dim 64")
        _abi.check(_abi.lib.nbl_attn_decode_peers(
            self.ctx.handle, kv.handle, _ptr(q), _ptr(page_table), page_table.shape[-1], _ptr(seq_lens), max_seq_len,
            q.shape[0], q.shape[1], self.world, self.rank, self._recv_ptrs, self._flag_ptrs, _ptr(self.sync),
            _ptr(out), _ptr(lse)))

    def close(self):
        self._handles = None
        self.recv = self.flags = self.sync = None
