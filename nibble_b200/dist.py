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
