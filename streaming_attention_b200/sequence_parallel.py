"""Sequence-parallel decode attention across ranks (one GPU per rank).

The reference splits the KV sequence over MPI ranks and merges the per-rank
online-softmax states on rank 0 (streaming_attention_mpi_simple,
attention/src/streaming_mpi.cpp:252-309: Bcast q, local partial, Gather m, l, O,
sequential merge).  Here the same decomposition runs over torch.distributed:
rank 0's query is broadcast, every rank reduces its contiguous KV slice to
per-head partials (m, l, O) on its GPU, one all-gather moves hq*(d+2) floats
per rank (NCCL over NVLink), and the merge runs on the device.

``partial_fn`` / ``merge_fn`` default to the CUDA library; they are
parameters so the orchestration (collective order, rank-0 semantics) can be
exercised with other implementations.
"""
from __future__ import annotations


def _default_partial(q, k, v, scale, block):
    from .attention import attn_decode_partial
    return attn_decode_partial(q, k, v, scale, block)


def _default_merge(m, l, o):
    from .attention import attn_merge
    return attn_merge(m, l, o)


def sp_decode(q, k_local, v_local, scale: float = 1.0, block: int = 64, group=None,
              partial_fn=None, merge_fn=None, all_ranks: bool = False):
    """Decode attention over a KV sequence sharded across the group's ranks.

    q [hq, d] (meaningful on rank 0, as in the reference); k_local, v_local
    [hkv, T_local, d] this rank's contiguous slice (rank order = sequence
    order).  Returns [hq, d] fp32: the result on rank 0 and zeros on the
    others (streaming_mpi.cpp:306-308), or the result on every rank when
    ``all_ranks``.
    """
    import torch
    import torch.distributed as dist

    partial_fn = partial_fn or _default_partial
    merge_fn = merge_fn or _default_merge
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    src = dist.get_global_rank(group, 0) if group is not None else 0
    q = q.contiguous()
    dist.broadcast(q, src=src, group=group)
    hq, d = q.shape
    m, l, o = partial_fn(q, k_local, v_local, scale, block)
    packed = torch.cat([m.reshape(-1).float(), l.reshape(-1).float(), o.reshape(-1).float()])
    flat = torch.empty(world * packed.numel(), dtype=torch.float32, device=packed.device)
    dist.all_gather_into_tensor(flat, packed, group=group)
    gathered = flat.view(world, packed.numel())
    gm = gathered[:, :hq].contiguous()
    gl = gathered[:, hq:2 * hq].contiguous()
    go = gathered[:, 2 * hq:].reshape(world, hq, d).contiguous()
    out = merge_fn(gm, gl, go)
    if rank != 0 and not all_ranks:
        out = torch.zeros_like(out)
    return out
