"""Sequence-parallel attention across ranks (one GPU per rank).

Decode, fused (SpDecoder): one launch per rank.  Each rank's decode kernel
reduces its contiguous KV slice; the CTA that finishes each KV head stores
that head's (m, l, O) states into every rank's exchange buffer over NVLink
(CUDA IPC mappings whose handles travel over any host channel) and merges all
ranks' states in rank order, so every rank ends the launch with the result
(sa_sp_* / sa_attn_decode_sp in include/sa_cuda.h).

Decode through a collective library (sp_decode):

The reference splits the KV sequence over MPI ranks and merges the per-rank
online-softmax states on rank 0 (streaming_attention_mpi_simple,
attention/src/streaming_mpi.cpp:252-309: Bcast q, local partial, Gather m, l, O,
sequential merge).  Here the same decomposition runs over torch.distributed:
rank 0's query is broadcast, every rank reduces its contiguous KV slice to
per-head partials (m, l, O) on its GPU, one all-gather moves hq*(d+2) floats
per rank (NCCL over NVLink), and the merge runs on the device.

Causal prefill (sp_prefill): the sequence is cut into 2P equal chunks and
rank r owns chunks r and 2P-1-r ("zig-zag"), so every rank gets the same
amount of causal work (chunk c costs about c + 1/2 chunk-squares, so the two
chunks of every rank add up to 2P).  One all-gather assembles the full K
and V on every rank; each rank then runs the causal prefill of its two query
chunks with their global offsets.  Outputs stay where their queries are: no
merge.  This is the load-balanced causal chunking of configs[2] (the
reference's sequence strategy, ops_mpi.cpp:1000-1212, without its
statistics bug).

``partial_fn`` / ``merge_fn`` / ``prefill_fn`` default to the CUDA library; they
are parameters so the orchestration (collective order, rank-0 semantics,
chunk placement) can be exercised with other implementations.
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


def zigzag_chunks(rank: int, world: int, S: int):
    """(start, stop) of the two query chunks rank `rank` owns: chunks `rank`
    and 2*world-1-rank of 2*world equal chunks (S must divide evenly)."""
    n = 2 * world
    if S % n:
        raise ValueError(f"sp_prefill: S={S} is not a multiple of 2 x world size ({n})")
    C = S // n
    return [(rank * C, (rank + 1) * C), ((n - 1 - rank) * C, (n - rank) * C)]


def zigzag_shard(x, rank: int, world: int):
    """This rank's two zig-zag chunks of a token-major tensor x [S, ...],
    concatenated (the layout sp_prefill expects)."""
    import torch
    (a0, a1), (b0, b1) = zigzag_chunks(rank, world, x.shape[0])
    return torch.cat([x[a0:a1], x[b0:b1]]).contiguous()


def _default_prefill(q, k, v, scale, q_pos0, out):
    import torch
    from .attention import attn_prefill
    return attn_prefill(q, k, v, scale, q_pos0, "float32" if out.dtype == torch.float32 else "bfloat16",
                        None, out)


def sp_prefill(q_local, k_local, v_local, scale: float, group=None, prefill_fn=None, streams=None,
               out_dtype=None):
    """Causal prefill over a sequence sharded zig-zag across the group's ranks.

    q_local [2C, hq, d], k_local / v_local [2C, hkv, d]: this rank's chunks
    r and 2P-1-r of the sequence, concatenated (``zigzag_shard``).  Returns
    out_local [2C, hq, d] for the same query rows, in ``out_dtype`` (default:
    the dtype of q_local).  ``prefill_fn(q, k, v, scale, q_pos0, out)``
    computes causal attention of queries at q_pos0.. against keys
    0..len(k)-1 into ``out``; ``streams`` (two CUDA streams) let the two
    chunks run concurrently.

    One all-gather moves every rank's K and V chunks; the ranks' first chunks
    are chunks 0..P-1 in rank order and their second chunks chunks 2P-1..P,
    so two strided copies put the full K and V in sequence order.
    """
    import torch
    import torch.distributed as dist

    prefill_fn = prefill_fn or _default_prefill
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    C2 = q_local.shape[0]
    if C2 % 2 or k_local.shape[0] != C2 or v_local.shape[0] != C2:
        raise ValueError("sp_prefill: q/k/v_local must hold two equal chunks of the same tokens")
    C = C2 // 2
    S = C2 * world
    PC = world * C
    (a0, a1), (b0, b1) = zigzag_chunks(rank, world, S)
    # one all-gather of K and V together: [world, 2 (k, v), 2C, hkv, d]
    kv = torch.stack([k_local, v_local]).contiguous()
    flat = torch.empty((world * kv.shape[0],) + tuple(kv.shape[1:]), dtype=kv.dtype, device=kv.device)
    dist.all_gather_into_tensor(flat, kv, group=group)
    flat = flat.view((world,) + tuple(kv.shape))
    kv_full = torch.empty((2, S) + tuple(kv.shape[2:]), dtype=kv.dtype, device=kv.device)
    rest = tuple(kv.shape[2:])
    # [2, S, ...] viewed as [2, 2 halves, world, C, ...]; sequence chunk c < P is
    # rank c's first chunk, chunk P + i is rank P-1-i's second chunk
    dst = kv_full.view((2, 2, world, C) + rest)
    dst[:, 0].copy_(flat[:, :, :C].transpose(0, 1))
    dst[:, 1].copy_(flat.flip(0)[:, :, C:].transpose(0, 1))
    k_full, v_full = kv_full[0], kv_full[1]
    out = torch.empty((C2,) + tuple(q_local.shape[1:]), dtype=out_dtype or q_local.dtype, device=q_local.device)
    jobs = [(q_local[:C], a0, a1, out[:C]), (q_local[C:], b0, b1, out[C:])]
    if streams is None:
        for qc, q0, q1, oc in jobs:
            prefill_fn(qc, k_full[:q1], v_full[:q1], scale, q0, oc)
    else:
        cur = torch.cuda.current_stream()
        for st, (qc, q0, q1, oc) in zip(streams, jobs):
            st.wait_stream(cur)
            with torch.cuda.stream(st):
                prefill_fn(qc, k_full[:q1], v_full[:q1], scale, q0, oc)
        for st in streams:
            cur.wait_stream(st)
    return out


class SpDecoder:
    """This rank's share of the fused sequence-parallel decode.

    Every rank creates one with the same ``world``, exchanges handles
    (``connect_dist`` over torch.distributed, ``connect`` with handles from any
    other channel, or ``connect_local`` for several GPUs of one process), then
    calls ``decode`` with its own KV slice (rank order = sequence order) and
    the same q; the merged attention over the whole sequence comes back on
    every rank.  Ranks must be on distinct GPUs.
    """

    def __init__(self, ctx, rank: int, world: int, max_hq: int = 64, max_d: int = 128):
        import ctypes as C
        from ._capi import check, lib
        self.ctx, self.rank, self.world = ctx, rank, world
        h = C.c_void_p()
        check(lib().sa_sp_create(ctx.h, rank, world, max_hq, max_d, C.byref(h)))
        self.h = h

    def handle(self) -> bytes:
        import ctypes as C
        from ._capi import SA_SP_HANDLE_BYTES, check, lib
        buf = C.create_string_buffer(SA_SP_HANDLE_BYTES)
        check(lib().sa_sp_handle(self.h, buf))
        return buf.raw

    def connect(self, handles) -> None:
        import ctypes as C
        from ._capi import check, lib
        blob = b"".join(handles)
        check(lib().sa_sp_connect(self.h, C.create_string_buffer(blob, len(blob))))

    def connect_dist(self, group=None) -> None:
        import torch.distributed as dist
        hs = [None] * self.world
        dist.all_gather_object(hs, self.handle(), group=group)
        self.connect(hs)

    @staticmethod
    def connect_local(decoders) -> None:
        import ctypes as C
        from ._capi import check, lib
        arr = (C.c_void_p * len(decoders))(*[d.h.value for d in decoders])
        check(lib().sa_sp_connect_local(arr, len(decoders)))

    def decode(self, q, k, v, scale: float = 1.0, block: int = 64, out=None, with_state: bool = False,
               kv_static: bool = False):
        """q [hq, d]; k, v [hkv, T_local, d] (CUDA tensors, fp32 or bf16) ->
        out [hq, d] fp32 (and the merged m, l [hq] with ``with_state``).
        ``kv_static``: SA_KV_STATIC (K/V not written by a running kernel)."""
        import ctypes as C
        import torch
        from ._capi import SA_BF16, SA_F32, SA_KV_STATIC, check, lib
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        hq, d = q.shape
        hkv, T, _ = k.shape
        dt = SA_F32 if q.dtype == torch.float32 else SA_BF16
        if out is None:
            out = torch.empty(hq, d, dtype=torch.float32, device=q.device)
        m = torch.empty(hq, dtype=torch.float32, device=q.device) if with_state else None
        l = torch.empty(hq, dtype=torch.float32, device=q.device) if with_state else None
        P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
        self.ctx.set_stream(torch.cuda.current_stream(q.device).cuda_stream)
        check(lib().sa_attn_decode_sp(self.h, dt, P(q), P(k), P(v), T * d, T, d, hq, hkv, block, scale,
                                      P(out), P(m), P(l), SA_KV_STATIC if kv_static else 0))
        return (out, m, l) if with_state else out

    def close(self) -> None:
        from ._capi import lib
        if getattr(self, "h", None):
            lib().sa_sp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SpPrefill:
    """This rank's share of the sequence-parallel causal prefill (sa_spp_*).

    The sequence of S tokens is cut into 2P zig-zag chunks (``zigzag_shard``):
    rank r holds chunks r and 2P-1-r.  Every rank creates one with the same
    ``world``, exchanges handles (``connect_dist``, ``connect`` or
    ``connect_local`` for the GPUs of one process), then calls ``prefill``
    with its own chunks; the K/V chunks cross NVLink by direct stores into
    every rank's buffer and each rank gets the causal attention of its own
    query rows over the whole prefix.  Ranks must be on distinct GPUs.
    """

    def __init__(self, ctx, rank: int, world: int, max_seq: int, hkv: int, d: int = 128):
        import ctypes as C
        from ._capi import check, lib
        self.ctx, self.rank, self.world = ctx, rank, world
        h = C.c_void_p()
        check(lib().sa_spp_create(ctx.h, rank, world, max_seq, hkv, d, C.byref(h)))
        self.h = h

    def handle(self) -> bytes:
        import ctypes as C
        from ._capi import SA_SPP_HANDLE_BYTES, check, lib
        buf = C.create_string_buffer(SA_SPP_HANDLE_BYTES)
        check(lib().sa_spp_handle(self.h, buf))
        return buf.raw

    def connect(self, handles) -> None:
        import ctypes as C
        from ._capi import check, lib
        blob = b"".join(handles)
        check(lib().sa_spp_connect(self.h, C.create_string_buffer(blob, len(blob))))

    def connect_dist(self, group=None) -> None:
        import torch.distributed as dist
        hs = [None] * self.world
        dist.all_gather_object(hs, self.handle(), group=group)
        self.connect(hs)

    @staticmethod
    def connect_local(prefills) -> None:
        import ctypes as C
        from ._capi import check, lib
        arr = (C.c_void_p * len(prefills))(*[p.h.value for p in prefills])
        check(lib().sa_spp_connect_local(arr, len(prefills)))

    def prefill(self, q_local, k_local, v_local, scale: float, out=None, out_dtype=None):
        """q_local [2C, hq, 128], k_local / v_local [2C, hkv, 128] bf16 CUDA
        tensors (this rank's chunks r and 2P-1-r, in that order) ->
        out [2C, hq, 128] (bf16 unless ``out_dtype`` is torch.float32)."""
        import ctypes as C
        import torch
        from ._capi import SA_BF16, SA_F32, check, lib
        for name, t in (("q_local", q_local), ("k_local", k_local), ("v_local", v_local)):
            if t.dtype != torch.bfloat16 or not t.is_cuda or t.dim() != 3:
                raise TypeError(f"SpPrefill.prefill: {name} must be a 3-D bfloat16 CUDA tensor")
        q_local, k_local, v_local = q_local.contiguous(), k_local.contiguous(), v_local.contiguous()
        C2, hq, d = q_local.shape
        hkv = k_local.shape[1]
        if k_local.shape != (C2, hkv, d) or v_local.shape != k_local.shape:
            raise ValueError(f"SpPrefill.prefill: k_local / v_local must be [{C2}, hkv, {d}] like q_local's rows")
        if out is not None and (tuple(out.shape) != (C2, hq, d) or not out.is_contiguous() or
                                out.dtype not in (torch.bfloat16, torch.float32)):
            raise ValueError(f"SpPrefill.prefill: out must be a contiguous [{C2}, {hq}, {d}] bf16 or fp32 tensor")
        if out is None:
            out = torch.empty(C2, hq, d, dtype=out_dtype or torch.bfloat16, device=q_local.device)
        dt = SA_F32 if out.dtype == torch.float32 else SA_BF16
        P = lambda t: C.c_void_p(t.data_ptr())
        self.ctx.set_stream(torch.cuda.current_stream(q_local.device).cuda_stream)
        check(lib().sa_spp_prefill(self.h, P(q_local), P(k_local), P(v_local), C2 * self.world, hq, hkv, d,
                                   scale, P(out), dt, 0))
        return out

    def close(self) -> None:
        from ._capi import lib
        if getattr(self, "h", None):
            lib().sa_spp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
