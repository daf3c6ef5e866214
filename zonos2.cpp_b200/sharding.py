"""Batch sharding of decode streams over ranks (one process per GPU).

Decode streams are independent: each owns its logits row, history ring,
allow mask and generator, the generator of global stream ``g`` being
``Xoshiro256(seed + g)`` (the reference seeds one generator per call,
src/zonos2_generate.cpp:196; stream ``g`` of a batch takes ``seed + g``).
A rank therefore samples a contiguous slice of the global batch with
``first_stream`` set to the slice's start, and the only exchange of a step is
the all-gather of the int32 codes ``[n_local, n_cb]``.  Nothing else crosses
GPUs, so a rank's codes are bit-identical to the same rows of a one-device
run of the whole batch.

The slices are contiguous and as even as possible: the first
``n_streams % world_size`` ranks own one stream more.  For the gather every
rank pads its slice to the largest slice size, so one fixed-size collective
serves ragged splits too.
"""
from __future__ import annotations


def shard_range(n_streams: int, world_size: int, rank: int) -> tuple[int, int]:
    """(first global stream, number of streams) owned by `rank`."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    if n_streams < 0:
        raise ValueError("n_streams must be non-negative")
    base, extra = divmod(n_streams, world_size)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def max_shard(n_streams: int, world_size: int) -> int:
    return -(-n_streams // world_size) if world_size else 0


def gather_codes(codes_local, n_streams: int, world_size: int, rank: int, group=None,
                 out=None):
    """All-gather each rank's codes ``[count, n_cb]`` into ``[n_streams, n_cb]``
    on every rank.  `codes_local` holds this rank's slice; `out`, when given,
    receives the result.  NCCL groups use one ``all_gather_into_tensor`` of
    padded slices; other backends (gloo) a list all-gather."""
    import torch
    import torch.distributed as dist

    first, count = shard_range(n_streams, world_size, rank)
    if codes_local.shape[0] != count:
        raise ValueError(f"rank {rank} holds {codes_local.shape[0]} streams, owns {count}")
    n_cb = codes_local.shape[1]
    m = max_shard(n_streams, world_size)
    if count == m:
        send = codes_local.contiguous()
    else:
        send = torch.zeros((m, n_cb), dtype=codes_local.dtype, device=codes_local.device)
        send[:count].copy_(codes_local)
    even = n_streams % world_size == 0
    if out is None:
        out = torch.empty((n_streams, n_cb), dtype=send.dtype, device=send.device)
    if world_size == 1:
        padded = send.unsqueeze(0)
    elif dist.get_backend(group) == "nccl" and even and out.is_contiguous():
        dist.all_gather_into_tensor(out, send, group=group)   # straight into place
        return out
    elif dist.get_backend(group) == "nccl":
        padded = torch.empty((world_size, m, n_cb), dtype=send.dtype, device=send.device)
        dist.all_gather_into_tensor(padded, send, group=group)
    else:
        parts = [torch.empty_like(send) for _ in range(world_size)]
        dist.all_gather(parts, send, group=group)
        padded = torch.stack(parts)
    if even:
        out.copy_(padded.reshape(n_streams, n_cb))
    else:
        for r in range(world_size):
            f, c = shard_range(n_streams, world_size, r)
            out[f:f + c].copy_(padded[r, :c])
    return out
