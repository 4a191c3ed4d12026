"""Host side of the multi-GPU paths: which output rows a rank owns in the vocab-sharded full head,
the communicator-id exchange over torch.distributed, and the data-parallel split of sequences."""
from __future__ import annotations


def row_range(vocab: int, nranks: int, rank: int) -> tuple[int, int]:
    """[first, first + count) of the output matrix owned by `rank` (contiguous, ceil(vocab / nranks))."""
    if not 0 <= rank < nranks:
        raise ValueError("rank out of range")
    per = -(-vocab // nranks)
    first = min(vocab, rank * per)
    return first, min(per, vocab - first)


def seq_range(nseq: int, nranks: int, rank: int) -> tuple[int, int]:
    """[first, first + count) of the sequences a rank scores in data-parallel batched scoring."""
    if not 0 <= rank < nranks:
        raise ValueError("rank out of range")
    base, extra = divmod(nseq, nranks)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def exchange_id(uid: bytes | None, src: int = 0, group=None) -> bytes:
    """Broadcasts a communicator id from rank `src` (which passes it) to every rank of `group`."""
    import torch
    import torch.distributed as dist
    from . import NCCL_UNIQUE_ID_BYTES
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.zeros(NCCL_UNIQUE_ID_BYTES, dtype=torch.uint8, device=dev)
    if dist.get_rank(group) == src:
        if uid is None or len(uid) != NCCL_UNIQUE_ID_BYTES:
            raise ValueError("the source rank must pass a 128-byte id")
        t.copy_(torch.frombuffer(bytearray(uid), dtype=torch.uint8))
    dist.broadcast(t, src=src, group=group)
    return bytes(t.cpu().numpy().tobytes())


def init_vocab_shard(model, group=None) -> tuple[int, int]:
    """Shards `model`'s full head over the ranks of `group` (one GPU each); returns this rank's rows."""
    import torch.distributed as dist
    from . import nccl_unique_id
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    uid = exchange_id(nccl_unique_id() if rank == 0 else None, 0, group)
    model.shard(world, rank, uid)
    return row_range(model.vocab, world, rank)
