"""Host-side pieces of the data-parallel training step.

One process per GPU.  The global batch is split into equal contiguous row
shards; every rank starts from the same seeded parameters (the reference's
init is deterministic, src/nn.rs:12-26), computes the mean loss / gradients
of its shard, and the gradients are averaged across ranks (NCCL, on the GPU)
before the SGD update, so the update equals the full-batch one.  The NCCL
unique id, or the peer-sharded exchange's handles, travel over the
torch.distributed process group.
"""
from __future__ import annotations

import hashlib
from typing import Sequence, Tuple

import numpy as np


def shard_rows(n_rows: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of this rank's rows; the global batch must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n_rows % world:
        raise ValueError(f"global batch {n_rows} does not split evenly over {world} ranks")
    per = n_rows // world
    return rank * per, (rank + 1) * per


def exchange_unique_id(dist, rank: int, make_id) -> bytes:
    """Rank 0 creates the communicator id; everyone receives it."""
    box = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def all_gather_bytes(dist, data: bytes, world: int):
    """Every rank's ``data`` in rank order (peer-sharded exchange handles)."""
    out = [None] * world
    dist.all_gather_object(out, bytes(data))
    return out


def params_digest(arrays: Sequence[np.ndarray]) -> str:
    """SHA-256 over the raw bytes of the parameters (cross-rank identity check)."""
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def digests_agree(dist, digest: str, world: int) -> bool:
    """All-gather every rank's digest and compare."""
    out = [None] * world
    dist.all_gather_object(out, digest)
    return all(d == out[0] for d in out)
