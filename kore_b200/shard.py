"""Host-side plumbing of the multi-GPU paths.

* KV-sequence split (config 4): each rank's context holds the pages
  j = rank (mod n_ranks); ``exchange_handles`` gives every rank the
  exchange-buffer handles of all ranks so that
  ``KoreCuda.decode_sharded_dev`` can push partials over peer memory.
* Sequence sharding (config 5): ``assign_sequences`` places independent
  sequences on ranks, longest first onto the least-loaded rank.
"""
from __future__ import annotations


def exchange_handles(ctx, dist, group=None) -> list[bytes]:
    """All-gathers every rank's peer handle (rank order) and opens the peers."""
    mine = ctx.peer_handle()
    handles: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(handles, mine, group=group)
    ctx.peer_open(handles)
    return handles


def assign_sequences(lengths, n_ranks: int) -> list[list[int]]:
    """Longest-processing-time assignment: sequences sorted by length
    (descending, ties by index) go to the rank with the least cached positions
    so far (ties to the lowest rank). Deterministic, so every rank computes
    the same table without communicating."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be positive")
    load = [0] * n_ranks
    out: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(n_ranks), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += int(lengths[i])
    return out


def local_positions(limit: int, page_tokens: int, rank: int, n_ranks: int) -> int:
    """Cached positions below `limit` held by `rank` under the page split
    (the count the decode kernel and the context compute)."""
    full, rem = divmod(limit, page_tokens)
    full_local = (full - rank + n_ranks - 1) // n_ranks if full > rank else 0
    return full_local * page_tokens + (rem if full % n_ranks == rank else 0)
