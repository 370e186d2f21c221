"""How work is split across GPUs (one process per GPU).

* Long-context decode (split-KV): rank g holds the contiguous absolute
  positions [row_offset, row_offset + local_rows) of every layer.  The token at
  `pos` is stored by the rank whose shard holds `pos`; every rank attends its own
  rows and the shard results are combined by log-sum-exp
  (``picoattn_combine_shards``).
* Batched decode: independent sequences are dealt to ranks longest-first onto
  the least-loaded rank (greedy LPT), balancing the cache bytes each rank streams.
* Prefill: KV-head groups are dealt to ranks; each rank runs the q heads of its
  KV heads (no exchange inside attention).

Pure host arithmetic: no device, no collective.
"""
from __future__ import annotations

import heapq

import numpy as np


def shard_rows(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    """(row_offset, local_rows) of `rank` when total_rows are cut into `world` contiguous shards."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(total_rows, world)
    offset = rank * base + min(rank, extra)
    return offset, base + (1 if rank < extra else 0)


def owner_of(pos: int, total_rows: int, world: int) -> int:
    """The rank whose shard holds absolute position pos."""
    for r in range(world):
        off, n = shard_rows(total_rows, world, r)
        if off <= pos < off + n:
            return r
    raise ValueError("position outside the sharded range")


def lpt_assign(lengths, world: int) -> list[list[int]]:
    """Sequence indices per rank: longest first onto the least-loaded rank."""
    order = np.argsort(-np.asarray(lengths), kind="stable")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(int(i))
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(x) for x in out]


def kv_head_groups(n_kv_heads: int, world: int, rank: int) -> list[int]:
    """KV heads of `rank` for head-sharded prefill (round-robin)."""
    return [h for h in range(n_kv_heads) if h % world == rank]


def combine_shards_host(parts: np.ndarray) -> np.ndarray:
    """Host mirror of picoattn_combine_shards for tests.

    parts [n_shards, n_seqs, n_heads, hd+2]: normalised output and, at hd, the
    log2-sum-exp of the shard's scores (-inf for an empty shard)."""
    o = parts[..., :-2].astype(np.float64)
    lse = parts[..., -2].astype(np.float64)
    m = np.max(lse, axis=0)
    w = np.where(np.isneginf(lse), 0.0, np.exp2(lse - m))
    return (np.sum(w[..., None] * o, axis=0) / np.sum(w, axis=0)[..., None]).astype(np.float32)
