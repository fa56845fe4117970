"""Sharding of a batch of decode sequences across the GPUs of one box.

Batched serving is data parallel over sequences: each GPU holds whole
sequences (their paged KV for every attention layer and their GDN states) and
decodes them with no inter-GPU traffic.  Sequences are bin-packed by the HBM
bytes one decode step costs them, not by count, because a sequence's attention
cost grows with its context while its GDN cost does not:

    cost(len) = gdn_layers * heads * dk * dv * 4 * 2 + attn_layers * (len + 1) * kv_heads * 264 * 2

(the factor 2: GDN state read + written; INT4 K+V plus fp16 scale/min read,
counted at 2x to weight the attention kernel's lower bandwidth).
The reference serves one sequence on one GPU; this module has no counterpart there.
"""

from __future__ import annotations

import heapq


def sequence_cost(length: int, *, attn_layers: int = 6, gdn_layers: int = 18, kv_heads: int = 2,
                  gdn_heads: int = 16, gdn_dim: int = 128) -> int:
    gdn = gdn_layers * gdn_heads * gdn_dim * gdn_dim * 4 * 2
    attn = attn_layers * (int(length) + 1) * kv_heads * 264 * 2
    return gdn + attn


def shard_by_cost(lengths, world: int, **cost_kw) -> list[list[int]]:
    """Greedy longest-processing-time packing of sequence indices onto ``world`` ranks.

    Deterministic for a given input (ties broken by index), so every rank
    computes the same assignment without communicating.  Each shard is
    returned in ascending index order.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-sequence_cost(lengths[i], **cost_kw), i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + sequence_cost(lengths[i], **cost_kw), r))
    return [sorted(s) for s in shards]


def shard_loads(lengths, shards, **cost_kw) -> list[int]:
    return [sum(sequence_cost(lengths[i], **cost_kw) for i in s) for s in shards]


def longest_first(lengths, shard) -> list[int]:
    """A shard's sequence indices ordered for decoding: longest context first, ties by index.

    The attention launch runs one CTA per (sequence, KV head) in batch order, in many waves at
    serving batch sizes; with the longest sequences first the last wave holds short ones, so
    the launch does not wait on a long sequence that started late (longest-processing-time
    order).  The GDN step and the output rows do not depend on the order.
    """
    return sorted(shard, key=lambda i: (-int(lengths[i]), i))
