"""Host-side partitioning of the MLA decode work across GPUs (one process per
GPU).  The reference runtime is single-process (src/generate.c); these are the
B200 build's multi-GPU layouts:

  * batched decode shards independent sequences: no data-path collective;
    ragged lengths are balanced by longest-processing-time-first on sum(L);
  * one long sequence is split into contiguous KV ranges, one per GPU; each GPU
    produces a normalised partial (o [16][512], lse [16]) that an all-gather
    plus the merge kernel (kvl_mla_merge_partials) combine:
        M = max_g lse_g,  o = sum_g e^(lse_g - M) o_g / sum_g e^(lse_g - M);
  * one prompt's causal prefill is context-parallel: 2 * world chunks of query
    rows, rank r owning chunks r and 2 * world - 1 - r (zigzag: every rank gets
    one early and one late chunk, so the causal work is even), with one
    all-gather of the tokens' compressed 576-wide rows between the projection
    of each rank's rows and the attention (kvl_mla_prefill_cp_begin / _end).
"""
from __future__ import annotations

import heapq

import numpy as np


def shard_sequences(lengths, world: int) -> list[list[int]]:
    """Indices of the sequences each rank owns (LPT greedy on cached length).
    Deterministic: ties go to the lower rank / lower sequence index."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(v) for v in out]


def split_kv(length: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) KV row ranges, one per rank (last ranks may be shorter)."""
    per = (length + world - 1) // world
    return [(min(length, r * per), min(length, (r + 1) * per)) for r in range(world)]


def merge_partials(o: np.ndarray, lse: np.ndarray):
    """Reference combine of partials: o [P][NH][R], lse [P][NH] (natural log)
    -> (o [NH][R], lse [NH]).  Empty parts carry lse = -inf."""
    m = np.max(lse, axis=0)
    w = np.exp(lse - m[None, :])
    s = np.sum(w, axis=0)
    out = np.einsum("ph,phr->hr", w, o) / s[:, None]
    return out.astype(np.float32), (m + np.log(s)).astype(np.float32)


def zigzag_chunks(seq_len: int, world: int) -> list[tuple[tuple[int, int], tuple[int, int]]]:
    """Per rank, the [lo, hi) query rows of its early and late chunk in the
    context-parallel prefill (the split kvl_mla_prefill_cp_begin uses)."""
    if world <= 0 or seq_len % (2 * world):
        raise ValueError(f"{seq_len} rows do not split into {2 * world} chunks")
    c = seq_len // (2 * world)
    return [((r * c, (r + 1) * c), ((2 * world - 1 - r) * c, (2 * world - r) * c)) for r in range(world)]


def rank_rows(seq_len: int, world: int, rank: int) -> np.ndarray:
    """Prompt rows a rank holds, in the order of its compact buffers (the d_x
    and d_out of kvl_mla_prefill_cp_begin / _end): its early chunk, then its
    late chunk."""
    (a0, a1), (b0, b1) = zigzag_chunks(seq_len, world)[rank]
    return np.concatenate([np.arange(a0, a1), np.arange(b0, b1)])


def gathered_row_order(seq_len: int, world: int) -> np.ndarray:
    """Prompt row held at each row of the all-gathered buffer [world][2c]: rank
    order, each rank's early chunk then its late chunk."""
    return np.concatenate([rank_rows(seq_len, world, r) for r in range(world)])
