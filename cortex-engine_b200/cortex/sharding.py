"""Batch sharding across GPUs (one process per GPU, no data-path collective).

Every window of a batch is independent on the decoder path (the only
batch-invariant work, the latent and behaviour queries, is recomputed by each
replica), so a batch splits into contiguous window ranges, one per rank. Ranges
are balanced by event count, which matters for ragged batches, and each rank
receives only its slice of the flat event arrays with batch indices rebased
to start at 0.
"""

from __future__ import annotations

import numpy as np


def shard_bounds(counts: np.ndarray, world: int) -> list[tuple[int, int]]:
    """Contiguous [b0, b1) window ranges, one per rank, balanced by events.

    Rank r ends its range at the first window boundary whose cumulative event
    count reaches r+1 / world of the total (ties keep every rank non-empty when
    there are at least ``world`` windows).
    """
    counts = np.asarray(counts, dtype=np.int64)
    B = counts.shape[0]
    if world <= 0:
        raise ValueError("world must be positive")
    cum = np.concatenate([[0], np.cumsum(counts)])
    total = cum[-1]
    bounds = []
    b0 = 0
    for r in range(world):
        if r == world - 1:
            b1 = B
        else:
            target = total * (r + 1) / world
            b1 = int(np.searchsorted(cum, target, side="left"))
            b1 = max(b1, b0 + (1 if B - b0 > world - r - 1 else 0))
            b1 = min(b1, B - (world - r - 1)) if B >= world else min(max(b1, b0), B)
        bounds.append((b0, b1))
        b0 = b1
    return bounds


def slice_events(events: dict, counts: np.ndarray, b0: int, b1: int) -> dict:
    """Events of windows [b0, b1) from concatenated per-window events, with
    ``batch_indices`` rebased so the shard's first window is 0."""
    counts = np.asarray(counts, dtype=np.int64)
    off = np.concatenate([[0], np.cumsum(counts)])
    e0, e1 = int(off[b0]), int(off[b1])
    out = {k: v[e0:e1] for k, v in events.items()}
    out["batch_indices"] = out["batch_indices"] - b0
    return out
