"""CPU oracle for the event-ingest and batch-assembly rows of the hot path.

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` as the checker of the device
ingest kernels (``ck_collate_bins``), the host batch staging (``ck_batch_stage``)
and the inference worker's batch assembly. The product never imports it.

Plain numpy restatements of the reference functions, each citing the lines it
follows; ``tests/test_oracle_golden.py`` pins them against vectors that
``tests/golden/make_ingest_golden.py`` recorded from the reference itself.
"""

from __future__ import annotations

import numpy as np

BATCH_HEADER_WORDS = 4


def bucket_values(counts: np.ndarray, n_buckets: int) -> np.ndarray:
    """cortex/data/nlb.py:74-83: clip to [0, n_buckets - 1], int64."""
    if n_buckets <= 0:
        raise ValueError(f"n_buckets must be positive, got {n_buckets}")
    return np.clip(counts, 0, n_buckets - 1).astype(np.int64)


def events_from_bin_matrix(bin_counts: np.ndarray, n_buckets: int
                           ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """cortex/data/nlb.py:86-114: nonzero bins in row-major order (time, neuron)."""
    if bin_counts.ndim != 2:
        raise ValueError(f"bin_counts must be (T, N), got shape {bin_counts.shape}")
    t, n = np.nonzero(bin_counts)
    return n.astype(np.int64), t.astype(np.int64), bucket_values(bin_counts[t, n], n_buckets)


def window_events(counts: np.ndarray, start: int, window_bins: int, neuron_offset: int,
                  n_buckets: int, max_neurons: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """One NLBDataset item (cortex/data/nlb.py:249-263): the window's events with
    the session's neuron offset added; an id past max_neurons raises."""
    nid, tb, val = events_from_bin_matrix(counts[start:start + window_bins], n_buckets)
    nid = nid + neuron_offset
    if nid.size > 0 and int(nid.max()) >= max_neurons:
        raise ValueError(f"neuron_id {int(nid.max())} exceeds max_neurons={max_neurons}")
    return nid, tb, val


def collate(items: list[tuple[np.ndarray, np.ndarray, np.ndarray]]) -> tuple[np.ndarray, ...]:
    """collate_events (cortex/data/nlb.py:492-512) without the behaviour field:
    concatenation in item order and the item index of every event."""
    cat = [np.concatenate([it[k] for it in items]) if items else np.zeros(0, np.int64)
           for k in range(3)]
    bidx = np.concatenate([np.full(len(it[0]), i, dtype=np.int64) for i, it in enumerate(items)]) \
        if items else np.zeros(0, np.int64)
    return cat[0], cat[1], cat[2], bidx


def worker_lists(payloads: list[dict]) -> tuple[np.ndarray, ...]:
    """InferenceWorker._run_batch_sync's flat event lists
    (cortex/serve/worker.py:166-178), as int64 arrays."""
    cols: list[list[int]] = [[], [], [], []]
    for b, p in enumerate(payloads):
        for ev in p.get("events", []):
            cols[0].append(int(ev["neuron_id"]))
            cols[1].append(int(ev["time_bin"]))
            cols[2].append(int(ev["value"]))
            cols[3].append(b)
    return tuple(np.asarray(c, dtype=np.int64) for c in cols)


def batch_size(batch_indices: np.ndarray) -> int:
    """B = max(batch_indices) + 1 (cortex/models/cortex.py:137), 1 for no events."""
    return int(batch_indices.max()) + 1 if batch_indices.size else 1


def packed_batch(nid, tb, val, bidx, capacity: int) -> np.ndarray:
    """The packed event batch the device consumes (header n_valid, then the four
    int32 arrays of ``capacity`` slots); padding slots are left zero here and
    must be ignored by any comparison."""
    E = len(nid)
    out = np.zeros(BATCH_HEADER_WORDS + 4 * capacity, dtype=np.int64)
    out[0] = E
    for k, a in enumerate((nid, tb, val, bidx)):
        out[BATCH_HEADER_WORDS + k * capacity:BATCH_HEADER_WORDS + k * capacity + E] = a
    return out
