"""Golden vectors for the event-ingest and batch-assembly rows.

Run in the build container with the reference importable:

    PYTHONPATH=/path/to/cortex-engine python tests/golden/make_ingest_golden.py

It imports the UNMODIFIED reference (peterajhgraham/cortex-engine) and records
what its own functions return for seeded inputs:

* ``bucket_values`` and ``events_from_bin_matrix`` (cortex/data/nlb.py:74-114)
  on Poisson count matrices with zero rows, negative and large counts;
* ``collate_events`` (cortex/data/nlb.py:492-512) over per-window items;
* ``InferenceWorker._run_batch_sync`` (cortex/serve/worker.py:152-251) on CPU
  with a recording stand-in model: the four index tensors it hands the model
  and the per-request results (zeros for requests past max(batch_index)).

The reference's logging module needs ``structlog``, which this container lacks;
a no-op stand-in is registered under that name before the import (the recorded
functions do not log). Output: golden_ingest.pt next to this file.
"""

from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class _NopLogger:
    def __getattr__(self, name):
        return lambda *a, **k: None


_sl = types.ModuleType("structlog")
_sl.get_logger = lambda *a, **k: _NopLogger()
_sl.stdlib = types.SimpleNamespace(BoundLogger=object)
sys.modules.setdefault("structlog", _sl)

import cortex  # noqa: E402  (the reference package, from PYTHONPATH)

assert "cortex-engine_b200" not in os.path.abspath(cortex.__file__), \
    "run with the reference on PYTHONPATH, not this repository's package"

from cortex.data.nlb import bucket_values, collate_events, events_from_bin_matrix  # noqa: E402
from cortex.models.config import CORTEX_S  # noqa: E402
from cortex.serve.worker import InferenceWorker  # noqa: E402


def count_matrix(rng, T, N, rate):
    c = rng.poisson(rate, size=(T, N)).astype(np.int32)
    c[rng.integers(0, T, size=max(T // 10, 1))] = 0          # silent bins
    c[rng.integers(0, T), rng.integers(0, N)] = 40             # a burst past the top bucket
    return c


def main() -> None:
    rng = np.random.default_rng(2024)
    out: dict = {}
    raw = rng.integers(-3, 20, size=257).astype(np.int64)
    out["bucket"] = {"counts": raw, "n_buckets": 8, "out": bucket_values(raw, 8)}

    mats = []
    for T, N, rate, nb in ((120, 137, 0.05, 8), (64, 33, 0.4, 4), (30, 1, 1.0, 8)):
        c = count_matrix(rng, T, N, rate)
        nid, tb, val = events_from_bin_matrix(c, nb)
        mats.append({"counts": c, "n_buckets": nb, "neuron_ids": nid, "time_bins": tb,
                     "values": val})
    out["events"] = mats

    # windows of one session, as NLBDataset items, then collate_events
    sess = count_matrix(rng, 400, 96, 0.08)
    starts = [0, 10, 50, 51, 300, 340]
    W, nb, offset = 60, 8, 7
    items = []
    for s in starts:
        nid, tb, val = events_from_bin_matrix(sess[s:s + W], nb)
        items.append({"neuron_ids": torch.from_numpy(nid + offset),
                      "time_bins": torch.from_numpy(tb), "values": torch.from_numpy(val),
                      "behavior": torch.zeros(2)})
    col = collate_events(items)
    out["collate"] = {"counts": sess, "starts": np.asarray(starts), "window_bins": W,
                      "n_buckets": nb, "neuron_offset": offset,
                      **{k: col[k].numpy() for k in ("neuron_ids", "time_bins", "values",
                                                     "batch_indices")}}

    # the worker's batch assembly, through a recording model
    cfg = CORTEX_S
    seen = {}

    class Recorder(torch.nn.Module):
        def forward(self, nid, tb, val, bidx):
            seen.update(neuron_ids=nid.numpy().copy(), time_bins=tb.numpy().copy(),
                        values=val.numpy().copy(), batch_indices=bidx.numpy().copy())
            B = int(bidx.max()) + 1
            return {"behavior": torch.arange(B * cfg.behavior_dim, dtype=torch.float32)
                    .reshape(B, cfg.behavior_dim)}

    worker = InferenceWorker(Recorder(), cfg, torch.device("cpu"), max_batch_size=32)
    payloads = []
    for i, n in enumerate((5, 0, 12, 3, 0, 0)):
        ev = [{"neuron_id": int(a), "time_bin": int(b), "value": int(v)}
              for a, b, v in zip(rng.integers(0, 137, n), rng.integers(0, 600, n),
                                 rng.integers(0, 8, n))]
        payloads.append({"request_id": f"req{i}", "events": ev})
    res = worker._run_batch_sync(payloads)
    worker.shutdown()
    out["worker"] = {"payloads": payloads, **seen,
                     "request_ids": [r["request_id"] for r in res],
                     "behavior": [r["behavior"] for r in res]}
    path = os.path.join(HERE, "golden_ingest.pt")
    torch.save(out, path)
    print("wrote", path)


if __name__ == "__main__":
    main()
