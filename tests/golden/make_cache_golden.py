"""Golden trace of the reference StreamingKVCache (cortex/cache/streaming.py).

Run in the build container with the reference importable:

    PYTHONPATH=/path/to/cortex-engine python tests/golden/make_cache_golden.py

It drives the UNMODIFIED reference cache on the CPU through a seeded sequence of
write / read / evict_session calls on a small pool (so LRU eviction, page reuse
for a rewritten key and truncation to page_size all occur) and records every
observable: read results (rows or None), evict_session counts, hit_rate and
pages_used after each call. The reference's logging needs ``structlog``, which
this container lacks; a no-op stand-in is registered under that name first.
Output: golden_cache.pt next to this file.
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

from cortex.cache.streaming import StreamingKVCache  # noqa: E402

NUM_PAGES, PAGE_SIZE, DIM = 4, 8, 16


def main() -> None:
    rng = np.random.default_rng(77)
    cache = StreamingKVCache(num_pages=NUM_PAGES, page_size=PAGE_SIZE, hidden_dim=DIM,
                             dtype=torch.float32, device="cpu")
    sessions, starts = ["a", "b", "c"], [0, 5, 10, 15]
    ops, results = [], []
    for step in range(120):
        r = rng.random()
        sid = sessions[int(rng.integers(0, len(sessions)))]
        start = starts[int(rng.integers(0, len(starts)))]
        if r < 0.45:
            n = int(rng.integers(0, 2 * PAGE_SIZE))
            emb = torch.from_numpy(rng.standard_normal((n, DIM)).astype(np.float32))
            cache.write(sid, start, emb)
            ops.append(("write", sid, start, emb))
            out = None
        elif r < 0.93:
            got = cache.read(sid, start)
            ops.append(("read", sid, start, None))
            out = None if got is None else got.clone()
        else:
            ops.append(("evict", sid, None, None))
            out = cache.evict_session(sid)
        results.append({"out": out, "hit_rate": cache.hit_rate, "pages_used": cache.pages_used})
    path = os.path.join(HERE, "golden_cache.pt")
    torch.save({"num_pages": NUM_PAGES, "page_size": PAGE_SIZE, "hidden_dim": DIM, "ops": ops,
                "results": results}, path)
    print("wrote", path)


if __name__ == "__main__":
    main()
