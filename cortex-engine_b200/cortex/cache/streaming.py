"""Paged cache of per-window rows in HBM (cortex/cache/streaming.py:79-236).

Same API and policy as the reference ``StreamingKVCache``: a pool of
``num_pages`` pages of ``page_size`` rows of ``hidden_dim`` elements, a page
table keyed by ``(session_id, bin_start)``, least-recently-used eviction across
sessions, ``read`` / ``write`` / ``evict_session`` / ``hit_rate`` /
``pages_used``. The pool is one CUDA tensor; the table and the LRU order are
host metadata.

Two additions wire it to the forward (``CortexModel.forward_streaming``):

* an entry may span several pages (``write_rows``): the kv_proj rows of a
  whole window, ``ceil(rows / page_size)`` pages, evicted together;
* ``segments`` gives the (src_row, dst_row, rows) copy list between the pool
  and a packed row buffer that ``ck_copy_rows`` executes on the device, so
  cached rows move HBM to HBM with no host round trip.

What is cached must be a function of the key alone. kv_proj rows of a window
are (they depend only on the window's own events), so the key is the window
identity (session, first bin). Rows of the same spike in an overlapping window
are NOT the same: time bins are window-relative (a max_time_bins vocabulary),
so a shifted window shifts every time embedding.
"""

from __future__ import annotations

import time
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

from cortex import _lib as L


@dataclass
class PageMeta:
    """One cache entry (cortex/cache/streaming.py:67-75); ``pages`` lists its
    pages in row order (one page for entries made by ``write``)."""

    page_id: int
    session_id: str
    bin_start: int
    n_events: int
    last_used_at: float
    pages: list[int] = field(default_factory=list)


class StreamingKVCache:
    """Paged row cache in device memory.

    Args (cortex/cache/streaming.py:92-99): num_pages, page_size (rows per
    page), hidden_dim (elements per row), dtype, device (a CUDA device).
    """

    def __init__(self, num_pages: int = 128, page_size: int = 64, hidden_dim: int = 512,
                 dtype: torch.dtype = torch.float32, device: str | torch.device = "cuda") -> None:
        if num_pages <= 0 or page_size <= 0 or hidden_dim <= 0:
            raise ValueError("num_pages, page_size and hidden_dim must be positive")
        self.num_pages = num_pages
        self.page_size = page_size
        self.hidden_dim = hidden_dim
        self.device = torch.device(device)
        self._pool = torch.zeros(num_pages, page_size, hidden_dim, dtype=dtype,
                                 device=self.device)
        L.require_cuda(self._pool, what="StreamingKVCache")
        self.device = self._pool.device  # with its index (cuda -> cuda:N)
        self._table: dict[tuple[str, int], int] = {}      # key -> entry id (its first page)
        self._meta: dict[int, PageMeta] = {}              # entry id -> metadata
        self._free: list[int] = list(range(num_pages))
        self._lru: OrderedDict[int, None] = OrderedDict()  # entry ids, most recent last
        self._hits = 0
        self._misses = 0

    # ── reference API ────────────────────────────────────────────────────────

    def read(self, session_id: str, bin_start: int) -> torch.Tensor | None:
        """The cached rows of (session_id, bin_start), or None (a miss).
        A one-page entry returns a view of its page, as the reference does."""
        meta = self.lookup(session_id, bin_start)
        if meta is None:
            return None
        if len(meta.pages) == 1:
            return self._pool[meta.pages[0], :meta.n_events, :]
        return self._pool[meta.pages].reshape(-1, self.hidden_dim)[:meta.n_events]

    def write(self, session_id: str, bin_start: int, embeddings: torch.Tensor) -> None:
        """Cache the first ``page_size`` rows of ``embeddings`` in one page,
        reusing the key's page if present (cortex/cache/streaming.py:150-184)."""
        n = min(int(embeddings.shape[0]), self.page_size)
        meta = self._entry_for(session_id, bin_start, n_pages=1)
        self._pool[meta.pages[0], :n, :] = embeddings[:n].detach().to(
            dtype=self._pool.dtype, device=self.device)
        meta.n_events = n
        meta.last_used_at = time.monotonic()

    def evict_session(self, session_id: str) -> int:
        """Free every entry of ``session_id``; returns how many (:186-195)."""
        keys = [k for k in self._table if k[0] == session_id]
        for key in keys:
            self._free_entry(self._table[key])
        return len(keys)

    @property
    def hit_rate(self) -> float:
        total = self._hits + self._misses
        return self._hits / total if total > 0 else 0.0

    @property
    def pages_used(self) -> int:
        return self.num_pages - len(self._free)

    # ── multi-page entries and device copies ─────────────────────────────────

    def lookup(self, session_id: str, bin_start: int) -> PageMeta | None:
        """Entry of the key (counted as a hit, and made most recent) or None
        (counted as a miss)."""
        eid = self._table.get((session_id, bin_start))
        if eid is None:
            self._misses += 1
            return None
        self._lru.move_to_end(eid)
        meta = self._meta[eid]
        meta.last_used_at = time.monotonic()
        self._hits += 1
        return meta

    def write_rows(self, session_id: str, bin_start: int, n_rows: int) -> PageMeta | None:
        """Reserve pages for ``n_rows`` rows of the key (replacing an older
        entry); None when they cannot fit in the pool. The caller copies the
        rows in (``segments(meta, ..., into_pool=True)`` + ``ck_copy_rows``)."""
        n_pages = max(1, -(-n_rows // self.page_size))
        if n_pages > self.num_pages:
            return None
        meta = self._entry_for(session_id, bin_start, n_pages)
        meta.n_events = n_rows
        return meta

    def segments(self, meta: PageMeta, row0: int, into_pool: bool) -> list[tuple[int, int, int]]:
        """(src_row, dst_row, rows) between the entry's pages (pool rows) and
        rows row0.. of a packed buffer; pool -> buffer unless ``into_pool``."""
        out = []
        for k, page in enumerate(meta.pages):
            n = min(self.page_size, meta.n_events - k * self.page_size)
            if n <= 0:
                break
            p, b = page * self.page_size, row0 + k * self.page_size
            out.append((b, p, n) if into_pool else (p, b, n))
        return out

    def is_live(self, meta: PageMeta) -> bool:
        """Whether ``meta`` is still the entry that owns its pages."""
        return self._meta.get(meta.page_id) is meta

    @property
    def rows(self) -> torch.Tensor:
        """The pool as (num_pages * page_size, hidden_dim) rows."""
        return self._pool.view(self.num_pages * self.page_size, self.hidden_dim)

    # ── internals ────────────────────────────────────────────────────────────

    def _entry_for(self, session_id: str, bin_start: int, n_pages: int) -> PageMeta:
        key = (session_id, bin_start)
        eid = self._table.get(key)
        if eid is not None and len(self._meta[eid].pages) != n_pages:
            self._free_entry(eid)
            eid = None
        if eid is None:
            pages = self._allocate(n_pages)
            eid = pages[0]
            self._table[key] = eid
            self._meta[eid] = PageMeta(eid, session_id, bin_start, 0, time.monotonic(), pages)
            self._lru[eid] = None
        self._lru.move_to_end(eid)
        return self._meta[eid]

    def _allocate(self, n_pages: int) -> list[int]:
        """``n_pages`` free pages, evicting least-recently-used entries first."""
        while len(self._free) < n_pages:
            lru, _ = self._lru.popitem(last=False)
            self._free_entry(lru)
        return [self._free.pop() for _ in range(n_pages)]

    def _free_entry(self, eid: int) -> None:
        meta = self._meta.pop(eid, None)
        if meta is not None:
            self._table.pop((meta.session_id, meta.bin_start), None)
            self._free.extend(meta.pages)
        self._lru.pop(eid, None)


__all__ = ["PageMeta", "StreamingKVCache"]
