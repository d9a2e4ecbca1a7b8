"""CortexModel forwards that reuse cached kv_proj rows of whole windows.

For a batch of windows, each keyed by (session_id, bin_start):

1. windows found in the cache (same key, same event count) are hits; the
   others are misses;
2. ``ck_forward_kv`` runs packing, tokenizer + norm_kv and kv_proj for the
   missed windows only (one packed int32 batch, one host-to-device copy);
3. ``ck_copy_rows`` assembles the batch's packed K|V rows: hits from their
   pool pages, misses from step 2, and writes the missed windows' rows into
   newly reserved pages;
4. ``ck_forward_from_kv`` runs the rest of the forward (latent queries, cross
   attention, the self-attention stack, the head).

Every K|V row depends only on its own event, so the result is the forward of
the whole batch: the same kernels over the same rows in the same order.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from cortex import _lib as L


def _host_i64(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.cpu().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.int64))


def forward_with_kv_cache(model, windows: list[dict], cache) -> torch.Tensor:
    """(B, behavior_dim) for ``windows`` (dicts with session_id, bin_start,
    neuron_ids, time_bins, values as host (E_b,) int arrays)."""
    from cortex.batching import capacity_for

    cfg = model.config
    w0 = model.tokenizer.neuron_emb.weight
    dev, dtype = w0.device, w0.dtype
    D2 = 2 * cfg.latent_dim
    if cache.hidden_dim != D2 or cache._pool.dtype != dtype or cache.device != dev:
        raise ValueError(f"the cache must hold ({D2},) {dtype} rows on {dev} (kv_proj output)")
    B = len(windows)
    if B == 0:
        raise ValueError("forward_streaming: no windows")
    ev = [tuple(_host_i64(w[k]) for k in ("neuron_ids", "time_bins", "values")) for w in windows]
    counts = np.array([len(e[0]) for e in ev], dtype=np.int64)
    for b, e in enumerate(ev):
        if not len(e[0]) == len(e[1]) == len(e[2]):
            raise ValueError(f"window {b}: neuron_ids, time_bins and values differ in length")
    metas = [cache.lookup(w["session_id"], int(w["bin_start"])) for w in windows]
    hit = [mt is not None and mt.n_events == counts[b] for b, mt in enumerate(metas)]
    miss = [b for b in range(B) if not hit[b]]

    m = model.native_model()
    lib = L.load()
    stream = L.stream_of(dev)
    E_all = int(counts.sum())
    off_all = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(counts, out=off_all[1:])
    row_bytes = D2 * w0.element_size()

    # 2. K|V rows of the missed windows
    kv_miss = off_miss = None
    cap = 0
    ws_need = lib.ck_forward_workspace_bytes(ctypes.byref(m), max(E_all, 1), B)
    if miss:
        sel = [ev[b] for b in miss]
        E_miss = int(counts[miss].sum())
        cap = capacity_for(E_miss)
        host = torch.empty(L.batch_words(cap), dtype=torch.int32, pin_memory=True)
        cols = [np.concatenate([s[k] for s in sel]) for k in range(3)]
        cols.append(np.repeat(np.arange(len(miss), dtype=np.int64), counts[miss]))
        b_out = ctypes.c_int32(0)
        rc = lib.ck_batch_stage(*(c.ctypes.data for c in cols), L.CK_I64, E_miss,
                                host.data_ptr(), cap, ctypes.byref(b_out))
        L.check(rc, "ck_batch_stage")
        batch = host.to(dev, non_blocking=True)
        kv_miss = torch.empty(cap, D2, dtype=dtype, device=dev)
        off_miss = torch.empty(len(miss) + 1, dtype=torch.int32, device=dev)
        ws_need = max(ws_need, lib.ck_forward_workspace_bytes(ctypes.byref(m), cap, len(miss)))
        ws = model.workspace(dev, ws_need)
        rc = lib.ck_forward_kv(ctypes.byref(m), batch.data_ptr(), cap, len(miss),
                               kv_miss.data_ptr(), off_miss.data_ptr(), ws.data_ptr(),
                               ws.numel(), stream)
        L.check(rc, "ck_forward_kv")
    ws = model.workspace(dev, ws_need)

    # 3. assemble the batch's rows; cache the missed windows
    seg_hit, seg_miss, seg_write = [], [], []
    for b in range(B):
        if hit[b]:
            seg_hit += cache.segments(metas[b], int(off_all[b]), into_pool=False)
    miss_off = np.zeros(len(miss) + 1, dtype=np.int64)
    np.cumsum(counts[miss], out=miss_off[1:])
    written = []
    for j, b in enumerate(miss):
        seg_miss.append((int(miss_off[j]), int(off_all[b]), int(counts[b])))
        w = windows[b]
        meta = cache.write_rows(w["session_id"], int(w["bin_start"]), int(counts[b]))
        if meta is not None:
            written.append((meta, int(miss_off[j])))
    # A later window of this batch may have evicted an earlier one and taken its
    # pages: copy only the entries still live, so no two copies share a page.
    for meta, row0 in written:
        if cache.is_live(meta):
            seg_write += cache.segments(meta, row0, into_pool=True)
    all_missed = len(miss) == B
    meta_h = np.concatenate([off_all, np.asarray(seg_hit + seg_miss + seg_write,
                                                 dtype=np.int64).reshape(-1)]).astype(np.int32)
    meta_d = torch.from_numpy(meta_h).pin_memory().to(dev, non_blocking=True)
    off_d = meta_d[:B + 1]
    segs = meta_d[B + 1:]
    nh, nm, nw = len(seg_hit), len(seg_miss), len(seg_write)
    pool_rows = cache.num_pages * cache.page_size
    if all_missed:
        kv_all, off_d = kv_miss, off_miss
        n_rows = cap
    else:
        n_rows = max(E_all, 1)
        kv_all = torch.empty(n_rows, D2, dtype=dtype, device=dev)
        if nh:
            L.check(lib.ck_copy_rows(cache.rows.data_ptr(), pool_rows, kv_all.data_ptr(), n_rows,
                                     row_bytes, segs.data_ptr(), nh, stream), "ck_copy_rows")
        if nm:
            L.check(lib.ck_copy_rows(kv_miss.data_ptr(), cap, kv_all.data_ptr(), n_rows,
                                     row_bytes, segs[3 * nh:].data_ptr(), nm, stream),
                    "ck_copy_rows")
    if nw:
        L.check(lib.ck_copy_rows(kv_miss.data_ptr(), cap, cache.rows.data_ptr(), pool_rows,
                                 row_bytes, segs[3 * (nh + nm):].data_ptr(), nw, stream),
                "ck_copy_rows")

    # 4. the rest of the forward
    out = torch.empty(B, cfg.behavior_dim, dtype=dtype, device=dev)
    rc = lib.ck_forward_from_kv(ctypes.byref(m), kv_all.data_ptr(), n_rows, off_d.data_ptr(), B,
                                out.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    L.check(rc, "ck_forward_from_kv")
    return out


__all__ = ["forward_with_kv_cache"]
