"""Spike-count windows to packed event batches on the device.

The reference turns each window of a session's (T, N) bin-count matrix into an
event list on the host (``events_from_bin_matrix`` + ``bucket_values``,
cortex/data/nlb.py:74-114, called per item at :249-280), and ``collate_events``
concatenates the items of a batch and builds ``batch_indices``
(cortex/data/nlb.py:492-512). Here the count matrices stay in HBM and
``ck_collate_bins`` writes a whole batch of windows as one packed event batch
(the CK_BATCH layout of cortex_b200.h) in three kernel launches, which
``CortexModel.forward_packed`` consumes without a host round trip of the
events.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from cortex import _lib as L


class BinWindow(ctypes.Structure):
    """ck_bin_window (cortex_b200.h)."""

    _fields_ = [("counts", ctypes.c_void_p), ("ld", ctypes.c_int64), ("n_rows", ctypes.c_int64),
                ("start", ctypes.c_int64), ("n_neurons", ctypes.c_int32),
                ("neuron_offset", ctypes.c_int32)]


@dataclass
class PackedBatch:
    """A packed event batch on the device.

    ``batch`` holds ``L.batch_words(capacity)`` int32 words: the header (n_valid)
    and the four event arrays of ``capacity`` slots; ``n_events`` is the number
    of real events, ``batch_size`` the number of windows (B).
    """

    batch: torch.Tensor
    capacity: int
    n_events: int
    batch_size: int

    def events(self) -> tuple[torch.Tensor, ...]:
        """(neuron_ids, time_bins, values, batch_indices) int32 views of the real events."""
        a = self.batch[L.CK_BATCH_HEADER_WORDS:]
        c, n = self.capacity, self.n_events
        return tuple(a[k * c:k * c + n] for k in range(4))


def _check_counts(counts: torch.Tensor) -> None:
    if counts.dim() != 2:
        raise ValueError(f"bin_counts must be (T, N), got shape {tuple(counts.shape)}")
    if counts.dtype != torch.int32:
        raise TypeError(f"bin_counts must be int32 (got {counts.dtype})")
    if counts.stride(1) != 1:
        raise ValueError("bin_counts rows must be contiguous")
    L.require_cuda(counts, what="collate_windows")


def collate_windows(windows: list[tuple[torch.Tensor, int, int]], window_bins: int,
                    n_buckets: int, max_neurons: int, capacity: int | None = None
                    ) -> PackedBatch:
    """Events of B windows as one packed batch on the device.

    Args:
        windows: (bin_counts, start_bin, neuron_id_offset) per window; bin_counts
            is a session's (T, N) int32 CUDA tensor, the window is rows
            ``start_bin : start_bin + window_bins``.
        window_bins: rows per window (NLBDataset window length in bins).
        n_buckets: value buckets (``bucket_values``).
        max_neurons: size of the neuron vocabulary; a larger id raises.
        capacity: event slots; default: the count's bucket (one host read).

    The result equals ``collate_events`` over ``events_from_bin_matrix`` of each
    window (with its neuron offset added), as int32.
    """
    if not windows:
        raise ValueError("collate_windows: no windows")
    if window_bins <= 0 or n_buckets <= 0:
        raise ValueError("window_bins and n_buckets must be positive")
    dev = windows[0][0].device
    B = len(windows)
    host = (BinWindow * B)()
    for i, (counts, start, offset) in enumerate(windows):
        _check_counts(counts)
        if counts.device != dev:
            raise ValueError("collate_windows: windows on different devices")
        T, N = counts.shape
        if not 0 <= int(start) <= T - window_bins:
            raise ValueError(f"window {i}: rows {start}..{int(start) + window_bins} outside (0, {T})")
        host[i].counts, host[i].ld, host[i].n_rows = counts.data_ptr(), counts.stride(0), T
        host[i].start, host[i].n_neurons, host[i].neuron_offset = int(start), N, int(offset)
    wins_h = torch.frombuffer(bytearray(host), dtype=torch.uint8)
    wins = wins_h.to(dev)
    lib = L.load()
    ws = torch.empty(max(lib.ck_collate_bins_workspace_bytes(B, window_bins), 1),
                     dtype=torch.uint8, device=dev)
    total = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = L.stream_of(dev)

    def run(batch: torch.Tensor, cap: int) -> None:
        rc = lib.ck_collate_bins(wins.data_ptr(), B, window_bins, n_buckets, max_neurons,
                                 batch.data_ptr(), cap, ws.data_ptr(), ws.numel(),
                                 total.data_ptr(), stream)
        L.check(rc, "ck_collate_bins")

    if capacity is None:
        from cortex.batching import capacity_for

        header = torch.empty(L.CK_BATCH_HEADER_WORDS, dtype=torch.int32, device=dev)
        run(header, 0)
        capacity = capacity_for(int(total.item()))
    if capacity % 4 != 0:
        raise ValueError("capacity must be a multiple of 4")
    batch = torch.empty(L.batch_words(capacity), dtype=torch.int32, device=dev)
    run(batch, capacity)
    n = int(total.item())
    code, info = L.device_status()
    if code == L.CK_ERR_INDEX:  # NLBDataset raises ValueError here (cortex/data/nlb.py:259-263)
        raise ValueError(f"neuron_id {info[1] if len(info) > 1 else '?'} exceeds "
                         f"max_neurons={max_neurons} (or a window lies outside its matrix)")
    if code != L.CK_OK:
        raise ValueError(f"ck_collate_bins: {L.status_string(code)} (info {info}); "
                         f"{n} events for capacity {capacity}")
    return PackedBatch(batch, capacity, n, B)


def events_from_bin_matrix(bin_counts: torch.Tensor, n_buckets: int
                           ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Nonzero bins of a (T, N) int32 CUDA matrix as int64 (neuron_ids,
    time_bins, values), values bucketed (cortex/data/nlb.py:86-114)."""
    _check_counts(bin_counts)
    T, N = bin_counts.shape
    if T == 0:
        z = torch.zeros(0, dtype=torch.int64, device=bin_counts.device)
        return z, z, z
    pb = collate_windows([(bin_counts, 0, 0)], T, n_buckets, max_neurons=max(N, 1))
    nid, tb, val, _ = pb.events()
    return nid.long(), tb.long(), val.long()


def bucket_values(counts: torch.Tensor, n_buckets: int) -> torch.Tensor:
    """clamp(counts, 0, n_buckets - 1) as int64 (cortex/data/nlb.py:74-83), on the
    device. ``collate_windows`` applies the same clamp inside its emit kernel."""
    if n_buckets <= 0:
        raise ValueError(f"n_buckets must be positive, got {n_buckets}")
    L.require_cuda(counts, what="bucket_values")
    return counts.clamp(0, n_buckets - 1).to(torch.int64)


def collate_events(batch: list[dict[str, torch.Tensor]]) -> dict[str, torch.Tensor]:
    """The reference's collate (cortex/data/nlb.py:492-512): concatenated event
    tensors, ``batch_indices`` of each item's position, stacked behaviour."""
    out = {k: torch.cat([b[k] for b in batch]) for k in ("neuron_ids", "time_bins", "values")}
    out["batch_indices"] = torch.cat(
        [torch.full((len(b["neuron_ids"]),), i, dtype=torch.int64) for i, b in enumerate(batch)])
    out["behavior"] = torch.stack([b["behavior"] for b in batch])
    return out


__all__ = ["BinWindow", "PackedBatch", "bucket_values", "collate_events", "collate_windows",
           "events_from_bin_matrix"]
