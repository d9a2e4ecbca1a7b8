"""Packed event batches: one host->device copy and one graph launch per forward.

The reference serving path (cortex/serve/worker.py:166-214) builds four Python
lists per batch, turns them into four int64 device tensors (four copies) and
runs the eager forward, whose packing step reads ``B`` and ``E_max`` back to
the host (cortex/models/cortex.py:137-142). Here a batch of host index arrays
goes to the library's native runner (``ck_runner_*``, csrc/runner.cpp): it is
narrowed into one int32 buffer in pinned memory, crosses to the device in one
copy, and runs as the launch of the CUDA graph of ``ck_forward_batch`` captured
for its shape bucket ``(B, capacity)``. ``capacity`` rounds the event count up
to a bucket (at most 1/16 extra slots, ``capacity_for``); padding events are
skipped on the device, so one graph serves every batch of its bucket.

One runner serves one (device, stream). Its graphs bake in the weight pointers
of the model description they were captured with: when the description
changes (weights moved, recast or replaced, modules swapped) the runner drops
its graphs. They also bake in the kernel selection of their capture: the
library's environment switches (CK_PDL, CK_HEAD_FUSED, CK_LN_FUSE, CK_SIDE,
CK_GEMM_PAIR, CK_GEMM_SPLIT) are read then, and ``BatchRunner.invalidate()``
makes later batches capture afresh.
"""

from __future__ import annotations

import ctypes
import threading
import weakref

import torch

from cortex import _lib as L


def capacity_for(n_events: int) -> int:
    """Event slots of the bucket that holds ``n_events`` (a multiple of 256;
    the native runner uses the same rule)."""
    if n_events <= 256:
        return 256
    g = 1 << max(8, n_events.bit_length() - 5)
    return -(-n_events // g) * g


class _Arena:
    """A native runner for one (device, stream) and the description it uses."""

    def __init__(self, device: torch.device, model_desc) -> None:
        self.device = device
        handle = ctypes.c_void_p()
        L.check(L.load().ck_runner_create(ctypes.byref(model_desc), 64, ctypes.byref(handle)),
                "ck_runner_create")
        self.handle = handle
        self.native = None
        self._fin = weakref.finalize(self, L.load().ck_runner_destroy, handle)

    def counters(self) -> tuple[int, int]:
        c, r = ctypes.c_longlong(), ctypes.c_longlong()
        L.check(L.load().ck_runner_counters(self.handle, ctypes.byref(c), ctypes.byref(r)),
                "ck_runner_counters")
        return int(c.value), int(r.value)


class BatchRunner:
    """Runs ``CortexModel`` forwards from host index arrays (or a packed device
    batch) through the native runner. Thread-safe: one lock serialises staging
    and launch, as the reference's single executor thread does
    (cortex/serve/worker.py:112-113)."""

    def __init__(self, model) -> None:
        self.model = model
        self._arenas: dict[tuple[torch.device, int], _Arena] = {}
        self._lock = threading.Lock()
        self._bdim = int(model.config.behavior_dim)

    @property
    def captures(self) -> int:
        """Graphs captured so far (all arenas)."""
        return sum(a.counters()[0] for a in self._arenas.values())

    @property
    def replays(self) -> int:
        """Batches served by a graph launch so far (all arenas)."""
        return sum(a.counters()[1] for a in self._arenas.values())

    def invalidate(self) -> None:
        """Drop every captured graph; later batches capture again."""
        with self._lock:
            for a in self._arenas.values():
                L.check(L.load().ck_runner_invalidate(a.handle, None), "ck_runner_invalidate")

    def _arena(self, dev: torch.device, stream: int, m) -> _Arena:
        """The arena of (dev, stream), holding the model's current description m."""
        model = self.model
        native = model._native
        a = self._arenas.get((dev, stream))
        if a is None:
            a = _Arena(dev, m)
            self._arenas[(dev, stream)] = a
        elif a.native is not native:
            L.check(L.load().ck_runner_invalidate(a.handle, ctypes.byref(m)),
                    "ck_runner_invalidate")
        a.native = native  # keeps the weights the graphs point at alive
        return a

    def forward_host(self, neuron_ids: torch.Tensor, time_bins: torch.Tensor,
                     values: torch.Tensor, batch_indices: torch.Tensor,
                     batch_size: int | None = None) -> torch.Tensor:
        """(B, behavior_dim) on the model's device from four host (E,) index tensors."""
        idx = (neuron_ids, time_bins, values, batch_indices)
        dt = neuron_ids.dtype
        # (explicit comparisons: this runs once per request batch)
        if ((dt is not torch.int64 and dt is not torch.int32) or time_bins.dtype is not dt
                or values.dtype is not dt or batch_indices.dtype is not dt):
            dt = torch.int64
            idx = tuple(x.to(torch.int64) for x in idx)
        n_, t_, v_, b_ = idx
        if not (n_.is_contiguous() and t_.is_contiguous() and v_.is_contiguous()
                and b_.is_contiguous()):
            n_, t_, v_, b_ = (x.contiguous() for x in idx)
        E = n_.shape[0]
        lib = L.load()
        with self._lock:
            m, dev, wdt = self.model.native_info()
            stream = L.stream_of(dev)
            a = self._arena(dev, stream, m)
            B = ctypes.c_int32(0)
            rc = lib.ck_runner_stage(a.handle, n_.data_ptr(), t_.data_ptr(), v_.data_ptr(),
                                     b_.data_ptr(), L.CK_I64 if dt is torch.int64 else L.CK_I32,
                                     E, int(batch_size) if batch_size is not None else 0,
                                     ctypes.byref(B))
            L.check(rc, "ck_runner_stage")
            out = torch.empty(B.value, self._bdim, dtype=wdt, device=dev)
            L.check(lib.ck_runner_launch(a.handle, out.data_ptr(), stream), "ck_runner_launch")
            return out

    def forward_batch(self, batch: torch.Tensor, capacity: int, batch_size: int) -> torch.Tensor:
        """(B, behavior_dim) from a packed batch already on the model's device
        (e.g. written by ck_collate_bins): one device copy into the runner's
        buffer, then the graph of its bucket."""
        m, dev, wdt = self.model.native_info()
        if (batch.device != dev or batch.dtype != torch.int32
                or batch.numel() < L.batch_words(capacity)):
            raise ValueError("forward_batch: an int32 packed batch on the model's device")
        with self._lock:
            m, dev, wdt = self.model.native_info()
            stream = L.stream_of(dev)
            a = self._arena(dev, stream, m)
            out = torch.empty(int(batch_size), self._bdim, dtype=wdt, device=dev)
            L.check(L.load().ck_runner_launch_batch(a.handle, batch.data_ptr(), capacity,
                                                    int(batch_size), out.data_ptr(), stream),
                    "ck_runner_launch_batch")
            return out


__all__ = ["BatchRunner", "capacity_for"]
