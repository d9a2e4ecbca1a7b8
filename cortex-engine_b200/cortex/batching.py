"""Packed event batches: one host->device copy and one graph replay per forward.

The reference serving path (cortex/serve/worker.py:166-214) builds four Python
lists per batch, turns them into four int64 device tensors (four copies) and
runs the eager forward, whose packing step reads ``B`` and ``E_max`` back to
the host (cortex/models/cortex.py:137-142). Here a batch of host index arrays
becomes one int32 buffer in pinned memory (``ck_batch_stage``, native, one
pass per array), crosses to the device in one ``cudaMemcpyAsync`` and runs as
the replay of a CUDA graph of ``ck_forward_batch`` captured for its shape
bucket ``(B, capacity)``. ``capacity`` rounds the event count up to a bucket
(at most 1/32 to 1/16 extra slots); the padding events are skipped on the
device, so one graph serves every batch of its bucket.

The device batch buffer, the forward workspace and the graphs belong to one
``_Arena`` per (device, stream): graphs bake in those addresses, so an arena
that has to grow drops its graphs and re-captures them on demand. A graph also
bakes in the kernel selection of its capture: the library's environment
switches (CK_PDL, CK_HEAD_FUSED, CK_NORM_FOLD, CK_LN_FUSE) are read then, and
``BatchRunner.invalidate()`` makes later batches capture afresh.
"""

from __future__ import annotations

import ctypes
import os
import threading
from collections import OrderedDict

import torch

from cortex import _lib as L


def capacity_for(n_events: int) -> int:
    """Event slots of the bucket that holds ``n_events`` (a multiple of 256)."""
    if n_events <= 256:
        return 256
    g = 1 << max(8, n_events.bit_length() - 5)
    return -(-n_events // g) * g


def graphs_enabled() -> bool:
    """CK_BATCH_GRAPHS=0 in the environment runs every batch as eager launches."""
    return os.environ.get("CK_BATCH_GRAPHS", "1") != "0"


class _Slot:
    """One pinned staging buffer and the event after the copy that read it."""

    def __init__(self, words: int) -> None:
        self.host = torch.empty(words, dtype=torch.int32, pin_memory=True)
        self.copied: torch.cuda.Event | None = None


class _Arena:
    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.capacity = 0
        self.batch: torch.Tensor | None = None      # device int32 batch buffer
        self.ws: torch.Tensor | None = None         # forward workspace
        self.slots: list[_Slot] = []
        self.next_slot = 0
        self.graphs: OrderedDict[tuple[int, int], tuple[torch.cuda.CUDAGraph, torch.Tensor]] = \
            OrderedDict()
        self.native = None                          # the weight description the graphs use

    def drop_graphs(self) -> None:
        self.graphs.clear()

    def reserve(self, capacity: int) -> None:
        """Device buffer and pinned slots for ``capacity`` events (grows by 1.25x)."""
        if capacity <= self.capacity:
            return
        cap = max(capacity, capacity_for(int(self.capacity * 1.25)))
        words = L.batch_words(cap)
        self.drop_graphs()
        torch.cuda.synchronize(self.device)  # earlier copies may still read the old slots
        self.batch = torch.empty(words, dtype=torch.int32, device=self.device)
        self.slots = [_Slot(words), _Slot(words)]
        self.next_slot = 0
        self.capacity = cap

    def workspace(self, nbytes: int) -> torch.Tensor:
        if self.ws is None or self.ws.numel() < nbytes:
            self.drop_graphs()
            torch.cuda.synchronize(self.device)
            self.ws = torch.empty(int(nbytes * 1.25) + 4096, dtype=torch.uint8,
                                  device=self.device)
        return self.ws


class BatchRunner:
    """Runs ``CortexModel`` forwards from host index arrays through packed batches.

    Used by ``CortexModel.forward`` for host-resident inputs and by the
    inference worker. Thread-safe: one lock serialises staging and launch, as
    the reference's single executor thread does (cortex/serve/worker.py:112-113).
    """

    def __init__(self, model, max_graphs: int = 64) -> None:
        self.model = model
        self.max_graphs = max_graphs
        self._arenas: dict[tuple[torch.device, int], _Arena] = {}
        self._lock = threading.Lock()
        self.captures = 0   # graphs captured so far (tests and diagnostics)
        self.replays = 0

    def _arena(self, dev: torch.device, stream: int) -> _Arena:
        key = (dev, stream)
        a = self._arenas.get(key)
        if a is None:
            a = _Arena(dev)
            self._arenas[key] = a
        return a

    def invalidate(self) -> None:
        """Drop every captured graph (weights moved, recast or replaced)."""
        with self._lock:
            for a in self._arenas.values():
                a.drop_graphs()
                a.native = None

    def forward_host(self, neuron_ids: torch.Tensor, time_bins: torch.Tensor,
                     values: torch.Tensor, batch_indices: torch.Tensor,
                     batch_size: int | None = None) -> torch.Tensor:
        """(B, behavior_dim) on the model's device from four host (E,) index tensors."""
        idx = [neuron_ids, time_bins, values, batch_indices]
        dt = idx[0].dtype if all(x.dtype == idx[0].dtype for x in idx) else torch.int64
        if dt not in (torch.int32, torch.int64):
            dt = torch.int64
        idx = [x.to(dtype=dt).contiguous() for x in idx]
        E = int(idx[0].shape[0])
        model = self.model
        dev = model.tokenizer.neuron_emb.weight.device
        with self._lock:
            stream = L.stream_of(dev)
            arena = self._arena(dev, stream)
            cap = capacity_for(E)
            arena.reserve(cap)
            slot = arena.slots[arena.next_slot]
            arena.next_slot ^= 1
            if slot.copied is not None:
                slot.copied.synchronize()  # the copy two batches ago has read this slot
            b_out = ctypes.c_int32(0)
            lib = L.load()
            rc = lib.ck_batch_stage(idx[0].data_ptr(), idx[1].data_ptr(), idx[2].data_ptr(),
                                    idx[3].data_ptr(), L.dtype_code(dt), E,
                                    slot.host.data_ptr(), cap, ctypes.byref(b_out))
            L.check(rc, "ck_batch_stage")
            B = int(batch_size) if batch_size is not None else int(b_out.value)
            words = L.batch_words(cap)
            arena.batch[:words].copy_(slot.host[:words], non_blocking=True)
            if slot.copied is None:
                slot.copied = torch.cuda.Event()
            slot.copied.record(torch.cuda.current_stream(dev))
            return self._run(arena, B, cap, stream)

    def forward_batch(self, batch: torch.Tensor, capacity: int, batch_size: int) -> torch.Tensor:
        """(B, behavior_dim) from a packed batch already on the model's device
        (e.g. written by ck_collate_bins): one device copy into the arena's
        buffer, then the graph of its bucket."""
        model = self.model
        dev = model.tokenizer.neuron_emb.weight.device
        words = L.batch_words(capacity)
        if batch.device != dev or batch.dtype != torch.int32 or batch.numel() < words:
            raise ValueError("forward_batch: an int32 packed batch on the model's device")
        with self._lock:
            stream = L.stream_of(dev)
            arena = self._arena(dev, stream)
            arena.reserve(capacity)
            # the launch's capacity fixes the layout; the arena buffer may be longer
            arena.batch[:words].copy_(batch[:words])
            return self._run(arena, int(batch_size), capacity, stream)

    def _run(self, arena: _Arena, B: int, cap: int, stream: int) -> torch.Tensor:
        model = self.model
        m = model.native_model()
        model._refresh_folds()
        native = model._native
        if arena.native is not native:
            arena.drop_graphs()
            arena.native = native  # keeps the weights the graphs point at alive
        lib = L.load()
        ws = arena.workspace(lib.ck_forward_workspace_bytes(ctypes.byref(m), cap, B))
        dev = arena.device
        dim = model.config.behavior_dim
        dtype = model.tokenizer.neuron_emb.weight.dtype
        key = (B, cap)
        hit = arena.graphs.get(key)
        if hit is not None:
            arena.graphs.move_to_end(key)
            hit[0].replay()
            self.replays += 1
            return hit[1].clone()

        def launch(out: torch.Tensor, strm: int) -> None:
            rc = lib.ck_forward_batch(ctypes.byref(m), arena.batch.data_ptr(), cap, B,
                                      out.data_ptr(), ws.data_ptr(), ws.numel(), strm)
            L.check(rc, "ck_forward_batch")

        out = torch.empty(B, dim, dtype=dtype, device=dev)
        launch(out, stream)  # this batch's result, and first-use setup outside capture
        if graphs_enabled():
            g_out = torch.empty(B, dim, dtype=dtype, device=dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                launch(g_out, L.stream_of(dev))
            arena.graphs[key] = (g, g_out)
            self.captures += 1
            while len(arena.graphs) > self.max_graphs:
                arena.graphs.popitem(last=False)
        return out


__all__ = ["BatchRunner", "capacity_for", "graphs_enabled"]
