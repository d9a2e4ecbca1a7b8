"""Inference worker: batched forwards from request payloads (cortex/serve/worker.py).

Same contract as the reference ``InferenceWorker`` (cortex/serve/worker.py:93-260):
payloads ``{"request_id", "events": [{"neuron_id", "time_bin", "value"}, ...]}``
in, ``{"request_id", "behavior", "inference_ms"}`` out; forwards serialised on
one executor thread; a batch whose payloads hold no events returns zeros, and
trailing payloads without events get zeros, because ``B = max(batch_index) + 1``
drops them (cortex/serve/worker.py:182-190, 240-249).

The batch assembly is the B200 path: the events are read out of the payload
dicts by C-level iterators (``operator.itemgetter``), the four index arrays go
through ``CortexModel.forward``'s host path -- one packed int32 batch in pinned
memory (native ``ck_batch_stage``), one host-to-device copy and a CUDA-graph
replay per (B, event-capacity) bucket (cortex.batching) -- on the worker's
compute stream. The Prometheus metrics of the reference's control plane are not
part of this package; ``last_batch`` keeps the same figures for a caller.
"""

from __future__ import annotations

import asyncio
import time
from concurrent.futures import ThreadPoolExecutor
from operator import itemgetter
from typing import Any

import numpy as np
import torch
from torch import nn

from cortex.models.config import CortexConfig

def load_model(config: CortexConfig, checkpoint_path: str | None = None,
               device: torch.device | None = None) -> nn.Module:
    """CortexModel on ``device`` in eval mode, optionally from a checkpoint
    (cortex/serve/worker.py:59-89). The B200 path needs a CUDA device."""
    from cortex.models.cortex import CortexModel

    if device is None:
        device = torch.device("cuda")
    model = CortexModel(config).to(device).eval()
    if checkpoint_path:
        try:
            payload = torch.load(checkpoint_path, map_location=device, weights_only=False)
        except FileNotFoundError:
            return model
        state = payload.get("model_state_dict", payload)
        model.load_state_dict(state, strict=False)
    return model


def assemble_events(payloads: list[dict[str, Any]]) -> tuple[np.ndarray, ...]:
    """(neuron_ids, time_bins, values, batch_indices) int64 arrays of a batch, in
    payload order (cortex/serve/worker.py:166-178). Each field is read out of the
    event dicts by one C-level iterator (``np.fromiter`` over ``itemgetter``)."""
    counts = np.fromiter((len(p.get("events", ())) for p in payloads), np.int64, len(payloads))
    evs = [ev for p in payloads for ev in p.get("events", ())]
    E = len(evs)
    cols = tuple(np.fromiter(map(itemgetter(f), evs), np.int64, E)
                 for f in ("neuron_id", "time_bin", "value"))
    bidx = np.repeat(np.arange(len(payloads), dtype=np.int64), counts)
    return cols + (bidx,)


class InferenceWorker:
    """Batched inference worker: one model, one GPU, one executor thread."""

    def __init__(self, model: nn.Module, config: CortexConfig, device: torch.device,
                 max_batch_size: int = 32) -> None:
        self.model = model
        self.config = config
        self.device = torch.device(device)
        self.max_batch_size = max_batch_size
        self._executor = ThreadPoolExecutor(max_workers=1, thread_name_prefix="inference")
        if self.device.type != "cuda":
            raise RuntimeError("InferenceWorker: the B200 forward needs a CUDA device")
        self._compute_stream = torch.cuda.Stream(device=self.device)
        self._loaded = False
        self.last_batch: dict[str, float] = {}

    def warmup(self, n_iters: int = 3) -> None:
        """Dummy batches (cortex/serve/worker.py:138-150); the first one also
        captures the graph of its shape bucket."""
        dummy = [{"request_id": f"warmup_{i}",
                  "events": [{"neuron_id": 0, "time_bin": 0, "value": 0} for _ in range(64)]}
                 for i in range(min(n_iters, self.max_batch_size))]
        for _ in range(n_iters):
            self._run_batch_sync(dummy)
        self._loaded = True

    @property
    def ready(self) -> bool:
        return self._loaded

    async def run_batch(self, payloads: list[dict[str, Any]]) -> list[dict[str, Any]]:
        if not payloads:
            return []
        loop = asyncio.get_running_loop()
        return await loop.run_in_executor(self._executor, self._run_batch_sync, payloads)

    def _run_batch_sync(self, payloads: list[dict[str, Any]]) -> list[dict[str, Any]]:
        t0 = time.perf_counter()
        dim = self.config.behavior_dim
        nids, tbs, vals, bidx = assemble_events(payloads)
        if nids.size == 0:
            ms = (time.perf_counter() - t0) * 1000
            return [{"request_id": p["request_id"], "behavior": [0.0] * dim, "inference_ms": ms}
                    for p in payloads]
        with torch.cuda.stream(self._compute_stream), torch.inference_mode():
            out = self.model(torch.from_numpy(nids), torch.from_numpy(tbs),
                             torch.from_numpy(vals), torch.from_numpy(bidx))["behavior"]
            behavior = out.float().cpu().tolist()  # synchronises the compute stream
        ms = (time.perf_counter() - t0) * 1000
        self.last_batch = {"batch_size": float(len(payloads)), "n_events": float(nids.size),
                           "inference_ms": ms}
        return [{"request_id": p["request_id"],
                 "behavior": behavior[i] if i < len(behavior) else [0.0] * dim,
                 "inference_ms": ms} for i, p in enumerate(payloads)]

    def shutdown(self) -> None:
        self._executor.shutdown(wait=False)


__all__ = ["InferenceWorker", "assemble_events", "load_model"]
