"""Seeded synthetic workloads for the five benchmark configurations.

The reference profiles on MC_Maze recordings (scripts/profile_inference.py:81-108),
which are not available offline. These generators stand in for them with the
shapes and value distributions the benchmark names:

* ``neuron_id ~ U[0, 137)``, ``time_bin ~ U[0, 600)`` sorted within a sample,
* ``value = clip(Poisson(1.5) + 1, 0, 7)`` as an integer bucket index (the model
  embeds values through ``nn.Embedding(spike_value_buckets, D)``,
  cortex/models/tokenizer.py:48, and the data path buckets with
  ``clip(count, 0, n_buckets - 1)``, cortex/data/nlb.py:74-83),
* events concatenated in sample order, so ``batch_indices`` is sorted, which is
  the layout ``collate_events`` produces (cortex/data/nlb.py:492-512).

Weights are random init under ``torch.manual_seed(seed)`` followed by
``CortexModel(cfg)``; bf16 configs cast with ``.to(torch.bfloat16)`` and the
INT8 configs then quantize the 4 self-attention linears of every block with
``scale = absmax_row / 127`` through ``convert_model``
(cortex/quantization/calibrate.py:127-164, 240-264).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from cortex.models.config import CORTEX_S, CortexConfig

N_NEURONS_ACTIVE = 137
N_TIME_BINS_ACTIVE = 600
POISSON_LAMBDA = 1.5


@dataclass(frozen=True)
class Workload:
    name: str
    config: CortexConfig
    dtype: str  # "float32" | "bfloat16"
    int8: bool
    batch: int
    events_per_sample: int | None  # None: ragged log-uniform in [32, 4096]
    description: str


def _cfg_xs_variant() -> CortexConfig:
    return CortexConfig(
        hidden_dim=256, num_layers=4, num_heads=4, head_dim=64, num_latents=64,
        latent_dim=256, cross_attn_heads=4, max_neurons=512, max_time_bins=1024,
        behavior_dim=2,
    )


def _cfg_m_variant() -> CortexConfig:
    return CortexConfig(
        hidden_dim=768, num_layers=10, num_heads=12, head_dim=64, num_latents=512,
        latent_dim=768, cross_attn_heads=12, max_neurons=512, max_time_bins=1024,
        behavior_dim=2,
    )


WORKLOADS: dict[str, Workload] = {
    "cfg0": Workload("cfg0", _cfg_xs_variant(), "float32", False, 8, 256,
                     "Cortex-XS variant (D256 H4 4 layers L64) fp32, B=8 x 256 events"),
    "cfg1": Workload("cfg1", CORTEX_S, "bfloat16", False, 32, 512,
                     "Cortex-S bf16, B=32 x 512 events"),
    "cfg2": Workload("cfg2", CORTEX_S, "bfloat16", True, 32, 512,
                     "Cortex-S bf16 + per-channel INT8 self-attention weights, B=32 x 512 events"),
    "cfg3": Workload("cfg3", CORTEX_S, "bfloat16", False, 256, None,
                     "Cortex-S bf16, B=256 ragged log-uniform [32, 4096] events"),
    "cfg4": Workload("cfg4", _cfg_m_variant(), "bfloat16", True, 4096, 1024,
                     "Cortex-M variant (D768 H12 10 layers L512) bf16 + INT8, B=4096 x 1024 events"),
}


def events_per_sample(workload: Workload, seed: int = 0, batch: int | None = None) -> np.ndarray:
    """Per-sample event counts (int64, length ``batch``)."""
    b = workload.batch if batch is None else batch
    if workload.events_per_sample is not None:
        return np.full(b, workload.events_per_sample, dtype=np.int64)
    rng = np.random.default_rng(seed + 7919)
    u = rng.uniform(math.log(32.0), math.log(4096.0), size=b)
    return np.floor(np.exp(u)).astype(np.int64)


def make_events(counts: np.ndarray, seed: int = 0) -> dict[str, np.ndarray]:
    """Concatenated per-sample events as int64 numpy arrays.

    Sample ``b`` contributes ``counts[b]`` events drawn as: neuron ids, then
    sorted time bins, then values, all from one ``default_rng(seed)`` stream.
    """
    rng = np.random.default_rng(seed)
    nid, tb, val, bidx = [], [], [], []
    for b, n in enumerate(np.asarray(counts, dtype=np.int64).tolist()):
        nid.append(rng.integers(0, N_NEURONS_ACTIVE, size=n, dtype=np.int64))
        tb.append(np.sort(rng.integers(0, N_TIME_BINS_ACTIVE, size=n, dtype=np.int64)))
        val.append(np.clip(rng.poisson(POISSON_LAMBDA, size=n) + 1, 0, 7).astype(np.int64))
        bidx.append(np.full(n, b, dtype=np.int64))
    cat = (lambda xs: np.concatenate(xs) if xs else np.zeros(0, dtype=np.int64))
    return {
        "neuron_ids": cat(nid),
        "time_bins": cat(tb),
        "values": cat(val),
        "batch_indices": cat(bidx),
    }


def int8_layer_names(cfg: CortexConfig) -> list[str]:
    """Qualified names of the linears the INT8 configs quantize."""
    names = []
    for i in range(cfg.num_layers):
        for leaf in ("qkv_proj", "out_proj", "mlp.0", "mlp.2"):
            names.append(f"encoder.self_attn_blocks.{i}.{leaf}")
    return names


def build_model(workload: Workload, device="cpu", seed: int = 0):
    """``torch.manual_seed(seed); CortexModel(cfg)`` (+ bf16 cast, + INT8 conversion)."""
    import torch

    from cortex.models.cortex import CortexModel
    from cortex.quantization.calibrate import LayerScales, convert_model, weight_scales

    torch.manual_seed(seed)
    model = CortexModel(workload.config).eval()
    if workload.dtype == "bfloat16":
        model = model.to(torch.bfloat16)
    if workload.int8:
        scales = {n: LayerScales(weight_scale=weight_scales(model.get_submodule(n).weight),
                                 act_scale=1.0)
                  for n in int8_layer_names(workload.config)}
        convert_model(model, scales)
    return model.to(device)


def make_inputs(workload: Workload, seed: int = 0, batch: int | None = None):
    """Seeded events of ``batch`` windows (default: the workload's batch) as int64 tensors."""
    import torch

    counts = events_per_sample(workload, seed=seed)
    if batch is not None:
        if workload.events_per_sample is None:
            counts = events_per_sample(workload, seed=seed, batch=max(batch, workload.batch))
        else:
            counts = np.full(batch, workload.events_per_sample, dtype=np.int64)
        counts = counts[:batch]
    ev = make_events(counts, seed=seed)
    return {k: torch.from_numpy(v) for k, v in ev.items()}, counts
