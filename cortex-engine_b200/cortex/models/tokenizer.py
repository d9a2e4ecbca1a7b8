"""Spike tokenizer (drop-in for ``cortex.models.tokenizer``).

Same module, parameter names and initialisation as the reference
(cortex/models/tokenizer.py:39-54: three ``nn.Embedding`` tables re-initialised
with ``normal_(std=0.02)``), so ``state_dict``s and seeded random inits match.
``forward`` always runs the B200 fused tokenizer kernel.
"""

from __future__ import annotations

import torch
from torch import nn

from cortex.kernels.tokenizer import fused_tokenizer
from cortex.models.config import CortexConfig


class SpikeTokenizer(nn.Module):
    """Embed spike events as tokens: ``n_emb[nid] + t_emb[tb] + v_emb[val]``."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.config = config
        self.neuron_emb = nn.Embedding(config.max_neurons, config.hidden_dim)
        self.time_emb = nn.Embedding(config.max_time_bins, config.hidden_dim)
        self.value_emb = nn.Embedding(config.spike_value_buckets, config.hidden_dim)
        self._init_weights()

    def _init_weights(self) -> None:
        for emb in (self.neuron_emb, self.time_emb, self.value_emb):
            nn.init.normal_(emb.weight, std=0.02)

    def forward(self, neuron_ids: torch.Tensor, time_bins: torch.Tensor,
                values: torch.Tensor) -> torch.Tensor:
        """(E,) index tensors -> (E, hidden_dim) tokens (cortex/models/tokenizer.py:56-93)."""
        if not (neuron_ids.shape == time_bins.shape == values.shape):
            raise ValueError(
                f"shape mismatch: neuron_ids={neuron_ids.shape}, "
                f"time_bins={time_bins.shape}, values={values.shape}")
        dev = self.neuron_emb.weight.device
        return fused_tokenizer(self.neuron_emb.weight, self.time_emb.weight,
                               self.value_emb.weight, neuron_ids.to(dev), time_bins.to(dev),
                               values.to(dev))
