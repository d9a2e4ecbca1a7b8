"""Model configuration for the Cortex decoder (drop-in for ``cortex.models.config``).

The field names, constraints, validator messages and the three presets mirror
the reference's ``CortexConfig`` (cortex/models/config.py:14-103) so that
existing configs, Hydra YAMLs and checkpoints keep working unchanged.

``use_kernels`` is kept for source compatibility (cortex/models/config.py:48).
This package only ships the B200 CUDA path: every forward runs the sm_100a
kernels and raises if a tensor is not on a CUDA device, whatever the flag says.
"""

from __future__ import annotations

from pydantic import BaseModel, Field, model_validator


class CortexConfig(BaseModel):
    """Configuration for the Cortex model family (cortex/models/config.py:14-61)."""

    hidden_dim: int = Field(..., gt=0, description="Embedding/hidden dimension")
    num_layers: int = Field(..., gt=0, description="Number of transformer layers")
    num_heads: int = Field(..., gt=0, description="Number of attention heads")
    head_dim: int = Field(..., gt=0, description="Per-head dimension")
    mlp_ratio: float = Field(4.0, gt=0, description="MLP hidden = mlp_ratio * hidden_dim")
    dropout: float = Field(0.0, ge=0, lt=1)

    num_latents: int = Field(..., gt=0, description="Size of latent array")
    latent_dim: int = Field(..., gt=0, description="Latent array hidden dimension")
    cross_attn_heads: int = Field(..., gt=0)

    max_neurons: int = Field(..., gt=0, description="Max neuron index across all sessions")
    max_time_bins: int = Field(..., gt=0, description="Max time bin index per window")
    spike_value_buckets: int = Field(8, gt=0, description="Quantization buckets for spike count")

    behavior_dim: int = Field(..., gt=0, description="Output dim of behavior decoder")
    use_masked_spike_head: bool = True

    dtype: str = Field("bfloat16", pattern="^(float32|float16|bfloat16)$")

    use_kernels: bool = False

    @model_validator(mode="after")
    def _check_head_consistency(self) -> CortexConfig:
        if self.hidden_dim % self.num_heads != 0:
            raise ValueError(
                f"hidden_dim ({self.hidden_dim}) must be divisible by num_heads ({self.num_heads})"
            )
        if self.head_dim * self.num_heads != self.hidden_dim:
            raise ValueError(
                f"head_dim ({self.head_dim}) * num_heads ({self.num_heads}) "
                f"must equal hidden_dim ({self.hidden_dim})"
            )
        return self


CORTEX_XS = CortexConfig(
    hidden_dim=256,
    num_layers=5,
    num_heads=4,
    head_dim=64,
    num_latents=128,
    latent_dim=256,
    cross_attn_heads=4,
    max_neurons=512,
    max_time_bins=1024,
    behavior_dim=2,
)

CORTEX_S = CortexConfig(
    hidden_dim=512,
    num_layers=7,
    num_heads=8,
    head_dim=64,
    num_latents=256,
    latent_dim=512,
    cross_attn_heads=8,
    max_neurons=512,
    max_time_bins=1024,
    behavior_dim=2,
)

CORTEX_M = CortexConfig(
    hidden_dim=768,
    num_layers=11,
    num_heads=12,
    head_dim=64,
    num_latents=384,
    latent_dim=768,
    cross_attn_heads=12,
    max_neurons=512,
    max_time_bins=1024,
    behavior_dim=2,
)
