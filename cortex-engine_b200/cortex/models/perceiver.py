"""Perceiver encoder (drop-in for ``cortex.models.perceiver``).

Module tree, parameter names and initialisation order are the reference's
(cortex/models/perceiver.py:35-158), so checkpoints and seeded inits are
interchangeable. The forwards are composed from the B200 kernels:

* norms: ``ck_row_norm`` (LayerNorm, eps 1e-5);
* linears: the tcgen05 GEMM (bf16 / INT8 weights) with the residual add or the
  exact-erf GELU fused into its epilogue;
* attention: the tcgen05 attention kernel, reading heads straight out of the
  packed projection outputs (no rearrange copies) and honouring the token mask.

``CortexModel.forward`` does not use these module forwards; it runs the whole
graph through ``ck_forward``. These are for callers that use the blocks alone.
"""

from __future__ import annotations

import torch
from torch import nn

from cortex import _lib as L
from cortex.kernels import _ops
from cortex.models.config import CortexConfig

def _layer_norm(x: torch.Tensor, ln: nn.LayerNorm) -> torch.Tensor:
    return _ops.row_norm(x, ln.weight, ln.bias, ln.eps, L.CK_NORM_LAYER)


def _linear(module: nn.Module, x: torch.Tensor, epi: int = L.CK_EPI_STORE,
            aux: torch.Tensor | None = None) -> torch.Tensor:
    """Run ``nn.Linear`` or ``QuantizedLinear`` weights through the B200 GEMM.

    Bias (only ``MaskedSpikeHead.proj`` has one on this model) is applied with
    the BIAS epilogue; it cannot be combined with another epilogue."""
    from cortex.quantization.calibrate import QuantizedLinear

    if isinstance(module, QuantizedLinear):
        w, sc, bias = module.weight_int8, module.weight_scale, module.bias
    elif isinstance(module, nn.Linear):
        w, sc, bias = module.weight, None, module.bias
    else:
        raise TypeError(f"unsupported linear module {type(module)}")
    if bias is not None:
        if epi != L.CK_EPI_STORE:
            raise NotImplementedError("bias together with a fused epilogue")
        return _ops.linear(x, w, w_scale=sc, epi=L.CK_EPI_BIAS, aux=bias.to(x.dtype))
    return _ops.linear(x, w, w_scale=sc, epi=epi, aux=aux)


class CrossAttentionBlock(nn.Module):
    """Cross-attention from input tokens into the latent array (perceiver.py:35-82)."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.config = config
        self.num_heads = config.cross_attn_heads
        self.head_dim = config.latent_dim // config.cross_attn_heads
        if self.head_dim * self.num_heads != config.latent_dim:
            raise ValueError("latent_dim must be divisible by cross_attn_heads")
        self.q_proj = nn.Linear(config.latent_dim, config.latent_dim, bias=False)
        self.kv_proj = nn.Linear(config.hidden_dim, 2 * config.latent_dim, bias=False)
        self.out_proj = nn.Linear(config.latent_dim, config.latent_dim, bias=False)
        self.norm_q = nn.LayerNorm(config.latent_dim)
        self.norm_kv = nn.LayerNorm(config.hidden_dim)

    def forward(self, latents: torch.Tensor, tokens: torch.Tensor,
                token_mask: torch.Tensor | None = None) -> torch.Tensor:
        """latents (B, L, D), tokens (B, E, D_hid), token_mask (B, E) bool -> (B, L, D)."""
        B, Lq, D = latents.shape
        E = tokens.shape[1]
        latents = latents.contiguous()
        q = _linear(self.q_proj, _layer_norm(latents, self.norm_q)).reshape(B * Lq, D)
        kv = _linear(self.kv_proj, _layer_norm(tokens.contiguous(), self.norm_kv)).reshape(B * E, 2 * D)
        att = torch.empty(B * Lq, D, dtype=latents.dtype, device=latents.device)
        km = None
        if token_mask is not None:
            km = token_mask.to(device=latents.device, dtype=torch.uint8).contiguous()
        if E == 0:
            att.zero_()
        else:
            _ops.attention(
                q, kv, kv[:, D:], B=B, H=self.num_heads, Dh=self.head_dim, Lq=Lq, n_keys=E,
                q_geom=(D, B * Lq, Lq, 0, self.head_dim),
                k_geom=(2 * D, B * E, E, 0, self.head_dim),
                v_geom=(2 * D, B * E, E, 0, self.head_dim),
                o=att, o_geom=(D, Lq, 0, self.head_dim), key_mask=km,
                scale=self.head_dim ** -0.5)
        out = _linear(self.out_proj, att, L.CK_EPI_RESID, aux=latents.reshape(B * Lq, D))
        return out.reshape(B, Lq, D)


class SelfAttentionBlock(nn.Module):
    """Self-attention within the latent array (perceiver.py:85-126)."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.config = config
        self.num_heads = config.num_heads
        self.head_dim = config.head_dim
        self.qkv_proj = nn.Linear(config.latent_dim, 3 * config.latent_dim, bias=False)
        self.out_proj = nn.Linear(config.latent_dim, config.latent_dim, bias=False)
        self.norm_attn = nn.LayerNorm(config.latent_dim)
        self.norm_mlp = nn.LayerNorm(config.latent_dim)
        mlp_hidden = int(config.latent_dim * config.mlp_ratio)
        self.mlp = nn.Sequential(
            nn.Linear(config.latent_dim, mlp_hidden, bias=False),
            nn.GELU(),
            nn.Linear(mlp_hidden, config.latent_dim, bias=False),
        )

    def forward(self, latents: torch.Tensor) -> torch.Tensor:
        B, Lq, D = latents.shape
        lat = latents.contiguous().reshape(B * Lq, D)
        qkv = _linear(self.qkv_proj, _layer_norm(lat, self.norm_attn))
        att = torch.empty(B * Lq, D, dtype=lat.dtype, device=lat.device)
        _ops.attention(
            qkv, qkv[:, D:], qkv[:, 2 * D:], B=B, H=self.num_heads, Dh=self.head_dim, Lq=Lq,
            n_keys=Lq,
            q_geom=(3 * D, B * Lq, Lq, 0, self.head_dim),
            k_geom=(3 * D, B * Lq, Lq, 0, self.head_dim),
            v_geom=(3 * D, B * Lq, Lq, 0, self.head_dim),
            o=att, o_geom=(D, Lq, 0, self.head_dim), scale=self.head_dim ** -0.5)
        lat = _linear(self.out_proj, att, L.CK_EPI_RESID, aux=lat)
        h = _linear(self.mlp[0], _layer_norm(lat, self.norm_mlp), L.CK_EPI_GELU)
        lat = _linear(self.mlp[2], h, L.CK_EPI_RESID, aux=lat)
        return lat.reshape(B, Lq, D)


class PerceiverEncoder(nn.Module):
    """Cross-attention into latents, then N self-attention blocks (perceiver.py:129-158)."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.config = config
        self.latents = nn.Parameter(torch.randn(config.num_latents, config.latent_dim) * 0.02)
        self.cross_attn = CrossAttentionBlock(config)
        self.self_attn_blocks = nn.ModuleList(
            [SelfAttentionBlock(config) for _ in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.latent_dim)

    def forward(self, tokens: torch.Tensor, token_mask: torch.Tensor | None = None) -> torch.Tensor:
        batch_size = tokens.shape[0]
        latents = self.latents.unsqueeze(0).expand(batch_size, -1, -1)
        latents = self.cross_attn(latents, tokens, token_mask)
        for block in self.self_attn_blocks:
            latents = block(latents)
        return _layer_norm(latents, self.final_norm)
