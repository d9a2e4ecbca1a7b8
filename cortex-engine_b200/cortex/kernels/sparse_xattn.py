"""Block-sparse cross-attention on B200 (drop-in for ``cortex.kernels.sparse_xattn``).

``sparse_cross_attention`` keeps the reference signature, defaults and shape
assertion (cortex/kernels/sparse_xattn.py:340-434). bf16 inputs with head dim
64 run the tcgen05 kernel (TMA-fed Q/K/V tiles, S and O accumulators in TMEM,
online softmax with the running output in registers); every (latent-tile,
event-tile) pair whose ``block_mask`` entry is False is skipped before its keys
are loaded. fp32 inputs (and other head dims) run an fp32 CUDA-core kernel with
the same masking. A query row with no unmasked key returns 0, as the reference
Triton kernel's ``l = 0`` guard does (:326-328). ``block_mask=None`` means
dense attention (the reference calls SDPA there, :374-376); it runs the same
kernels without a mask. CUDA tensors only.

``build_temporal_block_mask`` is the host-side mask builder (:152-200),
vectorised but with identical arithmetic: latent centres ``i / L * T`` in
float32, truncated, widened by ``window_bins``, overlapped with each event
tile's [min, max] time bin. It returns a CPU bool tensor like the reference.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from cortex.kernels import _ops


def sparse_cross_attention_reference(q, k, v, block_mask=None, BLOCK_L: int = 64,
                                     BLOCK_E: int = 64, scale: float | None = None):
    """The reference's eager twin (cortex/kernels/sparse_xattn.py:96-146), kept for
    callers that test against it. No function of this package calls it."""
    _, _, L, Dh = q.shape
    E = k.shape[2]
    s = scale if scale is not None else Dh ** -0.5
    if block_mask is None:
        return F.scaled_dot_product_attention(q, k, v, scale=s)
    n_q, n_k = math.ceil(L / BLOCK_L), math.ceil(E / BLOCK_E)
    assert block_mask.shape == (n_q, n_k), \
        f"block_mask shape {block_mask.shape} != expected ({n_q}, {n_k})"
    dense = block_mask.to(q.device).bool().repeat_interleave(BLOCK_L, 0) \
        .repeat_interleave(BLOCK_E, 1)[:L, :E]
    float_mask = torch.zeros(L, E, device=q.device, dtype=q.dtype).masked_fill(~dense, float("-inf"))
    scores = torch.matmul(q, k.transpose(-2, -1)) * s + float_mask
    attn = torch.softmax(scores.float(), dim=-1).to(q.dtype)
    return torch.matmul(attn, v)


def build_temporal_block_mask(event_times: torch.Tensor, n_latents: int, max_time_bins: int,
                              window_bins: int = 30, BLOCK_L: int = 64,
                              BLOCK_E: int = 64) -> torch.Tensor:
    """(n_q_tiles, n_k_tiles) CPU bool mask: True = compute this tile."""
    t = event_times.detach().to("cpu", torch.int64).reshape(-1)
    E = t.shape[0]
    n_q = math.ceil(n_latents / BLOCK_L)
    n_k = math.ceil(E / BLOCK_E)
    if n_k == 0:
        return torch.zeros(n_q, 0, dtype=torch.bool)
    pad = n_k * BLOCK_E - E
    big = torch.iinfo(torch.int64).max
    tmin = torch.cat([t, torch.full((pad,), big, dtype=torch.int64)]).view(n_k, BLOCK_E).amin(1)
    tmax = torch.cat([t, torch.full((pad,), -big, dtype=torch.int64)]).view(n_k, BLOCK_E).amax(1)
    centres = torch.arange(0, n_latents, dtype=torch.float32) / n_latents * max_time_bins
    cpad = n_q * BLOCK_L - n_latents
    cmin = torch.cat([centres, torch.full((cpad,), float("inf"))]).view(n_q, BLOCK_L).amin(1)
    cmax = torch.cat([centres, torch.full((cpad,), float("-inf"))]).view(n_q, BLOCK_L).amax(1)
    lat_lo = cmin.to(torch.int64) - window_bins  # int() truncates; centres are >= 0
    lat_hi = cmax.to(torch.int64) + window_bins
    return (tmin[None, :] <= lat_hi[:, None]) & (tmax[None, :] >= lat_lo[:, None])


def sparse_cross_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: torch.Tensor | None = None, BLOCK_L: int = 64,
                           BLOCK_E: int = 64, scale: float | None = None) -> torch.Tensor:
    """Block-sparse cross-attention, (B, H, L, Dh) x (B, H, E, Dh) -> (B, H, L, Dh)."""
    B, H, L, Dh = q.shape
    _B, _H, E, _Dh = k.shape
    if (_B, _H, _Dh) != (B, H, Dh) or tuple(v.shape) != tuple(k.shape):
        raise ValueError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, "
                         f"v {tuple(v.shape)}")
    s = scale if scale is not None else Dh ** -0.5
    n_q, n_k = math.ceil(L / BLOCK_L), math.ceil(E / BLOCK_E)
    if block_mask is not None:
        assert tuple(block_mask.shape) == (n_q, n_k), \
            f"block_mask shape {tuple(block_mask.shape)} != expected ({n_q}, {n_k})"
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty_like(q)
    if B == 0 or H == 0 or L == 0:
        return out
    bm = None
    if block_mask is not None:
        bm = block_mask.to(device=q.device, dtype=torch.uint8).contiguous()
    return _ops.attention(
        q, k, v, B=B, H=H, Dh=Dh, Lq=L, n_keys=E,
        q_geom=(Dh, B * H * L, H * L, L, 0),
        k_geom=(Dh, max(B * H * E, 1), H * E, E, 0),
        v_geom=(Dh, max(B * H * E, 1), H * E, E, 0),
        o=out, o_geom=(Dh, H * L, L, 0),
        block_mask=bm, block_l=BLOCK_L, block_e=BLOCK_E, scale=float(s))
