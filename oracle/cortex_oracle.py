"""CPU oracle for the Cortex decoder forward hot path.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA path is
compared against; it is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``. The product (``cortex-engine_b200/``) never imports it.

It restates, on the host, the reference algorithm of peterajhgraham/cortex-engine
for every function on the path. Integer work (event packing) is plain numpy;
floating-point work uses the same torch CPU operators the reference composes
(``nn.Embedding`` gather, ``F.layer_norm``, ``F.linear``,
``F.scaled_dot_product_attention``, exact-erf GELU), in the same order and at the
same rounding points, operating on a plain ``state_dict`` so that nothing of the
product's module code is involved. Each function cites the reference lines it
follows.

Parity is pinned by ``tests/test_oracle_golden.py`` against golden vectors that
``tests/golden/make_golden.py`` produced by importing and running the reference
itself in the build container.
"""

from __future__ import annotations

import math
from typing import Mapping

import numpy as np
import torch
import torch.nn.functional as F

LN_EPS = 1e-5  # nn.LayerNorm default, used by every norm in the model


# ── Event packing (cortex/models/cortex.py:125-165) ──────────────────────────


def pack_events_index(batch_indices: np.ndarray) -> dict[str, np.ndarray | int]:
    """Index-side restatement of ``_pack_events``.

    Returns ``B`` (= max(bidx)+1, or 1 when empty; cortex/models/cortex.py:140),
    ``counts`` (bincount with minlength B; :141), ``E_max`` (:142), ``offsets``
    (exclusive cumsum, length B+1; the reference's ``cum`` at :155-160 plus the
    total), ``order`` (the stable argsort, :149) and ``dest`` (the flat packed
    row, ``offsets[b] + pos_within`` for every input event, :161).
    """
    bidx = np.asarray(batch_indices, dtype=np.int64)
    E = bidx.shape[0]
    B = int(bidx.max()) + 1 if E > 0 else 1
    counts = np.bincount(bidx, minlength=B).astype(np.int64)
    e_max = int(counts.max()) if counts.size > 0 else 0
    offsets = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    order = np.argsort(bidx, kind="stable")
    sorted_b = bidx[order]
    pos_within = np.arange(E, dtype=np.int64) - offsets[sorted_b]
    dest = np.empty(E, dtype=np.int64)
    dest[order] = offsets[sorted_b] + pos_within
    return {"B": B, "counts": counts, "E_max": e_max, "offsets": offsets,
            "order": order, "dest": dest, "pos_within_sorted": pos_within}


def pack_events(flat_tokens: torch.Tensor, batch_indices: torch.Tensor
                ) -> tuple[torch.Tensor, torch.Tensor]:
    """Padded ``(B, E_max, D)`` tokens and ``(B, E_max)`` bool mask
    (cortex/models/cortex.py:143-165)."""
    info = pack_events_index(batch_indices.cpu().numpy())
    B, e_max = info["B"], info["E_max"]
    D = flat_tokens.shape[-1]
    out = torch.zeros(B, e_max, D, dtype=flat_tokens.dtype)
    mask = torch.zeros(B, e_max, dtype=torch.bool)
    order = torch.from_numpy(info["order"])
    sb = batch_indices.cpu()[order]
    pw = torch.from_numpy(info["pos_within_sorted"])
    out[sb, pw] = flat_tokens.cpu()[order]
    mask[sb, pw] = True
    return out, mask


def tile_mask(counts: np.ndarray, e_max: int, block_e: int) -> np.ndarray:
    """Per-sample event-tile occupancy: ``mask.view(B, n_k, BLOCK_E).any(-1)``
    after padding ``E_max`` up to a multiple of ``BLOCK_E``."""
    B = counts.shape[0]
    n_k = (e_max + block_e - 1) // block_e
    t = np.arange(n_k, dtype=np.int64)[None, :] * block_e
    return (t < counts[:, None]).reshape(B, n_k)


# ── Tokenizer (cortex/kernels/tokenizer.py:68-81, cortex/models/tokenizer.py:90-93) ──


def tokenize(n_emb: torch.Tensor, t_emb: torch.Tensor, v_emb: torch.Tensor,
             nid: torch.Tensor, tb: torch.Tensor, val: torch.Tensor) -> torch.Tensor:
    """``n_emb[nid] + t_emb[tb] + v_emb[val]`` evaluated left to right, so that a
    bf16 table gives ``bf16(bf16(n + t) + v)``."""
    return n_emb[nid] + t_emb[tb] + v_emb[val]


# ── Norms and linears ───────────────────────────────────────────────────────


def layer_norm(x: torch.Tensor, p: Mapping[str, torch.Tensor], prefix: str) -> torch.Tensor:
    """``nn.LayerNorm(D)`` with eps 1e-5 (cortex/models/perceiver.py:51-52,97-98,143)."""
    return F.layer_norm(x, (x.shape[-1],), p[prefix + ".weight"], p[prefix + ".bias"], LN_EPS)


def linear(x: torch.Tensor, p: Mapping[str, torch.Tensor], prefix: str) -> torch.Tensor:
    """Bias-free ``nn.Linear`` or ``QuantizedLinear`` (dequantize then ``F.linear``,
    cortex/quantization/calibrate.py:225-228)."""
    if prefix + ".weight_int8" in p:
        w_dq = p[prefix + ".weight_int8"].float() * p[prefix + ".weight_scale"][:, None]
        bias = p.get(prefix + ".bias")
        return F.linear(x, w_dq.to(x.dtype), bias)
    return F.linear(x, p[prefix + ".weight"], p.get(prefix + ".bias"))


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric INT8: ``scale = absmax_row/127`` (min 1e-8),
    ``w_int8 = round(w/scale).clamp(-127, 127)`` (cortex/quantization/calibrate.py:154,
    205-211)."""
    wf = w.detach().float()
    scale = wf.abs().amax(dim=1).clamp(min=1e-8) / 127.0
    w8 = (wf / scale[:, None]).round().clamp(-127, 127).to(torch.int8)
    return w8, scale


def rms_norm_linear(x: torch.Tensor, gamma: torch.Tensor, w: torch.Tensor,
                    bias: torch.Tensor | None, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm then ``@ w`` with ``w`` shaped (K, N) (cortex/kernels/fused_rmsnorm.py:86-108)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    xf = x2.float()
    rms = torch.sqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    xn = (xf / rms) * gamma.float()
    out = xn.to(x.dtype) @ w
    if bias is not None:
        out = out + bias
    return out.reshape(*lead, w.shape[1])


# ── Attention ───────────────────────────────────────────────────────────────


def _heads(t: torch.Tensor, h: int) -> torch.Tensor:
    b, n, d = t.shape
    return t.reshape(b, n, h, d // h).transpose(1, 2)


def _merge(t: torch.Tensor) -> torch.Tensor:
    b, h, n, dh = t.shape
    return t.transpose(1, 2).reshape(b, n, h * dh)


def cross_attention_block(p: Mapping[str, torch.Tensor], prefix: str, latents: torch.Tensor,
                          tokens: torch.Tensor, mask: torch.Tensor | None, heads: int
                          ) -> torch.Tensor:
    """cortex/models/perceiver.py:54-82."""
    q = linear(layer_norm(latents, p, prefix + ".norm_q"), p, prefix + ".q_proj")
    kv = linear(layer_norm(tokens, p, prefix + ".norm_kv"), p, prefix + ".kv_proj")
    k, v = kv.chunk(2, dim=-1)
    am = mask[:, None, None, :] if mask is not None else None
    o = F.scaled_dot_product_attention(_heads(q, heads), _heads(k, heads), _heads(v, heads),
                                       attn_mask=am)
    return latents + linear(_merge(o), p, prefix + ".out_proj")


def self_attention_block(p: Mapping[str, torch.Tensor], prefix: str, latents: torch.Tensor,
                         heads: int) -> torch.Tensor:
    """cortex/models/perceiver.py:107-126 (GELU is exact erf, :102)."""
    x = layer_norm(latents, p, prefix + ".norm_attn")
    qkv = linear(x, p, prefix + ".qkv_proj")
    q, k, v = qkv.chunk(3, dim=-1)
    o = F.scaled_dot_product_attention(_heads(q, heads), _heads(k, heads), _heads(v, heads))
    latents = latents + linear(_merge(o), p, prefix + ".out_proj")
    h = F.gelu(linear(layer_norm(latents, p, prefix + ".norm_mlp"), p, prefix + ".mlp.0"))
    return latents + linear(h, p, prefix + ".mlp.2")


def behavior_head(p: Mapping[str, torch.Tensor], latents: torch.Tensor, heads: int
                  ) -> torch.Tensor:
    """cortex/models/cortex.py:29-53: LN, learned queries, kv_proj, SDPA, out_proj."""
    x = layer_norm(latents, p, "behavior_head.norm")
    B = x.shape[0]
    query = p["behavior_head.query"].unsqueeze(0).expand(B, -1, -1)
    q = linear(query, p, "behavior_head.q_proj")
    kv = linear(x, p, "behavior_head.kv_proj")
    k, v = kv.chunk(2, dim=-1)
    o = F.scaled_dot_product_attention(_heads(q, heads), _heads(k, heads), _heads(v, heads))
    return linear(_merge(o), p, "behavior_head.out_proj").squeeze(-1)


def forward(p: Mapping[str, torch.Tensor], cfg, neuron_ids: torch.Tensor,
            time_bins: torch.Tensor, values: torch.Tensor, batch_indices: torch.Tensor,
            return_intermediates: bool = False):
    """``CortexModel.forward`` (cortex/models/cortex.py:90-122) on a state_dict.

    Runs in the dtype of the floating-point parameters (fp32, or bf16 after
    ``.to(torch.bfloat16)``). Returns ``(B, behavior_dim)``.
    """
    with torch.no_grad():
        flat = tokenize(p["tokenizer.neuron_emb.weight"], p["tokenizer.time_emb.weight"],
                        p["tokenizer.value_emb.weight"], neuron_ids, time_bins, values)
        tokens, mask = pack_events(flat, batch_indices)
        B = tokens.shape[0]
        lat = p["encoder.latents"].unsqueeze(0).expand(B, -1, -1)
        lat = cross_attention_block(p, "encoder.cross_attn", lat, tokens, mask,
                                    cfg.cross_attn_heads)
        inter = {"tokens": flat, "after_cross": lat}
        for i in range(cfg.num_layers):
            lat = self_attention_block(p, f"encoder.self_attn_blocks.{i}", lat, cfg.num_heads)
        inter["after_sa"] = lat
        lat = layer_norm(lat, p, "encoder.final_norm")
        inter["latents"] = lat
        out = behavior_head(p, lat, cfg.num_heads)
    if return_intermediates:
        return out, inter
    return out


# ── Kernel-level APIs (cortex/kernels/sparse_xattn.py) ────────────────────────


def sparse_cross_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: torch.Tensor | None = None, BLOCK_L: int = 64,
                           BLOCK_E: int = 64, scale: float | None = None) -> torch.Tensor:
    """Dense attention with tile-level masking (cortex/kernels/sparse_xattn.py:96-146).

    Differs from the reference's own CPU twin in one place, on purpose: a query
    row whose every tile is masked returns 0 (the reference Triton kernel's
    ``l = 0`` guard, cortex/kernels/sparse_xattn.py:326-328), where the twin
    returns NaN from ``softmax`` over all ``-inf``.
    """
    L, Dh = q.shape[-2], q.shape[-1]
    E = k.shape[-2]
    s = scale if scale is not None else Dh ** -0.5
    if block_mask is None:
        return F.scaled_dot_product_attention(q, k, v, scale=s)
    n_q, n_k = math.ceil(L / BLOCK_L), math.ceil(E / BLOCK_E)
    assert tuple(block_mask.shape) == (n_q, n_k)
    dense = block_mask.bool().repeat_interleave(BLOCK_L, 0).repeat_interleave(BLOCK_E, 1)[:L, :E]
    scores = torch.matmul(q.float(), k.float().transpose(-2, -1)) * s
    scores = scores.masked_fill(~dense, float("-inf"))
    m = scores.amax(dim=-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    e = torch.exp(scores - m)
    den = e.sum(dim=-1, keepdim=True)
    pr = torch.where(den > 0, e / den.clamp_min(1e-30), torch.zeros_like(e))
    return torch.matmul(pr, v.float()).to(q.dtype)


def build_temporal_block_mask(event_times: torch.Tensor, n_latents: int, max_time_bins: int,
                              window_bins: int = 30, BLOCK_L: int = 64, BLOCK_E: int = 64
                              ) -> torch.Tensor:
    """Coarse temporal tile mask (cortex/kernels/sparse_xattn.py:152-200).

    Latent ``i`` sits at time ``i / L * T`` (float32); latent tile ``qi`` spans
    ``[int(min centre) - w, int(max centre) + w]``; event tile ``kj`` spans the
    min..max time bin of its events; the mask is their interval overlap.
    """
    t = np.asarray(event_times.cpu().numpy(), dtype=np.int64)
    E = t.shape[0]
    n_q, n_k = math.ceil(n_latents / BLOCK_L), math.ceil(E / BLOCK_E)
    tmin = np.array([t[j * BLOCK_E:min((j + 1) * BLOCK_E, E)].min() for j in range(n_k)],
                    dtype=np.int64)
    tmax = np.array([t[j * BLOCK_E:min((j + 1) * BLOCK_E, E)].max() for j in range(n_k)],
                    dtype=np.int64)
    mask = np.zeros((n_q, n_k), dtype=bool)
    for qi in range(n_q):
        l0, l1 = qi * BLOCK_L, min((qi + 1) * BLOCK_L, n_latents)
        centres = np.arange(l0, l1, dtype=np.float32) / np.float32(n_latents) \
            * np.float32(max_time_bins)
        lo = int(centres.min()) - window_bins
        hi = int(centres.max()) + window_bins
        mask[qi] = (tmin <= hi) & (tmax >= lo)
    return torch.from_numpy(mask)
