"""Top-level Cortex model on B200 (drop-in for ``cortex.models.cortex``).

``CortexModel`` has the reference's module tree, parameter names, initialisation
order and ``forward`` signature (cortex/models/cortex.py:72-122). With
``return_aux=False`` -- the inference hot path -- ``forward`` hands the whole
graph to ``ck_forward``: packing, tokenizer with the fused norm_kv, batch-
invariant latent queries, packed varlen cross-attention, the self-attention
stack and the behaviour head, launched back to back on the current stream with
no host synchronisation inside. Index tensors may be on the device, or on
the host: then they go through ``cortex.batching`` -- one packed int32 batch in
pinned memory, one copy to the device and the replay of a CUDA graph captured
for the batch's (B, event-capacity) bucket.

``_pack_events`` keeps the reference's padded-output contract
(cortex/models/cortex.py:125-165) on top of the device packing kernels.
"""

from __future__ import annotations

import ctypes
import operator
import threading
from typing import cast

import torch
from torch import nn

from cortex import _lib as L
from cortex.kernels import _ops
from cortex.models.config import CortexConfig
from cortex.models.perceiver import PerceiverEncoder, _layer_norm, _linear
from cortex.models.tokenizer import SpikeTokenizer


# Counts module / parameter / buffer registrations in the process (torch's
# global registration hooks): while it is unchanged, no submodule swap or
# parameter assignment can have happened, and a cached weight description
# skips its slot-by-slot identity check.
_REGISTRATIONS = [0]


def _registered(*_args) -> None:
    _REGISTRATIONS[0] += 1


torch.nn.modules.module.register_module_module_registration_hook(_registered)
torch.nn.modules.module.register_module_parameter_registration_hook(_registered)
torch.nn.modules.module.register_module_buffer_registration_hook(_registered)


class BehaviorDecoder(nn.Module):
    """Decode behaviour from the latent array (cortex/models/cortex.py:15-53)."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.query = nn.Parameter(torch.randn(config.behavior_dim, config.latent_dim) * 0.02)
        self.q_proj = nn.Linear(config.latent_dim, config.latent_dim, bias=False)
        self.kv_proj = nn.Linear(config.latent_dim, 2 * config.latent_dim, bias=False)
        self.out_proj = nn.Linear(config.latent_dim, 1, bias=False)
        self.norm = nn.LayerNorm(config.latent_dim)
        self.num_heads = config.num_heads
        self.head_dim = config.head_dim

    def forward(self, latents: torch.Tensor) -> torch.Tensor:
        """latents (B, L, D) -> (B, behavior_dim)."""
        B, Lk, D = latents.shape
        nq = self.query.shape[0]
        x = _layer_norm(latents.contiguous(), self.norm).reshape(B * Lk, D)
        q = _linear(self.q_proj, self.query)  # batch-invariant: once, not per sample
        kv = _linear(self.kv_proj, x)
        o = torch.empty(B * nq, D, dtype=latents.dtype, device=latents.device)
        _ops.attention(
            q, kv, kv[:, D:], B=B, H=self.num_heads, Dh=self.head_dim, Lq=nq, n_keys=Lk,
            q_geom=(D, nq, 0, 0, self.head_dim),
            k_geom=(2 * D, B * Lk, Lk, 0, self.head_dim),
            v_geom=(2 * D, B * Lk, Lk, 0, self.head_dim),
            o=o, o_geom=(D, nq, 0, self.head_dim), scale=self.head_dim ** -0.5)
        return _linear(self.out_proj, o).reshape(B, nq)


class MaskedSpikeHead(nn.Module):
    """Self-supervised head (cortex/models/cortex.py:56-69); training-only, off the
    inference hot path. Its projection runs on the B200 GEMM with a bias epilogue."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.proj = nn.Linear(config.latent_dim, config.spike_value_buckets)

    def forward(self, latents: torch.Tensor) -> torch.Tensor:
        return _linear(self.proj, latents.mean(dim=1))


class CortexModel(nn.Module):
    """Cortex: tokenizer -> Perceiver encoder -> behaviour head."""

    def __init__(self, config: CortexConfig) -> None:
        super().__init__()
        self.config = config
        self.tokenizer = SpikeTokenizer(config)
        self.encoder = PerceiverEncoder(config)
        self.behavior_head = BehaviorDecoder(config)
        self.masked_spike_head = MaskedSpikeHead(config) if config.use_masked_spike_head else None
        self._native_lock = threading.Lock()
        self._native_key = None
        self._native_epoch = -1
        self._native = None
        self._workspace: dict[torch.device, torch.Tensor] = {}
        self._batch_runner = None

    # ── native graph description ────────────────────────────────────────────

    def _lw(self, module: nn.Module, keep: list) -> L.LinearWeight:
        from cortex.quantization.calibrate import QuantizedLinear

        lw = L.LinearWeight()
        if isinstance(module, QuantizedLinear):
            sc = module.weight_scale
            if sc.dtype != torch.float32 or not sc.is_contiguous():
                sc = sc.float().contiguous()
            keep.append(sc.detach())
            w = module.weight_int8.contiguous()
            keep.append(w.detach())
            lw.w, lw.dtype, lw.scale = w.data_ptr(), L.CK_I8, sc.data_ptr()
            if module.bias is not None:
                raise NotImplementedError("biased linears are not on the Cortex hot path")
        else:
            w = module.weight.contiguous()
            keep.append(w.detach())
            lw.w, lw.dtype, lw.scale = w.data_ptr(), L.dtype_code(w.dtype), None
            if module.bias is not None:
                raise NotImplementedError("biased linears are not on the Cortex hot path")
        lw.bias = None
        return lw

    def _apply(self, fn, *args, **kwargs):
        self._native = None  # .to() / .cuda() / .bfloat16() move or recast the weights
        return super()._apply(fn, *args, **kwargs)

    def load_state_dict(self, *args, **kwargs):
        self._native = None
        return super().load_state_dict(*args, **kwargs)

    def _state_key(self):
        # Weight pointers only change through _apply / load_state_dict (both
        # invalidate the cache), by swapping submodules (convert_model) or by
        # assigning new Parameters. The key is every (child dict, name) slot of
        # the module tree with the identity of what it held at build time;
        # checking it is one C-level pass (map) instead of a module walk.
        dicts, names, objs = [], [], []
        for mod in self.modules():
            for d in (mod._modules, mod._parameters, mod._buffers):
                for n, c in d.items():
                    dicts.append(d)
                    names.append(n)
                    objs.append(c)  # held, so no later object can reuse its identity
        return dicts, names, objs

    def _state_unchanged(self) -> bool:
        if self._native_epoch == _REGISTRATIONS[0]:
            return True  # no module, parameter or buffer registered anywhere since the check
        key = self._native_key
        same = key is not None and all(map(operator.is_, map(dict.get, key[0], key[1]), key[2]))
        if same:
            self._native_epoch = _REGISTRATIONS[0]
        return same

    def native_model(self) -> L.Model:
        """The ``ck_model`` description of this module's weights (cached).

        The description holds raw device pointers of the parameters; in-place
        updates of parameter values are seen by the next forward as they are."""
        with self._native_lock:
            if self._native is not None and self._state_unchanged():
                return self._native[0]
            key = self._state_key()
            keep: list = []
            cfg = self.config
            tok, enc, head = self.tokenizer, self.encoder, self.behavior_head
            dt = tok.neuron_emb.weight.dtype
            L.require_cuda(tok.neuron_emb.weight, what="CortexModel")

            def t(x: torch.Tensor | None):
                if x is None:
                    return None
                if x.dtype != dt:
                    raise TypeError(f"parameter dtype {x.dtype} differs from the model dtype {dt}")
                x = x.contiguous()
                keep.append(x.detach())  # the storage itself, even if .data is reassigned
                return x.data_ptr()

            m = L.Model()
            m.dtype = L.dtype_code(dt)
            if m.dtype not in (L.CK_BF16, L.CK_F32):
                raise NotImplementedError(f"model dtype {dt}: the B200 path runs bf16 or fp32")
            m.hidden_dim, m.latent_dim = cfg.hidden_dim, cfg.latent_dim
            m.num_latents, m.num_layers = cfg.num_latents, cfg.num_layers
            m.num_heads, m.head_dim = cfg.num_heads, cfg.head_dim
            m.cross_heads = cfg.cross_attn_heads
            m.mlp_hidden = int(cfg.latent_dim * cfg.mlp_ratio)
            m.behavior_dim = cfg.behavior_dim
            m.n_vocab, m.t_vocab, m.v_vocab = (tok.neuron_emb.weight.shape[0],
                                               tok.time_emb.weight.shape[0],
                                               tok.value_emb.weight.shape[0])
            m.neuron_emb = t(tok.neuron_emb.weight)
            m.time_emb = t(tok.time_emb.weight)
            m.value_emb = t(tok.value_emb.weight)
            m.latents = t(enc.latents)
            ca = enc.cross_attn
            m.norm_q_w, m.norm_q_b = t(ca.norm_q.weight), t(ca.norm_q.bias)
            m.norm_kv_w, m.norm_kv_b = t(ca.norm_kv.weight), t(ca.norm_kv.bias)
            m.cross_q, m.cross_kv, m.cross_out = (self._lw(ca.q_proj, keep),
                                                  self._lw(ca.kv_proj, keep),
                                                  self._lw(ca.out_proj, keep))
            blocks = (L.BlockWeights * max(cfg.num_layers, 1))()
            for i, blk in enumerate(enc.self_attn_blocks):
                if not (isinstance(blk.mlp[1], nn.GELU) and blk.mlp[1].approximate == "none"):
                    raise NotImplementedError("the fused MLP epilogue implements exact-erf GELU")
                b = blocks[i]
                b.norm_attn_w, b.norm_attn_b = t(blk.norm_attn.weight), t(blk.norm_attn.bias)
                b.qkv, b.out = self._lw(blk.qkv_proj, keep), self._lw(blk.out_proj, keep)
                b.norm_mlp_w, b.norm_mlp_b = t(blk.norm_mlp.weight), t(blk.norm_mlp.bias)
                b.mlp0, b.mlp2 = self._lw(blk.mlp[0], keep), self._lw(blk.mlp[2], keep)
            keep.append(blocks)
            m.blocks = ctypes.cast(blocks, ctypes.POINTER(L.BlockWeights))
            m.final_norm_w, m.final_norm_b = t(enc.final_norm.weight), t(enc.final_norm.bias)
            m.head_query = t(head.query)
            m.head_norm_w, m.head_norm_b = t(head.norm.weight), t(head.norm.bias)
            m.head_q, m.head_kv, m.head_out = (self._lw(head.q_proj, keep),
                                               self._lw(head.kv_proj, keep),
                                               self._lw(head.out_proj, keep))
            self._native = (m, keep, None, tok.neuron_emb.weight.device, dt)
            self._native_key = key
            self._native_epoch = _REGISTRATIONS[0]
            return m

    def native_info(self) -> tuple:
        """(native description, weight device, weight dtype), from the cache when
        the module tree is unchanged."""
        self.native_model()
        n = self._native
        return n[0], n[3], n[4]

    def invalidate_native(self) -> None:
        """Drop the cached weight description."""
        self._native = None

    def forward_packed(self, packed) -> dict[str, torch.Tensor]:
        """``{"behavior": (B, behavior_dim)}`` for a ``cortex.data.PackedBatch``
        already on the device (``collate_windows``): the batch's events never
        leave HBM; one device copy and a graph replay of its bucket."""
        return {"behavior": self.batch_runner().forward_batch(packed.batch, packed.capacity,
                                                              packed.batch_size)}

    def forward_streaming(self, windows: list[dict], cache) -> dict[str, torch.Tensor]:
        """``{"behavior": (B, behavior_dim)}`` for windows keyed by (session_id,
        bin_start), reusing the kv_proj rows of windows held in ``cache`` (a
        ``cortex.cache.StreamingKVCache`` of (2 * latent_dim,) rows) and caching
        those of the others. Same result as ``forward`` on the same events."""
        from cortex.cache.kv_forward import forward_with_kv_cache

        return {"behavior": forward_with_kv_cache(self, windows, cache)}

    def batch_runner(self):
        """The packed-batch runner host-index forwards go through (cortex.batching)."""
        if self._batch_runner is None:
            from cortex.batching import BatchRunner

            self._batch_runner = BatchRunner(self)
        return self._batch_runner

    def workspace(self, device: torch.device, nbytes: int) -> torch.Tensor:
        ws = self._workspace.get(device)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
            self._workspace[device] = ws
        return ws

    # ── forward ─────────────────────────────────────────────────────────────

    def forward(self, neuron_ids: torch.Tensor, time_bins: torch.Tensor, values: torch.Tensor,
                batch_indices: torch.Tensor, return_aux: bool = False,
                batch_size: int | None = None) -> dict[str, torch.Tensor]:
        """Args (cortex/models/cortex.py:90-108):
            neuron_ids, time_bins, values, batch_indices: (E,) int64 (or int32), on the
                host or on the model's CUDA device.
            return_aux: also return ``masked_spike_logits`` (composed module path).
            batch_size: optional B; when omitted, B = max(batch_indices) + 1 as in the
                reference (one device read if batch_indices is on the device).

        Returns:
            {"behavior": (B, behavior_dim)} in the model dtype, on the model's device.
        """
        if not (neuron_ids.shape == time_bins.shape == values.shape == batch_indices.shape):
            raise ValueError(
                f"shape mismatch: neuron_ids={neuron_ids.shape}, time_bins={time_bins.shape}, "
                f"values={values.shape}, batch_indices={batch_indices.shape}")
        if not return_aux and (neuron_ids.is_cpu and time_bins.is_cpu and values.is_cpu
                               and batch_indices.is_cpu):
            # host indices: one packed int32 batch, one copy, one graph replay (the
            # weights' device is checked by the cached native description)
            return {"behavior": self.batch_runner().forward_host(
                neuron_ids, time_bins, values, batch_indices, batch_size)}
        dev = self.tokenizer.neuron_emb.weight.device
        L.require_cuda(self.tokenizer.neuron_emb.weight, what="CortexModel.forward")
        E = int(batch_indices.shape[0])
        if batch_size is None:
            batch_size = int(batch_indices.max().item()) + 1 if E > 0 else 1

        idx = [neuron_ids, time_bins, values, batch_indices]
        dt = idx[0].dtype if all(x.dtype == idx[0].dtype for x in idx) else torch.int64
        if dt not in (torch.int64, torch.int32):
            dt = torch.int64
        idx = [x.to(device=dev, dtype=dt, non_blocking=True).contiguous() for x in idx]

        if return_aux:
            return self._forward_modules(*idx, batch_size=batch_size)

        m = self.native_model()
        lib = L.load()
        nbytes = lib.ck_forward_workspace_bytes(ctypes.byref(m), E, batch_size)
        ws = self.workspace(dev, nbytes)
        out = torch.empty(batch_size, self.config.behavior_dim,
                          dtype=self.tokenizer.neuron_emb.weight.dtype, device=dev)
        rc = lib.ck_forward(ctypes.byref(m), idx[0].data_ptr(), idx[1].data_ptr(),
                            idx[2].data_ptr(), idx[3].data_ptr(),
                            L.CK_I64 if dt == torch.int64 else L.CK_I32, E, batch_size,
                            out.data_ptr(), ws.data_ptr(), ws.numel(), L.stream_of(dev))
        L.check(rc, "ck_forward")
        return {"behavior": out}

    def _forward_modules(self, nid, tb, val, bidx, batch_size):
        flat = self.tokenizer(nid, tb, val)
        tokens, mask = _pack_events(flat, bidx, batch_size=batch_size)
        latents = self.encoder(tokens, mask)
        out: dict[str, torch.Tensor] = {"behavior": self.behavior_head(latents)}
        if self.masked_spike_head is not None:
            out["masked_spike_logits"] = self.masked_spike_head(latents)
        return out


def _pack_events(flat_tokens: torch.Tensor, batch_indices: torch.Tensor,
                 batch_size: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Pack flat (E, D) tokens into (B, E_max, D) with a (B, E_max) bool mask.

    Same result as the reference (cortex/models/cortex.py:125-165): B = max+1,
    events of a sample in their original order (stable), zero padding. The
    index work (bincount, scan, stable ranks) runs on the device; the two host
    reads the padded shape needs (B and E_max) remain, as in the reference.
    """
    dev = L.require_cuda(flat_tokens, what="_pack_events")
    bidx = batch_indices.to(dev)
    E = int(bidx.shape[0])
    if batch_size is None:
        batch_size = int(bidx.max().item()) + 1 if E > 0 else 1
    counts, offsets, dest, e_max_t = _ops.pack_events(bidx, batch_size)
    e_max = int(e_max_t.item())
    return _ops.pack_scatter(flat_tokens, bidx, dest, offsets, batch_size, e_max)


__all__ = ["BehaviorDecoder", "CortexModel", "MaskedSpikeHead", "_pack_events", "cast"]
