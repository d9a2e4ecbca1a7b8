"""Fused spike tokenizer on B200 (drop-in for ``cortex.kernels.tokenizer``).

``fused_tokenizer`` keeps the reference signature and error behaviour
(cortex/kernels/tokenizer.py:177-249) and runs the sm_100a gather-sum kernel
(``ck_tokenize``): one warp per event, 16-byte vector loads of the three table
rows, the sum evaluated left to right in the table dtype (bf16 gives
``bf16(bf16(n + t) + v)``, bit-identical to the eager expression). It requires
CUDA tensors; there is no CPU fallback.

``fused_tokenizer_reference`` is the reference's eager twin
(cortex/kernels/tokenizer.py:68-81), kept for callers that test against it. No
function of this package calls it.
"""

from __future__ import annotations

import torch

from cortex.kernels import _ops


def fused_tokenizer_reference(neuron_emb: torch.Tensor, time_emb: torch.Tensor,
                              value_emb: torch.Tensor, neuron_ids: torch.Tensor,
                              time_bins: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    """Eager ``neuron_emb[nid] + time_emb[tb] + value_emb[val]``."""
    return neuron_emb[neuron_ids] + time_emb[time_bins] + value_emb[values]


def fused_tokenizer(neuron_emb: torch.Tensor, time_emb: torch.Tensor, value_emb: torch.Tensor,
                    neuron_ids: torch.Tensor, time_bins: torch.Tensor,
                    values: torch.Tensor) -> torch.Tensor:
    """B200 fused tokenizer.

    Args:
        neuron_emb, time_emb, value_emb: (vocab, D) float32/bfloat16 tables, contiguous.
        neuron_ids, time_bins, values: (E,) int64 (or int32) on the same CUDA device;
            strided views are read in place.

    Returns:
        (E, D) tokens in the tables' dtype.

    Raises:
        ValueError: non-contiguous tables, index shape mismatch, or differing D
            (same checks as the reference, cortex/kernels/tokenizer.py:208-218).
        RuntimeError: tensors not on a CUDA device.
    """
    if not (neuron_emb.is_contiguous() and time_emb.is_contiguous() and value_emb.is_contiguous()):
        raise ValueError("embedding tables must be contiguous (call .contiguous() first)")
    if not (neuron_ids.shape == time_bins.shape == values.shape):
        raise ValueError(
            f"index tensors must have identical shapes, got "
            f"{neuron_ids.shape}, {time_bins.shape}, {values.shape}")
    D = neuron_emb.shape[1]
    if time_emb.shape[1] != D or value_emb.shape[1] != D:
        raise ValueError("all embedding tables must have the same hidden dim D")
    if not (neuron_emb.dtype == time_emb.dtype == value_emb.dtype):
        raise ValueError("all embedding tables must share one dtype")
    E = neuron_ids.shape[0]
    if E == 0:
        from cortex import _lib
        dev = _lib.require_cuda(neuron_emb, what="fused_tokenizer")
        return torch.empty((0, D), dtype=neuron_emb.dtype, device=dev)
    if neuron_ids.dim() != 1:
        raise ValueError("index tensors must be 1-D")
    return _ops.tokenize(neuron_emb, time_emb, value_emb, neuron_ids, time_bins, values)
