"""Per-output-channel INT8 weight quantization (drop-in for
``cortex.quantization.calibrate``).

The storage format, scale rule and module surface are the reference's
(cortex/quantization/calibrate.py:1-362), so checkpoints written by either side
load in the other:

* ``scale[c] = max(|W[c, :]|) / 127`` (clamped at 1e-8),
  ``W_int8 = round(W / scale).clamp(-127, 127)`` as int8 (:154, :205-211);
* ``QuantizedLinear`` buffers ``weight_int8`` (out, in) int8, ``weight_scale`` (out,)
  fp32 and an optional ``bias`` (:170-234);
* ``convert_model`` replaces ``nn.Linear`` children by qualified name (:240-279).

What changes is ``QuantizedLinear.forward``: instead of dequantizing the whole
matrix to the activation dtype and calling ``F.linear`` (:225-228), it runs the
sm_100a GEMM with the int8 matrix as the B operand. Each int8 tile is widened to
bf16 in shared memory (exact for |w| <= 127) and the per-channel scale is
applied to the fp32 accumulator, so the weight crosses HBM as int8 and no bf16
copy of it ever exists. Activations stay in their dtype (the reference's
activation scale is computed but never used in the forward pass, :17-19). CUDA
only.

Activation calibration (hooks, percentile statistics, summaries) and the
checkpoint helpers of the reference module are not on the forward path and are
not part of this package; a model quantized with the reference's tools loads
here through ``convert_model`` and ``load_state_dict``.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass

import torch
import torch.nn as nn

from cortex import _lib as L
from cortex.kernels import _ops


@dataclass
class LayerScales:
    """Quantization scales for one linear layer (:119-124)."""

    weight_scale: torch.Tensor  # (out_features,) float32
    act_scale: float


def weight_scales(weight: torch.Tensor) -> torch.Tensor:
    """``absmax_row / 127`` clamped at 1e-8, in fp32 (:154)."""
    return weight.detach().float().abs().amax(dim=1).clamp(min=1e-8) / 127.0


class QuantizedLinear(nn.Module):
    """``nn.Linear`` replacement holding int8 weights and fp32 per-channel scales."""

    in_features: int
    out_features: int
    weight_int8: torch.Tensor
    weight_scale: torch.Tensor
    bias: torch.Tensor | None

    def __init__(self, weight_int8: torch.Tensor, weight_scale: torch.Tensor,
                 bias: torch.Tensor | None) -> None:
        super().__init__()
        self.in_features = weight_int8.shape[1]
        self.out_features = weight_int8.shape[0]
        self.register_buffer("weight_int8", weight_int8)
        self.register_buffer("weight_scale", weight_scale)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.register_buffer("bias", None)

    @classmethod
    def from_linear(cls, linear: nn.Linear, scales: LayerScales) -> QuantizedLinear:
        w = linear.weight.detach().float()
        w_scaled = w / scales.weight_scale.to(w.device)[:, None]
        w_int8 = w_scaled.round().clamp(-127, 127).to(torch.int8)
        bias = linear.bias.detach().clone() if linear.bias is not None else None
        return cls(w_int8, scales.weight_scale.to(w.device), bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """``x @ (W_int8 * scale).T (+ bias)`` on the B200 int8-weight GEMM."""
        L.require_cuda(x, self.weight_int8, what="QuantizedLinear")
        if self.bias is None:
            return _ops.linear(x, self.weight_int8, w_scale=self.weight_scale)
        return _ops.linear(x, self.weight_int8, w_scale=self.weight_scale,
                           epi=L.CK_EPI_BIAS, aux=self.bias.to(x.dtype).contiguous())

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, quantized=INT8")


def convert_model(model: nn.Module, scales: dict[str, LayerScales],
                  inplace: bool = True) -> nn.Module:
    """Replace ``nn.Linear`` layers with ``QuantizedLinear`` where scales exist."""
    if not inplace:
        model = copy.deepcopy(model)
    _replace_linears(model, scales, prefix="")
    return model


def _replace_linears(module: nn.Module, scales: dict[str, LayerScales], prefix: str) -> None:
    for name, child in list(module.named_children()):
        full_name = f"{prefix}.{name}".lstrip(".")
        if isinstance(child, nn.Linear) and full_name in scales:
            setattr(module, name, QuantizedLinear.from_linear(child, scales[full_name]))
        else:
            _replace_linears(child, scales, full_name)
