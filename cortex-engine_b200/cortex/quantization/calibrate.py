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

The calibration helpers (activation statistics, hooks, ``derive_scales``) are
plain torch utilities with the reference's semantics.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn

from cortex import _lib as L
from cortex.kernels import _ops


@dataclass
class ActivationStats:
    """Per-layer activation statistics (cortex/quantization/calibrate.py:55-79)."""

    abs_max_history: list[float] = field(default_factory=list)

    def update(self, x: torch.Tensor) -> None:
        self.abs_max_history.append(float(x.detach().abs().max().item()))

    @property
    def percentile_99(self) -> float:
        if not self.abs_max_history:
            return 1.0
        vals = sorted(self.abs_max_history)
        idx = max(0, int(len(vals) * 0.99) - 1)
        return vals[idx]

    @property
    def n_batches(self) -> int:
        return len(self.abs_max_history)


class CalibrationHook:
    """Forward pre-hook recording input statistics (:82-96)."""

    def __init__(self) -> None:
        self.stats = ActivationStats()
        self._handle: Any = None

    def __call__(self, module: nn.Module, args: tuple[Any, ...]) -> None:
        if args:
            self.stats.update(args[0])

    def remove(self) -> None:
        if self._handle is not None:
            self._handle.remove()
            self._handle = None


def attach_calibration_hooks(model: nn.Module) -> dict[str, CalibrationHook]:
    hooks: dict[str, CalibrationHook] = {}
    for name, module in model.named_modules():
        if isinstance(module, nn.Linear):
            hook = CalibrationHook()
            hook._handle = module.register_forward_pre_hook(hook)
            hooks[name] = hook
    return hooks


def remove_calibration_hooks(hooks: dict[str, CalibrationHook]) -> None:
    for hook in hooks.values():
        hook.remove()


@dataclass
class LayerScales:
    """Quantization scales for one linear layer (:119-124)."""

    weight_scale: torch.Tensor  # (out_features,) float32
    act_scale: float


def weight_scales(weight: torch.Tensor) -> torch.Tensor:
    """``absmax_row / 127`` clamped at 1e-8, in fp32 (:154)."""
    return weight.detach().float().abs().amax(dim=1).clamp(min=1e-8) / 127.0


def derive_scales(model: nn.Module, hooks: dict[str, CalibrationHook]) -> dict[str, LayerScales]:
    scales: dict[str, LayerScales] = {}
    for name, module in model.named_modules():
        if not isinstance(module, nn.Linear) or name not in hooks:
            continue
        hook = hooks[name]
        if hook.stats.n_batches == 0:
            continue
        scales[name] = LayerScales(weight_scale=weight_scales(module.weight).cpu(),
                                   act_scale=max(hook.stats.percentile_99, 1e-8) / 127.0)
    return scales


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


def model_weight_bytes(model: nn.Module) -> int:
    total = 0
    for p in model.parameters():
        total += p.numel() * p.element_size()
    for buf in model.buffers():
        total += buf.numel() * buf.element_size()
    return total


def count_quantized_linears(model: nn.Module) -> tuple[int, int]:
    n_quant = sum(1 for m in model.modules() if isinstance(m, QuantizedLinear))
    n_float = sum(1 for m in model.modules() if isinstance(m, nn.Linear))
    return n_quant, n_quant + n_float


def save_quantized(model: nn.Module, path: Path, meta: dict[str, Any] | None = None) -> None:
    """``torch.save({'state_dict': ..., 'meta': ...})`` (:305-318)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    torch.save({"state_dict": model.state_dict(), "meta": meta or {}}, path)


def load_quantized(path: Path, model: nn.Module) -> nn.Module:
    payload = torch.load(path, map_location="cpu", weights_only=True)
    model.load_state_dict(payload["state_dict"])
    return model


def calibration_summary(hooks: dict[str, CalibrationHook],
                        scales: dict[str, LayerScales]) -> list[dict[str, Any]]:
    rows = []
    for name, hook in hooks.items():
        s = scales.get(name)
        rows.append({
            "layer": name,
            "calib_batches": hook.stats.n_batches,
            "act_abs_max_p99": round(hook.stats.percentile_99, 6),
            "act_scale": round(s.act_scale, 8) if s else None,
            "weight_scale_min": round(float(s.weight_scale.min()), 8) if s else None,
            "weight_scale_max": round(float(s.weight_scale.max()), 8) if s else None,
        })
    return rows
