"""RMSNorm + linear on B200 (drop-in for ``cortex.kernels.fused_rmsnorm``).

``rms_norm_linear(x, gamma, w, bias=None, eps=1e-6)`` keeps the reference
signature (cortex/kernels/fused_rmsnorm.py:239-301): ``x`` is (..., K), ``w`` is
(K, N), the result (..., N). For bf16 it is one tcgen05 launch (``w`` read
N-major through TMA, no transpose copy): the GEMM's norm warps scale each
TMA-loaded tile of x by gamma in shared memory and sum x^2 per row, and the
epilogue multiplies each row by 1 / sqrt(mean(x^2) + eps) before the bias.
fp32 (and shapes whose strides TMA cannot take) normalise in fp32, round to
the input dtype as ``rms_norm_linear_reference`` does (:86-108), then run the
fp32 CUDA-core GEMM. A bias is added after rounding the product, as the
reference's ``out + bias`` does. CUDA tensors only.
"""

from __future__ import annotations

import torch

from cortex import _lib as L
from cortex.kernels import _ops


def rms_norm_linear_reference(x: torch.Tensor, gamma: torch.Tensor, w: torch.Tensor,
                              bias: torch.Tensor | None, eps: float = 1e-6) -> torch.Tensor:
    """The reference's eager twin (cortex/kernels/fused_rmsnorm.py:86-108), kept for
    callers that test against it. No function of this package calls it."""
    x_f32 = x.float()
    rms = torch.sqrt(x_f32.pow(2).mean(dim=-1, keepdim=True) + eps)
    x_norm = (x_f32 / rms) * gamma.float()
    out = x_norm.to(x.dtype) @ w
    if bias is not None:
        out = out + bias
    return out


def rms_norm_linear(x: torch.Tensor, gamma: torch.Tensor, w: torch.Tensor,
                    bias: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """Fused RMSNorm + linear; ``w`` is (K, N)."""
    lead = x.shape[:-1]
    K = x.shape[-1]
    if w.shape[0] != K:
        raise ValueError(f"w must be (K, N) with K={K}, got {tuple(w.shape)}")
    N = w.shape[1]
    dev = L.require_cuda(x, gamma, w, bias, what="rms_norm_linear")
    M = x.numel() // K if K > 0 else 0
    x2 = x.reshape(M, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    w = w.to(x.dtype) if w.dtype != x.dtype else w
    w = w.contiguous()
    out = torch.empty(M, N, dtype=x.dtype, device=dev)
    if M == 0 or N == 0:
        return out.reshape(*lead, N)
    lib = L.load()
    dt = L.dtype_code(x.dtype)
    g = gamma.to(x.dtype).contiguous()
    b = bias.to(x.dtype).contiguous() if bias is not None else None

    def call(ws, ws_bytes):
        return lib.ck_norm_linear(L.ptr(x2), dt, M, K, x2.stride(0), L.ptr(g), None, float(eps),
                                  L.CK_NORM_RMS, L.ptr(w), dt, L.CK_W_KN, N, w.stride(0), None,
                                  L.CK_EPI_BIAS if b is not None else L.CK_EPI_STORE, L.ptr(b),
                                  0, 0, L.ptr(out), out.stride(0), ws, ws_bytes,
                                  L.stream_of(dev))

    # bf16 rows run as one launch with the norm inside the GEMM and need no
    # workspace; the library says so (CK_ERR_WORKSPACE, nothing launched) when
    # a call needs one
    rc = call(None, 0)
    if rc == L.CK_ERR_WORKSPACE:
        ws_bytes = lib.ck_norm_linear_workspace_bytes(dt, M, K)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        rc = call(L.ptr(ws), ws_bytes)
    L.check(rc, "ck_norm_linear")
    return out.reshape(*lead, N)


__all__ = ["rms_norm_linear", "rms_norm_linear_reference", "_ops"]
