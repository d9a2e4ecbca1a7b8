"""GPU test of ck_norm_linear_static, the norm+linear entry point for callers
that cannot allocate device memory (for example a host runtime that binds the C
ABI without a CUDA allocator of its own, or a serving loop that must not
allocate). Where ck_norm_linear needs a caller-provided workspace (LayerNorm
rows, fp32 rows, the two-launch path), this entry point uses a fixed 8 MiB
device array inside the library instead; RMSNorm of bf16 rows runs as one
launch on both entry points and needs no scratch at all.

Both entry points are called through the C ABI on the same inputs, twice in a
row with different shapes and data (the static array keeps the previous call's
contents, which must not leak into the next result). They run the same kernels
on the same inputs, so their outputs must be bit-identical. The file is named so
that pytest collects it last.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    from cortex import _lib as L

    return L, L.load()


def _inputs(M, K, N, dtype, seed, int8=False):
    """x (M, K), gamma, beta (K,), and the weight: (K, N) in dtype, or (N, K)
    int8 with fp32 per-output-channel scales."""
    torch.manual_seed(seed)
    x = torch.randn(M, K, dtype=dtype, device=DEV)
    g = (torch.rand(K, device=DEV) + 0.5).to(dtype)
    b = (0.1 * torch.randn(K, device=DEV)).to(dtype)
    if int8:
        w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=DEV)
        sc = (torch.rand(N, device=DEV) + 0.5) * 1e-2
        return x, g, b, w, sc
    return x, g, b, torch.randn(K, N, dtype=dtype, device=DEV), None


def _args(L, x, g, b, w, sc, mode):
    M, K = x.shape
    dt = L.dtype_code(x.dtype)
    if sc is not None:  # int8 (N, K)
        N = w.shape[0]
        wargs = (w.data_ptr(), L.CK_I8, L.CK_W_NK, N, K, sc.data_ptr())
    else:
        N = w.shape[1]
        wargs = (w.data_ptr(), dt, L.CK_W_KN, N, N, None)
    beta = b.data_ptr() if mode == L.CK_NORM_LAYER else None
    return M, K, N, dt, beta, wargs


def _static(x, g, b, w, sc, mode):
    L, lib = _lib()
    M, K, N, dt, beta, wargs = _args(L, x, g, b, w, sc, mode)
    y = torch.full((M, N), float("nan"), dtype=x.dtype, device=DEV)
    rc = lib.ck_norm_linear_static(x.data_ptr(), dt, M, K, K, g.data_ptr(), beta, 1e-5, mode,
                                   *wargs, L.CK_EPI_STORE, None, 0, 0, y.data_ptr(), N,
                                   L.stream_of(x.device))
    return rc, y


def _with_workspace(x, g, b, w, sc, mode):
    L, lib = _lib()
    M, K, N, dt, beta, wargs = _args(L, x, g, b, w, sc, mode)
    y = torch.empty(M, N, dtype=x.dtype, device=DEV)
    nbytes = lib.ck_norm_linear_workspace_bytes(dt, M, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.ck_norm_linear(x.data_ptr(), dt, M, K, K, g.data_ptr(), beta, 1e-5, mode, *wargs,
                            L.CK_EPI_STORE, None, 0, 0, y.data_ptr(), N, ws.data_ptr(), nbytes,
                            L.stream_of(x.device))
    assert rc == 0, L.status_string(rc)
    return y


CASES = [  # (dtype, norm, int8 weights)
    (torch.bfloat16, "rms", False),    # one launch, no scratch
    (torch.bfloat16, "layer", False),  # LayerNorm with beta: through the scratch
    (torch.bfloat16, "layer", True),   # ... into the int8-weight GEMM with its scales
    (torch.bfloat16, "rms", True),     # one launch, int8 weights
    (torch.float32, "rms", False),     # fp32 rows: through the scratch
    (torch.float32, "layer", False),
]


@pytest.mark.parametrize("dtype,norm,int8", CASES)
def test_static_scratch_matches_workspace_entry_point(dtype, norm, int8):
    L, _ = _lib()
    mode = L.CK_NORM_RMS if norm == "rms" else L.CK_NORM_LAYER
    # two calls in a row: a problem that fills most of the array, then a
    # smaller one with other data
    big = 8192 if dtype == torch.bfloat16 else 4096
    for (M, K, N), seed in (((big, 512, 1536), 1), ((33, 64, 96), 2)):
        x, g, b, w, sc = _inputs(M, K, N, dtype, seed, int8)
        rc, y = _static(x, g, b, w, sc, mode)
        assert rc == 0, L.status_string(rc)
        ref = _with_workspace(x, g, b, w, sc, mode)
        assert torch.isfinite(y.float()).all()
        assert torch.equal(y, ref)
    assert L.device_status()[0] == 0


def test_static_plain_linear_passes_through():
    """CK_NORM_NONE is the plain linear on both entry points (no scratch)."""
    L, _ = _lib()
    x, g, b, w, sc = _inputs(256, 128, 64, torch.bfloat16, 4)
    rc, y = _static(x, g, b, w, sc, L.CK_NORM_NONE)
    assert rc == 0, L.status_string(rc)
    assert torch.equal(y, _with_workspace(x, g, b, w, sc, L.CK_NORM_NONE))


def test_static_scratch_rejects_problems_over_its_size():
    L, _ = _lib()
    # 8193 x 512 bf16 rows through the scratch (LayerNorm) are one row more than
    # the 8 MiB array holds: rejected before anything is launched
    x, g, b, w, sc = _inputs(8193, 512, 64, torch.bfloat16, 3)
    rc, y = _static(x, g, b, w, sc, L.CK_NORM_LAYER)
    assert rc == L.CK_ERR_INVALID_ARG
    torch.cuda.synchronize()
    assert torch.isnan(y.float()).all()  # nothing was launched
    # the one-launch RMSNorm path needs no scratch, so the same size runs
    rc, y = _static(x, g, b, w, sc, L.CK_NORM_RMS)
    assert rc == 0, L.status_string(rc)
    assert torch.equal(y, _with_workspace(x, g, b, w, sc, L.CK_NORM_RMS))
