"""GPU test of ck_norm_linear_static, the norm+linear entry point for callers
that cannot allocate device memory (for example a host runtime that binds the C
ABI without a CUDA allocator of its own, or a serving loop that must not
allocate). Its scratch is a fixed 8 MiB device array inside the library instead
of a caller-provided workspace.

Both entry points are called through the C ABI on the same inputs, twice in a
row with different shapes and data (the static array keeps the previous call's
contents, which must not leak into the next result), and the outputs compared
with the tolerances of the other RMSNorm+linear tests. The file is named so that
pytest collects it last.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    from cortex import _lib as L

    return L, L.load()


def _inputs(M, K, N, dtype, seed):
    torch.manual_seed(seed)
    x = torch.randn(M, K, dtype=dtype, device=DEV)
    g = (torch.rand(K, device=DEV) + 0.5).to(dtype)
    w = torch.randn(K, N, dtype=dtype, device=DEV)
    return x, g, w


def _static(x, g, w, mode):
    L, lib = _lib()
    M, K = x.shape
    N = w.shape[1]
    y = torch.full((M, N), float("nan"), dtype=x.dtype, device=DEV)
    dt = L.dtype_code(x.dtype)
    rc = lib.ck_norm_linear_static(x.data_ptr(), dt, M, K, K, g.data_ptr(), None, 1e-6, mode,
                                   w.data_ptr(), dt, L.CK_W_KN, N, N, None, L.CK_EPI_STORE, None,
                                   0, 0, y.data_ptr(), N, L.stream_of(x.device))
    return rc, y


def _with_workspace(x, g, w, mode):
    L, lib = _lib()
    M, K = x.shape
    N = w.shape[1]
    y = torch.empty(M, N, dtype=x.dtype, device=DEV)
    dt = L.dtype_code(x.dtype)
    nbytes = lib.ck_norm_linear_workspace_bytes(dt, M, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.ck_norm_linear(x.data_ptr(), dt, M, K, K, g.data_ptr(), None, 1e-6, mode,
                            w.data_ptr(), dt, L.CK_W_KN, N, N, None, L.CK_EPI_STORE, None, 0, 0,
                            y.data_ptr(), N, ws.data_ptr(), nbytes, L.stream_of(x.device))
    assert rc == 0
    return y


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_static_scratch_matches_workspace_entry_point(dtype):
    L, _ = _lib()
    tol = dict(rtol=1e-2, atol=1e-1) if dtype == torch.bfloat16 else dict(rtol=1e-4, atol=1e-4)
    # two calls in a row: a large problem, then a smaller one with other data
    for (M, K, N), seed in (((8192 if dtype == torch.bfloat16 else 4096, 512, 1536), 1),
                            ((33, 64, 97), 2)):
        x, g, w = _inputs(M, K, N, dtype, seed)
        rc, y = _static(x, g, w, L.CK_NORM_RMS)
        assert rc == 0, L.status_string(rc)
        torch.testing.assert_close(y, _with_workspace(x, g, w, L.CK_NORM_RMS), **tol)
    assert L.device_status()[0] == 0


def test_static_scratch_rejects_problems_over_its_size():
    L, _ = _lib()
    # 8193 x 512 bf16 is one row more than the 8 MiB array holds
    x, g, w = _inputs(8193, 512, 64, torch.bfloat16, 3)
    rc, y = _static(x, g, w, L.CK_NORM_RMS)
    assert rc == L.CK_ERR_INVALID_ARG
    torch.cuda.synchronize()
    assert torch.isnan(y.float()).all()  # nothing was launched
