"""Tensor-level wrappers over the C ABI. Every function launches on the current
CUDA stream of the tensors' device and allocates its outputs and workspaces with
torch (the library itself allocates nothing)."""

from __future__ import annotations

import ctypes

import torch

from cortex import _lib as L


def _idx_code(t: torch.Tensor) -> int:
    if t.dtype == torch.int64:
        return L.CK_I64
    if t.dtype == torch.int32:
        return L.CK_I32
    raise TypeError(f"index tensors must be int32 or int64, got {t.dtype}")


def pack_events(batch_indices: torch.Tensor, batch_size: int):
    """Device-side packing index work: (counts[B], offsets[B+1], dest[E], e_max[1])."""
    dev = L.require_cuda(batch_indices, what="pack_events")
    lib = L.load()
    E = batch_indices.shape[0]
    counts = torch.empty(batch_size, dtype=torch.int32, device=dev)
    offsets = torch.empty(batch_size + 1, dtype=torch.int32, device=dev)
    dest = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
    e_max = torch.empty(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.ck_pack_workspace_bytes(E, batch_size)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    rc = lib.ck_pack_events(L.ptr(batch_indices), _idx_code(batch_indices),
                            batch_indices.stride(0) if E > 0 else 1, E, batch_size,
                            L.ptr(counts), L.ptr(offsets), L.ptr(dest), L.ptr(e_max),
                            L.ptr(ws), ws_bytes, L.stream_of(dev))
    L.check(rc, "ck_pack_events")
    return counts, offsets, dest[:E], e_max


def pack_scatter(flat: torch.Tensor, batch_indices: torch.Tensor, dest: torch.Tensor,
                 offsets: torch.Tensor, batch_size: int, e_max: int):
    dev = L.require_cuda(flat, batch_indices, what="pack_scatter")
    E, D = flat.shape
    out = torch.zeros(batch_size, e_max, D, dtype=flat.dtype, device=dev)
    mask = torch.zeros(batch_size, e_max, dtype=torch.bool, device=dev)
    if E == 0:
        return out, mask
    rc = L.load().ck_pack_scatter(L.ptr(flat), L.dtype_code(flat.dtype), E, D, flat.stride(0),
                                  L.ptr(batch_indices), _idx_code(batch_indices),
                                  batch_indices.stride(0), L.ptr(dest), L.ptr(offsets), e_max,
                                  L.ptr(out), L.ptr(mask), L.stream_of(dev))
    L.check(rc, "ck_pack_scatter")
    return out, mask


def tokenize(n_emb, t_emb, v_emb, nid, tb, val, dest=None, gamma=None, beta=None,
             eps: float = 1e-5, out=None, out_rows: int | None = None):
    dev = L.require_cuda(n_emb, t_emb, v_emb, nid, tb, val, what="tokenize")
    E = nid.shape[0]
    D = n_emb.shape[1]
    if out is None:
        out = torch.empty(out_rows if out_rows is not None else E, D, dtype=n_emb.dtype,
                          device=dev)
    if E == 0:
        return out
    if not (nid.dtype == tb.dtype == val.dtype):
        tb = tb.to(nid.dtype)
        val = val.to(nid.dtype)
    for name, tab in (("neuron", n_emb), ("time", t_emb), ("value", v_emb)):
        if tab.stride(1) != 1:
            raise ValueError(f"{name} table rows must be contiguous")
    rc = L.load().ck_tokenize(
        L.ptr(n_emb), L.ptr(t_emb), L.ptr(v_emb), L.dtype_code(n_emb.dtype), D,
        n_emb.shape[0], t_emb.shape[0], v_emb.shape[0],
        n_emb.stride(0), t_emb.stride(0), v_emb.stride(0),
        L.ptr(nid), L.ptr(tb), L.ptr(val), _idx_code(nid),
        nid.stride(0), tb.stride(0), val.stride(0), E,
        L.ptr(dest), L.ptr(gamma), L.ptr(beta), eps, L.ptr(out), out.stride(0),
        L.stream_of(dev))
    L.check(rc, "ck_tokenize")
    return out


def tokenize_packed(n_emb, t_emb, v_emb, nid, tb, val, batch_indices, batch_size: int,
                    gamma=None, beta=None, eps: float = 1e-5):
    """Window offsets and tokens in packed order in one call (ck_tokenize_packed):
    (tokens (E, D), offsets (B + 1,) int32). Tables and index arrays contiguous."""
    dev = L.require_cuda(n_emb, t_emb, v_emb, nid, tb, val, batch_indices, what="tokenize_packed")
    lib = L.load()
    E, D = nid.shape[0], n_emb.shape[1]
    idx = [t.to(nid.dtype).contiguous() for t in (nid, tb, val, batch_indices)]
    tabs = [t.contiguous() for t in (n_emb, t_emb, v_emb)]
    out = torch.empty(max(E, 1), D, dtype=n_emb.dtype, device=dev)
    offsets = torch.empty(batch_size + 1, dtype=torch.int32, device=dev)
    ws_bytes = lib.ck_tokenize_packed_workspace_bytes()
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    rc = lib.ck_tokenize_packed(
        L.ptr(tabs[0]), L.ptr(tabs[1]), L.ptr(tabs[2]), L.dtype_code(n_emb.dtype), D,
        n_emb.shape[0], t_emb.shape[0], v_emb.shape[0], *(L.ptr(t) for t in idx),
        _idx_code(idx[0]), E, batch_size, L.ptr(gamma), L.ptr(beta), eps, L.ptr(out), D,
        L.ptr(offsets), L.ptr(ws), ws_bytes, L.stream_of(dev))
    L.check(rc, "ck_tokenize_packed")
    return out[:E], offsets


def row_norm(x: torch.Tensor, gamma, beta, eps: float, mode: int = L.CK_NORM_LAYER, out=None):
    dev = L.require_cuda(x, gamma, what="row_norm")
    D = x.shape[-1]
    x2 = x.reshape(-1, D)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x2.shape[0], D, dtype=x.dtype, device=dev)
    rc = L.load().ck_row_norm(L.ptr(x2), L.dtype_code(x.dtype), x2.shape[0], D, x2.stride(0),
                              L.ptr(gamma.contiguous()),
                              L.ptr(beta.contiguous() if beta is not None else None),
                              eps, mode, L.ptr(out), out.stride(0), L.stream_of(dev))
    L.check(rc, "ck_row_norm")
    return out.reshape(*x.shape[:-1], D)


def linear(x: torch.Tensor, w: torch.Tensor, *, w_scale=None, w_layout: int = L.CK_W_NK,
           epi: int = L.CK_EPI_STORE, aux=None, aux_row_mod: int = 0, out=None):
    """y = epi(x @ w.T) for w (N, K) or epi(x @ w) for w (K, N) (w_layout=CK_W_KN)."""
    dev = L.require_cuda(x, w, what="linear")
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    w = w if w.stride(-1) == 1 else w.contiguous()
    N = w.shape[0] if w_layout == L.CK_W_NK else w.shape[1]
    if (w.shape[1] if w_layout == L.CK_W_NK else w.shape[0]) != K:
        raise ValueError(f"linear: inner dims differ (x {tuple(x.shape)}, w {tuple(w.shape)})")
    if out is None:
        out = torch.empty(x2.shape[0], N, dtype=x.dtype, device=dev)
    ld_aux = 0
    if aux is not None:
        aux = aux if aux.stride(-1) == 1 else aux.contiguous()
        aux2 = aux.reshape(-1, aux.shape[-1])
        ld_aux = aux2.stride(0) if aux2.dim() == 2 else 0
    sc = None
    if w.dtype == torch.int8:
        sc = w_scale.float().contiguous()
    rc = L.load().ck_linear(L.ptr(x2), L.dtype_code(x.dtype), x2.shape[0], K, x2.stride(0),
                            L.ptr(w), L.dtype_code(w.dtype), w_layout, N, w.stride(0),
                            L.ptr(sc), epi, L.ptr(aux), ld_aux, aux_row_mod,
                            L.ptr(out), out.stride(0), L.stream_of(dev))
    L.check(rc, "ck_linear")
    return out.reshape(*x.shape[:-1], N)


def attention(q, k, v, *, B, H, Dh, Lq, n_keys=0, key_offsets=None,
              q_geom, k_geom, v_geom, o, o_geom, block_mask=None, block_l=1, block_e=1,
              key_mask=None, scale: float):
    """Generic attention launch. *_geom = (ld, rows, rows_per_b, rows_per_h, col_per_h)."""
    dev = L.require_cuda(q, k, v, o, what="attention")
    a = L.AttentionArgs()
    a.dtype = L.dtype_code(q.dtype)
    a.B, a.H, a.Dh, a.Lq, a.n_keys = B, H, Dh, Lq, n_keys
    a.key_offsets = L.ptr(key_offsets)
    a.q = L.ptr(q)
    a.q_ld, a.q_rows, a.q_rows_per_b, a.q_rows_per_h, a.q_col_per_h = q_geom
    a.k = L.ptr(k)
    a.k_ld, a.k_rows, a.k_rows_per_b, a.k_rows_per_h, a.k_col_per_h = k_geom
    a.v = L.ptr(v)
    a.v_ld, a.v_rows, a.v_rows_per_b, a.v_rows_per_h, a.v_col_per_h = v_geom
    a.o = L.ptr(o)
    a.o_ld, a.o_rows_per_b, a.o_rows_per_h, a.o_col_per_h = o_geom
    if block_mask is not None:
        a.block_mask = L.ptr(block_mask)
        a.n_q_tiles, a.n_k_tiles = block_mask.shape
        a.block_l, a.block_e = block_l, block_e
    if key_mask is not None:
        a.key_mask = L.ptr(key_mask)
        a.key_mask_ld = key_mask.stride(0)
    a.scale = scale
    rc = L.load().ck_attention(ctypes.byref(a), L.stream_of(dev))
    L.check(rc, "ck_attention")
    return o
