"""ctypes binding of libcortex_b200.so (the C ABI in include/cortex_b200.h).

The shared library is built in-tree by ``cortex-engine_b200/build.py`` and sits
next to this file. There is no fallback: if the library is missing or no CUDA
device is present, every kernel entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcortex_b200.so")

CK_OK = 0
CK_ERR_INVALID_ARG = -1
CK_ERR_UNSUPPORTED = -2
CK_ERR_CUDA = -3
CK_ERR_INDEX = -4
CK_ERR_TIMEOUT = -5
CK_ERR_WORKSPACE = -6

CK_F32, CK_BF16, CK_I8, CK_I32, CK_I64 = 0, 1, 2, 3, 4
CK_NORM_NONE, CK_NORM_LAYER, CK_NORM_RMS = 0, 1, 2
CK_EPI_STORE, CK_EPI_GELU, CK_EPI_RESID, CK_EPI_BIAS = 0, 1, 2, 3
CK_W_NK, CK_W_KN = 0, 1

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t


class AttentionArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", _int),
        ("B", _i32), ("H", _i32), ("Dh", _i32), ("Lq", _i32),
        ("n_keys", _i32),
        ("key_offsets", _vp),
        ("q", _vp), ("q_ld", _i64), ("q_rows", _i64), ("q_rows_per_b", _i64),
        ("q_rows_per_h", _i64), ("q_col_per_h", _i64),
        ("k", _vp), ("k_ld", _i64), ("k_rows", _i64), ("k_rows_per_b", _i64),
        ("k_rows_per_h", _i64), ("k_col_per_h", _i64),
        ("v", _vp), ("v_ld", _i64), ("v_rows", _i64), ("v_rows_per_b", _i64),
        ("v_rows_per_h", _i64), ("v_col_per_h", _i64),
        ("o", _vp), ("o_ld", _i64), ("o_rows_per_b", _i64), ("o_rows_per_h", _i64),
        ("o_col_per_h", _i64),
        ("block_mask", _vp),
        ("n_q_tiles", _i32), ("n_k_tiles", _i32), ("block_l", _i32), ("block_e", _i32),
        ("key_mask", _vp), ("key_mask_ld", _i64),
        ("scale", _f32),
    ]


class LinearWeight(ctypes.Structure):
    _fields_ = [("w", _vp), ("dtype", _int), ("scale", _vp), ("bias", _vp)]


class BlockWeights(ctypes.Structure):
    _fields_ = [
        ("norm_attn_w", _vp), ("norm_attn_b", _vp),
        ("qkv", LinearWeight), ("out", LinearWeight),
        ("norm_mlp_w", _vp), ("norm_mlp_b", _vp),
        ("mlp0", LinearWeight), ("mlp2", LinearWeight),
    ]


class Model(ctypes.Structure):
    _fields_ = [
        ("dtype", _int),
        ("hidden_dim", _i32), ("latent_dim", _i32), ("num_latents", _i32),
        ("num_layers", _i32), ("num_heads", _i32), ("head_dim", _i32),
        ("cross_heads", _i32), ("mlp_hidden", _i32), ("behavior_dim", _i32),
        ("n_vocab", _i64), ("t_vocab", _i64), ("v_vocab", _i64),
        ("neuron_emb", _vp), ("time_emb", _vp), ("value_emb", _vp),
        ("latents", _vp),
        ("norm_q_w", _vp), ("norm_q_b", _vp), ("norm_kv_w", _vp), ("norm_kv_b", _vp),
        ("cross_q", LinearWeight), ("cross_kv", LinearWeight), ("cross_out", LinearWeight),
        ("blocks", ctypes.POINTER(BlockWeights)),
        ("final_norm_w", _vp), ("final_norm_b", _vp),
        ("head_query", _vp),
        ("head_norm_w", _vp), ("head_norm_b", _vp),
        ("head_q", LinearWeight), ("head_kv", LinearWeight), ("head_out", LinearWeight),
    ]


class TraceRecord(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 96), ("stream", _vp), ("ms", _f32)]


_SIGS = {
    "ck_get_last_status": (_int, [ctypes.POINTER(_int)]),
    "ck_last_cuda_error": (_int, []),
    "ck_status_string": (ctypes.c_char_p, [_int]),
    "ck_num_sms": (_int, []),
    "ck_launch_count": (ctypes.c_longlong, []),
    "ck_trace_begin": (_int, [_i32]),
    "ck_trace_end": (_int, [ctypes.POINTER(TraceRecord), _i32, ctypes.POINTER(_i32)]),
    "ck_pack_workspace_bytes": (_sz, [_i64, _i32]),
    "ck_pack_events": (_int, [_vp, _int, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ck_pack_scatter": (_int, [_vp, _int, _i64, _i32, _i64, _vp, _int, _i64, _vp, _vp, _i32,
                               _vp, _vp, _vp]),
    "ck_tokenize": (_int, [_vp, _vp, _vp, _int, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                           _vp, _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _f32, _vp,
                           _i64, _vp]),
    "ck_dequantize_int8": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "ck_tokenize_packed_workspace_bytes": (_sz, []),
    "ck_tokenize_packed": (_int, [_vp, _vp, _vp, _int, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _vp,
                                  _int, _i64, _i32, _vp, _vp, _f32, _vp, _i64, _vp, _vp, _sz,
                                  _vp]),
    "ck_row_norm": (_int, [_vp, _int, _i64, _i32, _i64, _vp, _vp, _f32, _int, _vp, _i64, _vp]),
    "ck_linear": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _int, _int, _i64, _i64, _vp, _int,
                         _vp, _i64, _i64, _vp, _i64, _vp]),
    "ck_norm_linear_workspace_bytes": (_sz, [_int, _i64, _i64]),
    "ck_norm_linear": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _f32, _int, _vp, _int,
                              _int, _i64, _i64, _vp, _int, _vp, _i64, _i64, _vp, _i64, _vp,
                              _sz, _vp]),
    "ck_norm_linear_static": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _f32, _int, _vp,
                                     _int, _int, _i64, _i64, _vp, _int, _vp, _i64, _i64, _vp,
                                     _i64, _vp]),
    "ck_attention": (_int, [ctypes.POINTER(AttentionArgs), _vp]),
    "ck_forward_workspace_bytes": (_sz, [ctypes.POINTER(Model), _i64, _i32]),
    "ck_forward": (_int, [ctypes.POINTER(Model), _vp, _vp, _vp, _vp, _int, _i64, _i32, _vp, _vp,
                          _sz, _vp]),
    "ck_batch_stage": (_int, [_vp, _vp, _vp, _vp, _int, _i64, _vp, _i64,
                              ctypes.POINTER(_i32)]),
    "ck_forward_batch": (_int, [ctypes.POINTER(Model), _vp, _i64, _i32, _vp, _vp, _sz, _vp]),
    "ck_runner_create": (_int, [ctypes.POINTER(Model), _i32, ctypes.POINTER(_vp)]),
    "ck_runner_destroy": (None, [_vp]),
    "ck_runner_stage": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _i64, _i32, ctypes.POINTER(_i32)]),
    "ck_runner_launch": (_int, [_vp, _vp, _vp]),
    "ck_runner_launch_batch": (_int, [_vp, _vp, _i64, _i32, _vp, _vp]),
    "ck_runner_invalidate": (_int, [_vp, ctypes.POINTER(Model)]),
    "ck_runner_counters": (_int, [_vp, ctypes.POINTER(ctypes.c_longlong),
                                  ctypes.POINTER(ctypes.c_longlong)]),
    "ck_forward_kv": (_int, [ctypes.POINTER(Model), _vp, _i64, _i32, _vp, _vp, _vp, _sz, _vp]),
    "ck_forward_from_kv": (_int, [ctypes.POINTER(Model), _vp, _i64, _vp, _i32, _vp, _vp, _sz,
                                  _vp]),
    "ck_copy_rows": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _i32, _vp]),
    "ck_collate_bins_workspace_bytes": (_sz, [_i32, _i32]),
    "ck_collate_bins": (_int, [_vp, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _sz, _vp, _vp]),
}

CK_BATCH_HEADER_WORDS = 4


def batch_words(capacity: int) -> int:
    """int32 words of a packed event batch (CK_BATCH_WORDS in cortex_b200.h)."""
    return CK_BATCH_HEADER_WORDS + 4 * capacity

EXPORTED_SYMBOLS = tuple(_SIGS)

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the shared library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python cortex-engine_b200/build.py`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class DeviceStatusError(RuntimeError):
    pass


def status_string(code: int) -> str:
    return load().ck_status_string(code).decode()


def check(rc: int, what: str) -> None:
    if rc == CK_OK:
        return
    msg = f"{what}: {status_string(rc)} (code {rc})"
    if rc == CK_ERR_CUDA:
        msg += f", cudaError {load().ck_last_cuda_error()}"
    if rc == CK_ERR_INVALID_ARG:
        raise ValueError(msg)
    if rc == CK_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == CK_ERR_INDEX:
        raise IndexError(msg)
    raise RuntimeError(msg)


def device_status(clear: bool = True) -> tuple[int, list[int]]:
    """Synchronise the current device and read (then clear) its status word."""
    info = (_int * 4)()
    code = load().ck_get_last_status(info)
    return int(code), list(info)


def check_device_status(what: str = "device") -> None:
    code, info = device_status()
    if code == CK_OK:
        return
    msg = f"{what}: {status_string(code)} (code {code}, info {info})"
    if code == CK_ERR_INDEX:
        raise IndexError(msg)
    raise DeviceStatusError(msg)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return CK_F32
    if dt == torch.bfloat16:
        return CK_BF16
    if dt == torch.int8:
        return CK_I8
    if dt == torch.int32:
        return CK_I32
    if dt == torch.int64:
        return CK_I64
    raise NotImplementedError(f"dtype {dt} is not supported by the B200 kernels "
                              "(float32, bfloat16, int8 weights, int32/int64 indices)")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    """The handle of torch's current CUDA stream on ``device``."""
    if _raw_stream is not None:
        idx = device.index
        return _raw_stream(torch.cuda.current_device() if idx is None else idx)
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor, what: str) -> torch.device:
    """All tensors must live on one CUDA device; there is no CPU path."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(
                f"{what}: the B200 kernels need CUDA tensors (got {t.device}); "
                "this package has no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{what}: tensors are on different devices ({dev}, {t.device})")
    if dev is None:
        raise RuntimeError(f"{what}: no tensor given")
    load()
    return dev
