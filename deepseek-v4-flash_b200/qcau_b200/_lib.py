"""ctypes binding of libqcau_b200.so (the C ABI in include/qcau_b200.h).

The shared library is built in-tree by deepseek-v4-flash_b200/build.py.  There
is no fallback of any kind: if the library is missing, or no CUDA device is
present, the call raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libqcau_b200.so"

QCAU_OK = 0
QCAU_ERR_INVALID = -1
QCAU_ERR_CUDA = -2
QCAU_ERR_UNSUPPORTED = -3
QCAU_ERR_WORKSPACE = -4
QCAU_ERR_DEVICE = -5

DECODE_STATIC_SCRATCH_BYTES = 32 << 20  # QCAU_DECODE_STATIC_SCRATCH_BYTES

SCALE_F32 = 0
SCALE_E8M0 = 1
OUT_BF16 = 0
OUT_F32 = 1

DEVERR_TIMEOUT = 1
DEVERR_INDEX = 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_SZ = ctypes.c_size_t


class MlaDims(ctypes.Structure):
    """qcau_mla_dims of the header."""
    _fields_ = [
        ("batch", _I64), ("n_heads", _I64), ("dc", _I64), ("d_nope", _I64), ("d_rope", _I64),
        ("kv_lora", _I64), ("d_v", _I64), ("dim", _I64), ("page_size", _I64),
        ("max_pages", _I64), ("num_pages", _I64), ("max_seqlen", _I64), ("npos", _I64),
        ("softmax_scale", _F), ("w_scale_dtype", _I32), ("act_round_scale", _I32),
        ("out_dtype", _I32),
    ]


# Every function the header declares, with its ctypes signature.
SIGNATURES = {
    "qcau_version": ([], ctypes.c_int),
    "qcau_last_error": ([], ctypes.c_char_p),
    "qcau_device_error": ([_P], ctypes.c_int),
    "qcau_act_quant": ([_P, _P, _P, _I64, _I64, _I32, _I32, _I32, _I32, _P], ctypes.c_int),
    "qcau_fp8_gemm": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _P], ctypes.c_int),
    "qcau_head_norm_rope": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F,
                             _I32, _P], ctypes.c_int),
    "qcau_rope": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P],
                  ctypes.c_int),
    "qcau_sparse_attn": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                          _F, _I32, _P, _I64, _I64, _I64, _P], ctypes.c_int),
    "qcau_forward_workspace_size": ([_I64, _I64, _I64, _I64, _I64], _SZ),
    "qcau_forward": ([_P, _P, _P, _I32, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                      _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ, _P], ctypes.c_int),
    "qcau_decode_attn_workspace_size": ([_I64, _I64, _I64, _I64], _SZ),
    "qcau_decode_attn_paged": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                _I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "qcau_sparse_attn_fp8_workspace_size": ([_I64, _I64, _I64, _I64], _SZ),
    "qcau_sparse_attn_fp8": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P,
                              _SZ, _P], ctypes.c_int),
    "qcau_prefill_attn_workspace_size": ([_I64, _I64, _I64, _I64, _I64], _SZ),
    "qcau_prefill_attn_paged": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                 _I64, _I64, _I64, _I64, _F, _P, _SZ, _P], ctypes.c_int),
    "qcau_decode_attn_paged_blocked": ([_P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                        _I64, _I64, _I64, _I64, _I64, _I64, _F, _P, _SZ, _P],
                                       ctypes.c_int),
    "qcau_decode_attn_paged_noalloc": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                        _I64, _I64, _I64, _I64, _F, _P], ctypes.c_int),
    "qcau_dequant_fp8_weight": ([_P, _P, _I32, _P, _I64, _I64, _P], ctypes.c_int),
    "qcau_mla_decode_workspace_size": ([ctypes.POINTER(MlaDims)], _SZ),
    "qcau_mla_decode": ([ctypes.POINTER(MlaDims), _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                         _P, _P, _SZ, _P], ctypes.c_int),
    "qcau_mla_decode_q": ([ctypes.POINTER(MlaDims), _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P],
                          ctypes.c_int),
    "qcau_decode_attn_paged_cp": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                   _I64, _I64, _I64, _I64, _I64, _F, _I32, _P], ctypes.c_int),
    "qcau_attn_combine_ranks": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
                                ctypes.c_int),
    "qcau_mla_decode_out": ([ctypes.POINTER(MlaDims), _P, _P, _P, _P, _P, _P, _SZ, _P],
                            ctypes.c_int),
    "qcau_ipc_handle_size": ([], _SZ),
    "qcau_ipc_alloc": ([_SZ, ctypes.POINTER(ctypes.c_void_p), _P], ctypes.c_int),
    "qcau_ipc_open": ([_P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "qcau_ipc_close": ([_P], ctypes.c_int),
    "qcau_ipc_free": ([_P], ctypes.c_int),
    "qcau_decode_attn_paged_cp_p2p": ([_P, _P, _P, _P, _P, _P, _P, ctypes.c_uint32, _P, _I64,
                                       _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                       _I64, _F, _I32, _P], ctypes.c_int),
    "qcau_wait_flags": ([_P, _I64, ctypes.c_uint32, _P], ctypes.c_int),
    "qcau_gopu_workspace_size": ([_I64, _I64, _I64], _SZ),
    "qcau_gopu": ([_P, _P, _P, _P, _I32, _I32, _P, _I32, _I64, _I64, _I64, _I64, _I64, _P, _SZ,
                   _P], ctypes.c_int),
    "qcau_kv_build": ([_P, _P, _I64, _I64, _P, _I64, _F, _P, _P, _I64, _I64, _I64, _I32, _P, _P,
                       _I64, _P], ctypes.c_int),
    "qcau_compress": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I64, _P], ctypes.c_int),
    "qcau_compressor_step": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I64, _P, _F, _P,
                              _I64, _I64, _I32, _I32, _P, _I64, _I64, _P, _P], ctypes.c_int),
    "qcau_rotate_fp4": ([_P, _I64, _I64, _I32, _I32, _P], ctypes.c_int),
    "qcau_indexer_topk_workspace_size": ([_I64, _I64, _I64, _I64], _SZ),
    "qcau_indexer_topk": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                           _I64, _P, _SZ, _P], ctypes.c_int),
    "qcau_indexer_scores_workspace_size": ([_I64, _I64, _I64, _I64], _SZ),
    "qcau_indexer_scores": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P],
                            ctypes.c_int),
    "qcau_indexer_raw_scores": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P],
                                ctypes.c_int),
    "qcau_topk": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P], ctypes.c_int),
    "qcau_index_lists_width": ([_I64, _I64, _I64, _I64, _I64], _I64),
    "qcau_index_lists": ([_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P], ctypes.c_int),
}

_lib = None


class QcauError(RuntimeError):
    """A CUDA / device-side failure reported by the library."""


def lib() -> ctypes.CDLL:
    """Load the library once.  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python deepseek-v4-flash_b200/build.py`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    """Map a qcau_status to the reference's exception types."""
    if rc == QCAU_OK:
        return
    msg = lib().qcau_last_error().decode(errors="replace") or what
    if rc in (QCAU_ERR_INVALID, QCAU_ERR_WORKSPACE):
        raise ValueError(msg)
    if rc == QCAU_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise QcauError(f"{what}: {msg} (status {rc})")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("qcau_b200 runs on CUDA tensors only (no CPU path)")


def device_error(stream: int | None = None) -> int:
    """Synchronise the stream and return (and clear) the device error bits."""
    rc = lib().qcau_device_error(stream if stream is not None else stream_ptr())
    if rc < 0:
        check(rc, "qcau_device_error")
    return rc
