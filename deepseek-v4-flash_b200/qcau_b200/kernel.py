"""Drop-in for the reference kernel module (Deepseek_origin/inference/kernel.py).

`act_quant`, `fp8_gemm` and `sparse_attn` keep the reference signatures,
argument meaning, output allocation and assertion behaviour, and run on the
sm_100a kernels of libqcau_b200.so.  Installing this module as
``sys.modules["kernel"]`` makes the reference ``model.py`` (which does
``from kernel import ...``, model.py:12) run its QCAU path on these kernels.

fp4_act_quant serves the indexer's in-place FP4 round trip (kernel.py:186-200
with inplace=True).  The FP4 GEMM and the mHC kernel of the reference module
(fp4_gemm, hc_split_sinkhorn) are outside the QCAU path; they are exported so
the import succeeds, and raise NotImplementedError when called.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import check, lib, require_cuda, stream_ptr

__all__ = ["act_quant", "fp8_gemm", "sparse_attn", "fp4_act_quant", "fp4_gemm",
           "hc_split_sinkhorn"]


def _scale_code(scale_dtype: torch.dtype) -> int:
    if scale_dtype == torch.float8_e8m0fnu:
        return _lib.SCALE_E8M0
    if scale_dtype == torch.float32:
        return _lib.SCALE_F32
    raise ValueError(f"unsupported scale dtype {scale_dtype}")


def act_quant(x: torch.Tensor, block_size: int = 128, scale_fmt: Optional[str] = None,
              scale_dtype: torch.dtype = torch.float32, inplace: bool = False):
    """Block-wise FP8 quantization (kernel.py:105-125).

    Returns (y e4m3, s) or, with inplace=True, x overwritten by the FP8 round
    trip.  scale_fmt set -> power-of-two (UE8M0) scales.  Codes and scales are
    bit-exact with the reference.
    """
    N = x.size(-1)
    assert N % block_size == 0
    require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("act_quant: x must be bfloat16")
    z = x.contiguous()
    m = z.numel() // N
    code = _scale_code(scale_dtype)
    if inplace:
        check(lib().qcau_act_quant(z.data_ptr(), None, None, m, N, block_size,
                                   int(scale_fmt is not None), code, 1, stream_ptr(z.device)),
              "act_quant")
        if z.data_ptr() != x.data_ptr():
            x.copy_(z)
        return x
    y = torch.empty_like(z, dtype=torch.float8_e4m3fn)
    s = z.new_empty(*z.size()[:-1], N // block_size, dtype=scale_dtype)
    check(lib().qcau_act_quant(z.data_ptr(), y.data_ptr(), s.data_ptr(), m, N, block_size,
                               int(scale_fmt is not None), code, 0, stream_ptr(z.device)),
          "act_quant")
    return y, s


def fp8_gemm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
             scale_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """C[M,N] = A[M,K] @ B[N,K]^T with per-128 block FP8 scaling (kernel.py:257-273).

    The output dtype is torch.get_default_dtype() (bf16 in the model, fp32
    otherwise), as in the reference.
    """
    assert a.is_contiguous() and b.is_contiguous(), "Input tensors must be contiguous"
    assert a_s.is_contiguous() and b_s.is_contiguous(), (
        "Scaling factor tensors must be contiguous"
    )
    require_cuda(a, a_s, b, b_s)
    K = a.size(-1)
    M = a.numel() // K
    N = b.size(0)
    out_dtype = torch.get_default_dtype()
    if out_dtype == torch.bfloat16:
        oc = _lib.OUT_BF16
    elif out_dtype == torch.float32:
        oc = _lib.OUT_F32
    else:
        raise NotImplementedError(f"fp8_gemm: output dtype {out_dtype} is not supported")
    code = _scale_code(scale_dtype)
    if a_s.dtype != scale_dtype or b_s.dtype != scale_dtype:
        raise ValueError("fp8_gemm: a_s and b_s must both have dtype scale_dtype")
    c = a.new_empty(*a.size()[:-1], N, dtype=out_dtype)
    check(lib().qcau_fp8_gemm(a.data_ptr(), a_s.data_ptr(), b.data_ptr(), b_s.data_ptr(),
                              c.data_ptr(), M, N, K, code, oc, stream_ptr(a.device)), "fp8_gemm")
    return c


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor,
                topk_idxs: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    """Sparse MQA by index gathering + online softmax + sink (kernel.py:355-368).

    q [b, s, h, d] bf16, kv [b, n, d] bf16, attn_sink [h] fp32,
    topk_idxs [b, s, topk] int32 (-1 = invalid) -> o [b, s, h, d] bf16.
    Any head count is accepted (the reference pads to 16 internally).
    """
    require_cuda(q, kv, attn_sink, topk_idxs)
    b, s, h, d = q.size()
    if q.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
        raise ValueError("sparse_attn: q and kv must be bfloat16")
    q = q.contiguous()
    kv = kv.contiguous()
    idx = topk_idxs.to(torch.int32).contiguous()
    sink = attn_sink.to(torch.float32).contiguous()
    o = torch.empty_like(q)
    check(lib().qcau_sparse_attn(q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(),
                                 o.data_ptr(), b, s, h, d, d, kv.size(-1), kv.size(1),
                                 idx.size(-1), float(softmax_scale), 0, None, 0, 0, 0,
                                 stream_ptr(q.device)), "sparse_attn")
    return o


def _outside(name: str):
    def f(*args, **kwargs):
        raise NotImplementedError(f"{name} is outside the QCAU path served by qcau_b200")
    f.__name__ = name
    return f


def fp4_act_quant(x: torch.Tensor, block_size: int = 32, inplace: bool = False) -> torch.Tensor:
    """Block-wise FP4 e2m1 quantisation (kernel.py:186-200).  With
    inplace=True x is overwritten by the round trip (1x32 blocks, power-of-two
    scales, values rounded to e2m1 and scaled back to bf16); the packed FP4
    output of inplace=False feeds only the FP4 GEMM, which is outside this
    library."""
    N = x.size(-1)
    assert N % block_size == 0
    if not inplace:
        raise NotImplementedError("fp4_act_quant without inplace feeds fp4_gemm, outside qcau_b200")
    if block_size != 32:
        raise NotImplementedError("fp4_act_quant: block_size 32 is supported")
    require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("fp4_act_quant: x must be bfloat16")
    z = x.contiguous()
    if z.numel() % 128:
        raise NotImplementedError("fp4_act_quant: the element count must be a multiple of 128")
    # 32-value blocks are contiguous runs of z, so any row width that is a
    # multiple of 32 is processed as rows of 128
    check(lib().qcau_rotate_fp4(z.data_ptr(), z.numel() // 128, 128, 0, 1, stream_ptr(z.device)),
          "fp4_act_quant")
    if z.data_ptr() != x.data_ptr():
        x.copy_(z)
    return x


fp4_gemm = _outside("fp4_gemm")
hc_split_sinkhorn = _outside("hc_split_sinkhorn")
