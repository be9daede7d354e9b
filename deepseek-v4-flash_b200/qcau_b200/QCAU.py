"""Drop-in QCAU block (QCAU/QCAU_inference/inference/QCAU.py:245-319).

Same keyword-only signature, argument meaning and ValueError messages as the
reference, plus the extras its variants accept (``prob_dtype`` from
check/QCAU.py:300, ``use_tilelang_sparse`` / ``head_chunk`` from
framework/models/QCAU.py:444-445; they select nothing here).

Paths
  * ``w_uq`` is the model's ``wq_b`` (a Linear whose weight is FP8 e4m3 with a
    ``.scale``), or that FP8 weight tensor itself: one fused call
    ``qcau_forward`` runs act_quant -> FP8 GEMM -> per-head RMSNorm -> RoPE ->
    attention -> inverse RoPE on the sm_100a kernels.
  * any other callable, or a weight tensor in one of the reference's layouts:
    the projection runs first (the callable itself, or a plain library GEMM
    for a tensor), then RMSNorm + RoPE, attention and inverse RoPE run on the
    library kernels.
Computation is bf16 (as in the model); the attention core uses the reference
kernel's 64-key tile whatever ``tile_size`` says (it must still be > 0).
"""
from __future__ import annotations

from typing import Callable, Optional, Union

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_ptr

WeightOrProjector = Union[torch.Tensor, Callable[[torch.Tensor], torch.Tensor]]


def _freqs_view(freqs_cis: torch.Tensor, seqlen: int, start_pos: int, n_pairs: int):
    """Reference position selection (QCAU.py:46-57) -> (fp32 [P, n_pairs, 2], pos0)."""
    if freqs_cis.ndim != 2:
        raise ValueError("freqs_cis must have shape [S, rope_head_dim // 2]")
    if freqs_cis.size(-1) != n_pairs:
        raise ValueError("freqs_cis has the wrong number of rotary pairs")
    if freqs_cis.size(0) == seqlen:
        pos0 = 0
    elif freqs_cis.size(0) >= start_pos + seqlen:
        pos0 = start_pos
    else:
        raise ValueError("freqs_cis does not cover the QCAU query positions")
    if not freqs_cis.is_complex():
        raise ValueError("freqs_cis must be complex")
    f = torch.view_as_real(freqs_cis.to(torch.complex64))
    return f.contiguous(), pos0


def _fp8_weight(w_uq):
    """Return (weight e4m3 [N, Dc], scale) if w_uq is an FP8 projector, else None."""
    w = w_uq
    if not isinstance(w_uq, torch.Tensor):
        w = getattr(w_uq, "weight", None)
        if not isinstance(w, torch.Tensor) or getattr(w_uq, "bias", None) is not None:
            return None
    if w.dtype != torch.float8_e4m3fn or w.ndim != 2:
        return None
    scale = getattr(w, "scale", None)
    if scale is None:
        return None
    return w, scale


def QCAU(
    *,
    c_q: torch.Tensor,
    w_uq: WeightOrProjector,
    kv: torch.Tensor,
    topk_idxs: torch.Tensor,
    attn_sink: torch.Tensor,
    freqs_cis: torch.Tensor,
    q_head_norm_weight: Optional[torch.Tensor] = None,
    n_local_heads: Optional[int] = None,
    head_dim: int = 512,
    rope_head_dim: int = 64,
    start_pos: int = 0,
    norm_eps: float = 1e-6,
    softmax_scale: Optional[float] = None,
    tile_size: int = 64,
    prob_dtype: Optional[torch.dtype] = torch.bfloat16,
    use_tilelang_sparse: bool = True,
    head_chunk: int = 16,
) -> torch.Tensor:
    """Run the Query-Core Attention Unit; returns o [B, S, H_local, Dh] bf16."""
    if c_q.ndim != 3:
        raise ValueError("c_q must have shape [B,S,D_C]")
    if kv.ndim != 3:
        raise ValueError("kv must have shape [B,N,Dh]")
    if topk_idxs.ndim != 3:
        raise ValueError("topk_idxs must have shape [B,S,K]")
    if c_q.size(0) != kv.size(0) or c_q.size(0) != topk_idxs.size(0):
        raise ValueError("c_q, kv and topk_idxs batch dimensions must match")
    if c_q.size(1) != topk_idxs.size(1):
        raise ValueError("c_q and topk_idxs sequence dimensions must match")
    if kv.size(1) == 0:
        raise ValueError("kv must contain at least one latent row")
    if tile_size <= 0:
        raise ValueError("tile_size must be positive")
    if prob_dtype not in (torch.bfloat16, None):
        raise ValueError("prob_dtype must be torch.bfloat16 or None")
    if rope_head_dim % 2 != 0:
        raise ValueError("rope_head_dim must be even")
    require_cuda(c_q, kv, topk_idxs, attn_sink)
    if c_q.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
        raise ValueError("qcau_b200 computes in bfloat16: c_q and kv must be bfloat16")

    B, S, Dc = c_q.shape
    idx = topk_idxs.to(torch.int32).contiguous()
    sink = attn_sink.to(device=c_q.device, dtype=torch.float32).contiguous()
    gamma = None
    fp8 = _fp8_weight(w_uq)

    if fp8 is not None:
        w, w_scale = fp8
        if w.size(1) != Dc:
            raise ValueError("W_UQ input width does not match D_C")
        if w.size(0) % head_dim != 0:
            raise ValueError("W_UQ output is not divisible by head_dim")
        H = w.size(0) // head_dim
        if n_local_heads is not None and H != n_local_heads:
            raise ValueError("W_UQ output does not match n_local_heads")
        if q_head_norm_weight is not None:
            if tuple(q_head_norm_weight.shape) != (H, head_dim):
                raise ValueError(f"q_head_norm_weight must have shape {(H, head_dim)}")
            gamma = q_head_norm_weight.to(device=c_q.device, dtype=torch.bfloat16).contiguous()
        if head_dim != kv.size(-1):
            raise ValueError("Query Up head dimension must match KV width")
        if sink.numel() != H:
            raise ValueError("attn_sink must match the number of local query heads")
        if rope_head_dim > head_dim:
            raise ValueError("last dimension is smaller than rope_head_dim")
        freqs, pos0 = _freqs_view(freqs_cis.to(c_q.device), S, start_pos, rope_head_dim // 2)
        if softmax_scale is None:
            softmax_scale = head_dim ** -0.5
        if w_scale.dtype == torch.float8_e8m0fnu:
            w_code, round_act = _lib.SCALE_E8M0, 1
        elif w_scale.dtype == torch.float32:
            w_code, round_act = _lib.SCALE_F32, 0
        else:
            raise ValueError(f"unsupported W_UQ scale dtype {w_scale.dtype}")
        c = c_q.contiguous()
        kvc = kv.contiguous()
        o = torch.empty(B, S, H, head_dim, device=c_q.device, dtype=torch.bfloat16)
        ws_bytes = lib().qcau_forward_workspace_size(B, S, H, head_dim, Dc)
        ws = torch.empty(max(ws_bytes, 1), device=c_q.device, dtype=torch.uint8)
        check(lib().qcau_forward(c.data_ptr(), w.contiguous().data_ptr(),
                                 w_scale.contiguous().data_ptr(), w_code, round_act, ptr(gamma),
                                 kvc.data_ptr(), idx.data_ptr(), sink.data_ptr(),
                                 freqs.data_ptr(), o.data_ptr(), B, S, H, head_dim, Dc,
                                 kvc.size(1), idx.size(-1), rope_head_dim, freqs.size(0), pos0,
                                 float(norm_eps), float(softmax_scale), ws.data_ptr(), ws_bytes,
                                 stream_ptr(c_q.device)), "QCAU")
        return o

    # ---- projection outside the library, then the library kernels
    if callable(w_uq) and not isinstance(w_uq, torch.Tensor):
        q_projected = w_uq(c_q)
    elif isinstance(w_uq, torch.Tensor) and w_uq.ndim == 2:
        q_projected = torch.matmul(c_q, w_uq.to(c_q.dtype).transpose(-1, -2))
    elif isinstance(w_uq, torch.Tensor) and w_uq.ndim == 3:
        if w_uq.size(0) == Dc:
            q_projected = torch.einsum("bsd,dhc->bshc", c_q, w_uq.to(c_q.dtype))
        elif w_uq.size(1) == Dc:
            q_projected = torch.einsum("bsd,hdc->bshc", c_q, w_uq.to(c_q.dtype))
        else:
            raise ValueError("3D W_UQ must be [D_C,H,Dh] or [H,D_C,Dh]")
    else:
        raise ValueError("W_UQ must be a tensor or callable projector")

    if q_projected.ndim == 3:
        if q_projected.size(-1) % head_dim != 0:
            raise ValueError("W_UQ output is not divisible by head_dim")
        H = q_projected.size(-1) // head_dim
        if n_local_heads is not None and H != n_local_heads:
            raise ValueError("W_UQ output does not match n_local_heads")
        q = q_projected.unflatten(-1, (H, head_dim))
    elif q_projected.ndim == 4:
        if q_projected.size(-1) != head_dim:
            raise ValueError("W_UQ output head dimension does not match head_dim")
        if n_local_heads is not None and q_projected.size(-2) != n_local_heads:
            raise ValueError("W_UQ output does not match n_local_heads")
        q = q_projected
        H = q.size(-2)
    else:
        raise ValueError("W_UQ must produce [B,S,H*Dh] or [B,S,H,Dh]")
    if q_head_norm_weight is not None:
        expected = (q.size(-2), q.size(-1))
        if tuple(q_head_norm_weight.shape) != expected:
            raise ValueError(f"q_head_norm_weight must have shape {expected}")
        gamma = q_head_norm_weight.to(device=c_q.device, dtype=torch.bfloat16).contiguous()
    if q.size(-1) < rope_head_dim:
        raise ValueError("last dimension is smaller than rope_head_dim")
    freqs, pos0 = _freqs_view(freqs_cis.to(c_q.device), S, start_pos, rope_head_dim // 2)
    q = q.to(torch.bfloat16).contiguous().clone()
    stream = stream_ptr(c_q.device)
    check(lib().qcau_head_norm_rope(q.data_ptr(), ptr(gamma), freqs.data_ptr(), B, S, H,
                                    head_dim, head_dim, rope_head_dim, freqs.size(0), pos0,
                                    float(norm_eps), 1, stream), "QCAU query-up norm/RoPE")
    if q.size(-1) != kv.size(-1):
        raise ValueError("Query Up head dimension must match KV width")
    if sink.numel() != H:
        raise ValueError("attn_sink must match the number of local query heads")
    if softmax_scale is None:
        softmax_scale = q.size(-1) ** -0.5
    kvc = kv.contiguous()
    o = torch.empty(B, S, H, head_dim, device=c_q.device, dtype=torch.bfloat16)
    check(lib().qcau_sparse_attn(q.data_ptr(), kvc.data_ptr(), sink.data_ptr(), idx.data_ptr(),
                                 o.data_ptr(), B, S, H, head_dim, head_dim, kvc.size(-1),
                                 kvc.size(1), idx.size(-1), float(softmax_scale), 1,
                                 freqs.data_ptr(), rope_head_dim, freqs.size(0), pos0, stream),
          "QCAU attention")
    return o
