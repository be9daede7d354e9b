"""Index-list producers: what the sparse attention's topk_idxs come from.

Mirrors, on the library's kernels, the reference's functions of the same
names (QCAU/QCAU_inference/inference/model.py; Deepseek_origin/inference/
model.py:246-275 and :380-433 are the same code):

    rotate_activation(x)                      model.py:302-323
    fp4_act_quant(x, 32, inplace=True)        kernel.py:186-200
    get_window_topk_idxs(win, bsz, seqlen, start_pos)        model.py:326-357
    get_compress_topk_idxs(ratio, bsz, seqlen, start_pos, offset)  :359-376
    Indexer.forward's scoring and selection  model.py:512-533

and the concatenation Attention.forward makes of them (model.py:614-624) as
index_lists().  Everything returns int32 index lists on the device, the
dtype the attention reads (the reference casts with .int(), model.py:625).

The Indexer here starts from the projected, RoPE'd queries, the indexer's
compressed key cache and the head weights (the wq_b / weights_proj GEMMs and
the Compressor are the caller's), rotates and FP4-rounds the queries, and
produces topk_idxs with one batched tcgen05 GEMM, one weighted-sum kernel and
one top-k kernel.  Across head-sharded ranks the score rows are all-reduced
in bf16 between the last two, as model.py:520-521 does.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from ._lib import check, lib, require_cuda, stream_ptr


def _rotate_fp4(x: torch.Tensor, hadamard: bool, fp4: bool) -> torch.Tensor:
    require_cuda(x)
    if x.dtype != torch.bfloat16 or x.size(-1) != 128:
        raise ValueError("rows of 128 bf16 values are supported")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    check(lib().qcau_rotate_fp4(x.data_ptr(), x.numel() // 128, 128, int(hadamard), int(fp4),
                                stream_ptr(x.device)), "rotate_fp4")
    return x


def rotate_activation(x: torch.Tensor) -> torch.Tensor:
    """Walsh-Hadamard rotation of the last dimension (128) scaled by 128^-1/2,
    a new bf16 tensor (model.py:302-323)."""
    return _rotate_fp4(x.contiguous().clone(), True, False)


def fp4_act_quant(x: torch.Tensor, block_size: int = 32, inplace: bool = False) -> torch.Tensor:
    """The FP4 e2m1 round trip of 1x32 blocks, in place (kernel.py:186-200 with
    inplace=True; the packed FP4 output of inplace=False has no consumer on
    this path)."""
    if not inplace or block_size != 32:
        raise ValueError("fp4_act_quant: only inplace=True with block_size 32 is supported")
    return _rotate_fp4(x, False, True)


def rotate_fp4_(x: torch.Tensor) -> torch.Tensor:
    """rotate_activation then fp4_act_quant(x, 32, True), in place, in one
    kernel: the indexer's treatment of its queries (model.py:512-514) and of
    its compressed keys (model.py:466-468)."""
    return _rotate_fp4(x, True, True)


def _device(device) -> torch.device:
    return torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)


def index_lists(window_size: int, ratio: int, bsz: int, seqlen: int, start_pos: int,
                offset: int = 0, selected: Optional[torch.Tensor] = None,
                device=None) -> torch.Tensor:
    """The attention's index list [bsz, seqlen, W] int32: the window list,
    then `selected` (the indexer's [bsz, seqlen, k] list) or, with ratio > 0,
    the compressed positions; model.py:614-624."""
    if start_pos > 0 and seqlen != 1:
        raise ValueError("decode steps (start_pos > 0) have seqlen 1")
    dev = _device(device if selected is None else selected.device)
    sel_w = 0
    if selected is not None:
        require_cuda(selected)
        if selected.dtype != torch.int32:
            selected = selected.to(torch.int32)
        selected = selected.contiguous()
        if selected.dim() != 3 or selected.shape[:2] != (bsz, seqlen):
            raise ValueError("selected must be [bsz, seqlen, k]")
        sel_w = selected.size(-1)
    width = lib().qcau_index_lists_width(seqlen, start_pos, window_size, ratio, sel_w)
    if selected is not None and sel_w == 0:
        width = lib().qcau_index_lists_width(seqlen, start_pos, window_size, 0, 0)
    out = torch.empty(bsz, seqlen, width, dtype=torch.int32, device=dev)
    check(lib().qcau_index_lists(out.data_ptr(), bsz, seqlen, start_pos, window_size,
                                 0 if selected is not None else ratio, offset,
                                 selected.data_ptr() if selected is not None and sel_w else None,
                                 sel_w, stream_ptr(dev)), "index_lists")
    return out


def get_window_topk_idxs(window_size: int, bsz: int, seqlen: int, start_pos: int,
                         device=None) -> torch.Tensor:
    """model.py:326-357 as int32 [bsz, seqlen, w] (seqlen 1 at decode)."""
    return index_lists(window_size, 0, bsz, seqlen, start_pos, 0, None, device)


def get_compress_topk_idxs(ratio: int, bsz: int, seqlen: int, start_pos: int, offset: int,
                           device=None) -> torch.Tensor:
    """model.py:359-376 as int32 [bsz, seqlen, w]."""
    w = index_lists(1, ratio, bsz, seqlen, start_pos, offset, None, device)
    return w[..., 1:].contiguous()  # drop the one-wide window part


def raw_scores(q: torch.Tensor, kv_cache: torch.Tensor, t: int) -> torch.Tensor:
    """The indexer's einsum alone (model.py:518): raw [b, s, h, t] bf16 =
    q[b, s, h, :] . kv_cache[b, u, :] for u < t.  Indexer.forward keeps this
    intermediate on chip; this is for inspection."""
    require_cuda(q, kv_cache)
    b, s, h, d = q.shape
    if q.dtype != torch.bfloat16 or kv_cache.dtype != torch.bfloat16:
        raise ValueError("q and kv_cache must be bf16")
    if kv_cache.dim() != 3 or kv_cache.size(2) != d or kv_cache.stride(2) != 1 \
            or kv_cache.stride(1) != d or kv_cache.size(1) < t:
        raise ValueError("kv_cache must be [>= b, >= t, head_dim] with contiguous rows")
    q = q.contiguous()
    tp = (t + 127) // 128 * 128
    raw = torch.empty(b, s, h, tp, dtype=torch.bfloat16, device=q.device)
    check(lib().qcau_indexer_raw_scores(q.data_ptr(), kv_cache.data_ptr(), raw.data_ptr(), b, s,
                                        h, d, t, kv_cache.stride(0) // d, stream_ptr(q.device)),
          "indexer_raw_scores")
    return raw[..., :t]


def topk(score: torch.Tensor, k: int, offset: int = 0, seqlen: Optional[int] = None,
         mask_ratio: int = 0) -> torch.Tensor:
    """Indices [..., k] int32 of the k largest of each row of score [..., T]
    (fp32; score descending, equal scores by index ascending) plus offset, -1
    past the row's candidates.  -inf is never taken; with mask_ratio > 0
    (a prefill) neither are positions >= (s + 1) // mask_ratio of query s,
    s = row % seqlen (model.py:522-533)."""
    require_cuda(score)
    if score.dtype != torch.float32:
        score = score.float()
    score = score.contiguous()
    T = score.size(-1)
    rows = math.prod(score.shape[:-1])
    out = torch.empty(*score.shape[:-1], k, dtype=torch.int32, device=score.device)
    if mask_ratio and not seqlen:
        raise ValueError("the prefill mask needs seqlen")
    check(lib().qcau_topk(score.data_ptr(), out.data_ptr(), rows, T, k, seqlen or 0, mask_ratio,
                          offset, stream_ptr(score.device)), "topk")
    return out


class Indexer:
    """Selection half of the reference Indexer (model.py:478-534).

    n_heads / head_dim / index_topk / compress_ratio are the model's
    (index_n_heads 64, index_head_dim 128, index_topk 512, ratio 4); ranks own
    n_heads / world_size heads, and their score rows are summed over the
    process group as model.py:520-521 does.
    """

    def __init__(self, n_heads: int = 64, head_dim: int = 128, index_topk: int = 512,
                 compress_ratio: int = 4, device="cuda", rank: int = 0, world_size: int = 1,
                 process_group=None):
        if n_heads % world_size:
            raise ValueError("the heads must divide over the ranks")
        if head_dim != 128:
            raise ValueError("index_head_dim 128 is supported")
        if n_heads // world_size > 128:
            raise ValueError("up to 128 index heads a rank are supported")
        self.n_heads, self.head_dim = n_heads, head_dim
        self.n_local_heads = n_heads // world_size
        self.index_topk, self.compress_ratio = index_topk, compress_ratio
        self.softmax_scale = head_dim ** -0.5
        self.rank, self.world_size, self.group = rank, world_size, process_group
        self.device = torch.device(device)
        self._ws = None

    def weight_scale(self) -> float:
        """The factor the reference applies to weights_proj(x) (model.py:516)."""
        return self.softmax_scale * self.n_heads ** -0.5

    def _workspace(self, need: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, q: torch.Tensor, kv_cache: torch.Tensor, weights: torch.Tensor,
                start_pos: int, offset: int, rotate: bool = True) -> torch.Tensor:
        """topk_idxs [b, s, min(index_topk, end_pos // ratio)] int32.

        q [b, s, local heads, 128] bf16 after wq_b and RoPE (rotated and
        FP4-rounded here in a copy unless rotate=False: then q is taken as
        already treated); kv_cache [>= b, rows, 128] bf16, the indexer's
        compressed keys, of which the first end_pos // ratio rows are read;
        weights [b, s, local heads] bf16 = weights_proj(x) * weight_scale().
        """
        require_cuda(q, kv_cache, weights)
        b, s, h, d = q.shape
        if h != self.n_local_heads or d != self.head_dim:
            raise ValueError(f"q must be [b, s, {self.n_local_heads}, {self.head_dim}]")
        if q.dtype != torch.bfloat16 or kv_cache.dtype != torch.bfloat16 or weights.dtype != torch.bfloat16:
            raise ValueError("q, kv_cache and weights must be bf16")
        if tuple(weights.shape) != (b, s, h):
            raise ValueError("weights must be [b, s, heads]")
        if kv_cache.dim() != 3 or kv_cache.size(0) < b or kv_cache.size(2) != d or kv_cache.stride(2) != 1 \
                or kv_cache.stride(1) != d:
            raise ValueError("kv_cache must be [>= b, rows, head_dim] with contiguous rows")
        ratio = self.compress_ratio
        t = (start_pos + s) // ratio
        if t > kv_cache.size(1):
            raise ValueError("kv_cache holds fewer rows than end_pos // ratio")
        k = min(self.index_topk, t)
        q = q.contiguous()
        if rotate:
            q = rotate_fp4_(q.clone())
        weights = weights.contiguous()
        out = torch.empty(b, s, k, dtype=torch.int32, device=q.device)
        st = stream_ptr(q.device)
        kv_rows = kv_cache.stride(0) // d
        if self.world_size == 1:
            need = lib().qcau_indexer_topk_workspace_size(b, s, h, t)
            ws = self._workspace(need)
            check(lib().qcau_indexer_topk(q.data_ptr(), kv_cache.data_ptr(), weights.data_ptr(),
                                          out.data_ptr(), b, s, h, d, t, kv_rows, k, start_pos,
                                          ratio, offset, ws.data_ptr(), ws.numel(), st),
                  "indexer_topk")
            return out
        need = lib().qcau_indexer_scores_workspace_size(b, s, h, t)
        ws = self._workspace(need)
        score = torch.empty(b, s, t, dtype=torch.float32, device=q.device)
        check(lib().qcau_indexer_scores(q.data_ptr(), kv_cache.data_ptr(), weights.data_ptr(),
                                        score.data_ptr(), b, s, h, d, t, kv_rows, ws.data_ptr(),
                                        ws.numel(), st), "indexer_scores")
        part = score.to(torch.bfloat16)  # the reference's bf16 index_score
        dist.all_reduce(part, group=self.group)
        return topk(part.float(), k, offset, s, ratio if start_pos == 0 else 0)

    __call__ = forward
