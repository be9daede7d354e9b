"""Latent KV cache: the KV build of new tokens and the caches it writes.

kv_build replaces the KV half of the reference Attention.forward
(Deepseek_origin/inference/model.py:502-506 and the cache writes :517-533):

    kv = self.kv_norm(self.wkv(x))                     # RMSNorm, model.py:182-195
    apply_rotary_emb(kv[..., -rd:], freqs_cis)         # model.py:231-243
    act_quant(kv[..., :-rd], 64, scale_fmt, scale_dtype, True)   # FP8 round trip
    self.kv_cache[:bsz, start_pos % win] = kv          # window ring (decode)

as one kernel (qcau_kv_build) after the wkv GEMM.  The same kernel writes the
576-wide rows of the absorbed-MLA paged cache (RMSNorm of the 512 latent
values, RoPE of the 64 rope values, no FP8 round trip).

PagedKVCache is the block-table allocator of a multi-step decode loop: it hands
out 64-token pages of one physical cache to sequences, keeps their block
tables and lengths on the device in the layout the decode attention reads, and
gives the cache row of every appended token.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import check, lib, require_cuda, stream_ptr


def kv_build(kv: torch.Tensor, norm_weight: Optional[torch.Tensor], freqs_cis: torch.Tensor,
             positions: torch.Tensor, *, rope_dim: int = 64, norm_dim: Optional[int] = None,
             quant_dims: Optional[int] = None, scale_fmt: Optional[str] = "ue8m0",
             eps: float = 1e-6, out: Optional[torch.Tensor] = None,
             cache: Optional[torch.Tensor] = None, slots: Optional[torch.Tensor] = None,
             inplace: bool = False, return_rows: bool = True) -> Optional[torch.Tensor]:
    """KV rows of new tokens from the wkv projection.

    kv [..., d] bf16 (d a multiple of 64); norm_weight [norm_dim] (fp32 or
    bf16, None = ones); freqs_cis [npos, rope_dim/2] complex64 or [npos,
    rope_dim/2, 2] fp32; positions [...] int (one per row).  norm_dim defaults
    to d (V4 rows) and quant_dims to d - rope_dim (the reference's FP8 round
    trip of the non-rope values); pass quant_dims=0 for the absorbed-MLA cache
    row.  scale_fmt "ue8m0" gives power-of-two block scales (the model's
    setting, model.py:777), None fp32 amax/448 scales.

    Writes the built rows to `out` (allocated when None; the input itself
    when inplace) and, when `cache` is given, row r also to
    cache.view(-1, d)[slots[r]] (slots -1: not written).  With
    return_rows=False only the cache is written and None is returned.
    """
    require_cuda(kv)
    d = kv.size(-1)
    if kv.dtype != torch.bfloat16:
        raise ValueError("kv must be bf16")
    rows = kv.numel() // d
    kv = kv.contiguous()
    norm_dim = d if norm_dim is None else norm_dim
    quant_dims = d - rope_dim if quant_dims is None else quant_dims
    w = None
    if norm_weight is not None and norm_dim > 0:
        w = norm_weight.to(device=kv.device, dtype=torch.float32).contiguous()
        if w.numel() != norm_dim:
            raise ValueError(f"norm_weight has {w.numel()} values, expected {norm_dim}")
    if freqs_cis.is_complex():
        freqs = torch.view_as_real(freqs_cis).to(kv.device).contiguous()
    else:
        freqs = freqs_cis.to(device=kv.device, dtype=torch.float32).contiguous()
    pos = positions.to(device=kv.device, dtype=torch.int32).reshape(-1).contiguous()
    if pos.numel() != rows:
        raise ValueError("one position per row is needed")
    if not return_rows:
        if cache is None:
            raise ValueError("return_rows=False needs a cache")
        dst = None
    elif inplace:
        dst = kv
    else:
        dst = torch.empty_like(kv) if out is None else out
    cache_rows = 0
    sl = None
    if cache is not None:
        require_cuda(cache)
        if cache.size(-1) != d or cache.dtype != torch.bfloat16:
            raise ValueError("cache rows must be bf16 of the kv width")
        cache_rows = cache.numel() // d
        if slots is None:
            raise ValueError("a cache needs slots")
        sl = slots.to(device=kv.device, dtype=torch.int32).reshape(-1).contiguous()
        if sl.numel() != rows:
            raise ValueError("one slot per row is needed")
    check(lib().qcau_kv_build(kv.data_ptr(), None if dst is None else dst.data_ptr(), rows, d,
                              None if w is None else w.data_ptr(), norm_dim, float(eps),
                              freqs.data_ptr(), pos.data_ptr(), freqs.size(0), rope_dim,
                              quant_dims, 1 if scale_fmt == "ue8m0" else 0,
                              None if cache is None else cache.data_ptr(),
                              None if sl is None else sl.data_ptr(), cache_rows,
                              stream_ptr(kv.device)), "kv_build")
    return dst


def window_slots(bsz: int, seqlen: int, start_pos: int, window: int, ring_rows: int,
                 device) -> torch.Tensor:
    """Cache rows of the reference's sliding-window ring for tokens
    [start_pos, start_pos + seqlen) of bsz sequences (model.py:517-533): the
    ring of sequence b is rows [b * ring_rows, b * ring_rows + window), token
    at position p goes to row p % window, and in a prefill only the last
    `window` tokens are kept (earlier ones get -1)."""
    pos = torch.arange(start_pos, start_pos + seqlen, device=device, dtype=torch.int64)
    keep = pos >= start_pos + seqlen - window
    slot = torch.where(keep, pos % window, torch.full_like(pos, -1))
    base = torch.arange(bsz, device=device, dtype=torch.int64).unsqueeze(1) * ring_rows
    out = torch.where(slot.unsqueeze(0) >= 0, base + slot.unsqueeze(0), torch.full_like(base, -1))
    return out.to(torch.int32).reshape(-1)


class PagedKVCache:
    """A paged latent cache [num_pages, page_size, width] bf16 shared by up to
    max_seqs sequences, with their block tables [max_seqs, max_pages] and
    lengths [max_seqs] on the device (the layout qcau_decode_attn_paged reads).

    Pages are handed out from a free list as sequences grow and returned when
    a sequence is released.  append() reserves room for new tokens and returns
    each token's cache row (page * page_size + offset) for kv_build.
    """

    def __init__(self, num_pages: int, max_seqs: int, max_pages: int, width: int = 576,
                 page_size: int = 64, device="cuda", dtype=torch.bfloat16):
        self.num_pages, self.max_seqs, self.max_pages = num_pages, max_seqs, max_pages
        self.page_size, self.width = page_size, width
        self.device = torch.device(device)
        self.cache = torch.zeros(num_pages, page_size, width, device=self.device, dtype=dtype)
        self.block_table = torch.zeros(max_seqs, max_pages, device=self.device, dtype=torch.int32)
        self.seqlens = torch.zeros(max_seqs, device=self.device, dtype=torch.int32)
        self._free = list(range(num_pages - 1, -1, -1))
        self._pages: list[list[int]] = [[] for _ in range(max_seqs)]
        self._len = [0] * max_seqs

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def length(self, seq: int) -> int:
        return self._len[seq]

    def append(self, seqs: Sequence[int], counts: Sequence[int]) -> torch.Tensor:
        """Reserve counts[i] new tokens for sequence seqs[i]; returns the cache
        rows of the new tokens [sum(counts)] int32 (sequence by sequence, in
        position order).  Raises MemoryError when the pages run out and
        ValueError past max_pages."""
        rows = []
        for s, n in zip(seqs, counts):
            start = self._len[s]
            end = start + n
            need = (end + self.page_size - 1) // self.page_size
            if need > self.max_pages:
                raise ValueError(f"sequence {s} would need {need} pages (max_pages {self.max_pages})")
            grow = need - len(self._pages[s])
            if grow > len(self._free):
                raise MemoryError(f"cache has {len(self._free)} free pages, {grow} needed")
            for _ in range(grow):
                self._pages[s].append(self._free.pop())
            for p in range(start, end):
                rows.append(self._pages[s][p // self.page_size] * self.page_size + p % self.page_size)
            self._len[s] = end
        self._sync(seqs)
        return torch.tensor(rows, dtype=torch.int32, device=self.device)

    def positions(self, seqs: Sequence[int], counts: Sequence[int]) -> torch.Tensor:
        """Positions of the last counts[i] tokens of each sequence (after append)."""
        pos = []
        for s, n in zip(seqs, counts):
            pos.extend(range(self._len[s] - n, self._len[s]))
        return torch.tensor(pos, dtype=torch.int32, device=self.device)

    def release(self, seq: int) -> None:
        """Return the sequence's pages to the free list."""
        self._free.extend(reversed(self._pages[seq]))
        self._pages[seq] = []
        self._len[seq] = 0
        self._sync([seq])

    def _sync(self, seqs: Sequence[int]) -> None:
        for s in set(seqs):
            row = torch.zeros(self.max_pages, dtype=torch.int32)
            if self._pages[s]:
                row[:len(self._pages[s])] = torch.tensor(self._pages[s], dtype=torch.int32)
            self.block_table[s].copy_(row)
            self.seqlens[s] = self._len[s]


class Compressor:
    """The KV compressor (QCAU/QCAU_inference/inference/model.py:376-476,
    Compressor.forward) after its two fp32 projections: gated pooling of
    every `compress_ratio` tokens (qcau_compress), then the compressor's
    RMSNorm, RoPE at the group's first position and, for the attention's
    compressor, the FP8 round trip of the non-rope values (qcau_kv_build), or
    for the indexer's (rotate=True) the Hadamard rotation and FP4 round trip
    (qcau_rotate_fp4); the rows are written to the cache.

    head_dim / rope_dim / compress_ratio are the layer's (512 or 128, 64, 4 or
    128); the ratio-4 compressor overlaps its windows (model.py:387).  The
    cache is the caller's [max_batch, rows, head_dim] bf16 tensor; compressed
    row i of sequence b goes to cache[b, cache_offset + i] (the attention's
    compressed rows follow its window ring: cache_offset = window_size,
    model.py:599-600).  freqs_cis [max_seq, rope_dim / 2] complex64.
    """

    def __init__(self, head_dim: int, compress_ratio: int = 4, rope_dim: int = 64,
                 rotate: bool = False, max_batch: int = 4, norm_eps: float = 1e-6,
                 scale_fmt: Optional[str] = "ue8m0", device="cuda"):
        self.d, self.ratio, self.rd, self.rotate = head_dim, compress_ratio, rope_dim, rotate
        self.overlap = compress_ratio == 4
        coff = 2 if self.overlap else 1
        self.eps, self.scale_fmt = norm_eps, scale_fmt
        self.device = torch.device(device)
        dev = self.device
        self.ape = torch.zeros(compress_ratio, coff * head_dim, device=dev)
        self.norm_weight = torch.ones(head_dim, device=dev)
        self.kv_state = torch.zeros(max_batch, coff * compress_ratio, coff * head_dim, device=dev)
        self.score_state = torch.full_like(self.kv_state, float("-inf"))
        self.kv_cache: Optional[torch.Tensor] = None
        self.cache_offset = 0
        self.freqs_cis: Optional[torch.Tensor] = None

    def forward(self, kv: torch.Tensor, score: torch.Tensor, start_pos: int) -> Optional[torch.Tensor]:
        """kv, score [b, s, cw] fp32 (wkv / wgate of x.float(); cw = 2 * head_dim
        with overlap): the compressed rows [b, n, head_dim] bf16 written to the
        cache (n = s // ratio at prefill, 1 at a decode step that closes a
        group), or None when a decode step closes none."""
        require_cuda(kv, score)
        b, s, cw = kv.shape
        if kv.dtype != torch.float32 or score.dtype != torch.float32 or score.shape != kv.shape:
            raise ValueError("kv and score must be fp32 of the same shape")
        if cw != (2 if self.overlap else 1) * self.d:
            raise ValueError("projection width must be 2 * head_dim with overlap, else head_dim")
        if b > self.kv_state.size(0):
            raise ValueError("batch above max_batch")
        if self.kv_cache is None or self.freqs_cis is None:
            raise ValueError("assign kv_cache and freqs_cis first")
        if not self.kv_cache.is_contiguous() or self.kv_cache.dtype != torch.bfloat16:
            raise ValueError("kv_cache must be a contiguous bf16 [batch, rows, head_dim] tensor")
        ratio, d = self.ratio, self.d
        kv, score = kv.contiguous(), score.contiguous()
        if start_pos == 0:
            n = s // ratio
        else:
            if s != 1:
                raise ValueError("decode steps have one token")
            n = 1 if (start_pos + 1) % ratio == 0 else 0
        first = 0 if start_pos == 0 else start_pos // ratio
        if n and self.cache_offset + first + n > self.kv_cache.size(1):
            raise ValueError("the compressed rows do not fit the cache")
        freqs = self.freqs_cis
        freqs = torch.view_as_real(freqs) if freqs.is_complex() else freqs
        freqs = freqs.to(device=kv.device, dtype=torch.float32).contiguous()
        w = self.norm_weight.to(device=kv.device, dtype=torch.float32).contiguous()
        ape = self.ape.to(device=kv.device, dtype=torch.float32).contiguous()
        rows = torch.empty(b, max(n, 1), d, device=kv.device, dtype=torch.bfloat16)
        # the state of the first b sequences (the reference's state[:bsz]) is
        # contiguous because the state rows of a sequence are
        ks, ss = self.kv_state[:b], self.score_state[:b]
        check(lib().qcau_compressor_step(
            kv.data_ptr(), score.data_ptr(), ape.data_ptr(), ks.data_ptr(), ss.data_ptr(), b, s, d,
            ratio, int(self.overlap), start_pos, w.data_ptr(), self.eps, freqs.data_ptr(),
            freqs.size(0), self.rd, int(self.rotate),
            1 if self.scale_fmt == "ue8m0" else 0, self.kv_cache.data_ptr(), self.kv_cache.size(1),
            self.cache_offset, rows.data_ptr(), stream_ptr(kv.device)), "compressor_step")
        if n == 0:
            return None
        return rows[:, :n]

    __call__ = forward
