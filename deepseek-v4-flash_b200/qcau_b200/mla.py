"""Absorbed-MLA decode layer on the QCAU kernels, head-sharded over ranks.

One decode step for `batch` sequences (one new token each):

    q      = wq_b(act_quant(q_lora))                 FP8 block-scaled GEMM
    q_rope = RoPE(q[..., 128:192], position)         freqs_cis at each position
    q_lat  = q_nope . W_UK[h]                        absorption into the latent space
    o_lat  = softmax(q_abs . cache^T * scale) . cache[..., :512]   paged decode attention
    o_v    = o_lat . W_UV[h]^T                       v-up
    y      = wo(act_quant(o_v))                      row-parallel FP8 GEMM
    y      = all_reduce(y) over the head shards      NCCL over NVLink

Heads are sharded like the reference's tensor parallelism: wq_b / wkv_b are
column-parallel (this rank's heads, ColumnParallelLinear model.py:155-163),
wo is row-parallel with an all-reduce of the partial outputs
(RowParallelLinear model.py:166-180).  The latent cache is shared by all heads
(MQA).  Two ways to run the attention of N ranks:

  attn_split="heads"    each rank attends with its own heads over the whole
                        cache: every rank streams all of it, so the step time
                        barely falls with N;
  attn_split="rows"     (the default) each rank attends with all heads over 1/N of the
                        sequences: an all-to-all of the absorbed queries
                        (B/N rows x h/N heads per pair of ranks) in, one of
                        the bf16 outputs back; each rank streams the pages
                        of its own sequences and nothing is merged across
                        ranks (a batch that does not divide by the ranks
                        runs the context split);
  attn_split="context"  the ranks all-gather their absorbed queries, each
                        attends with all heads over 1/N of every sequence's
                        tiles, and an all-to-all brings each rank the
                        partial softmax states of its heads, which it merges
                        before the v-up.  Each rank streams 1/N of the cache
                        and exchanges b*h/N*(N-1)*(512+2)*4 bytes:
    exchange="nccl"     with an NCCL all-to-all (the faster one measured);
    exchange="p2p"      stored by the attention kernel itself into the
                        owning rank's receive area (CUDA IPC peer memory
                        over NVLink), with a flag per source rank.  Its
                        epilogue's 16-byte remote stores hold up each CTA
                        pair, which costs more than the all-to-all at 8 GPUs.

The reference's V4 attention has no wkv_b; this layer serves the absorbed-MLA
decode configuration (kv_lora 512 + rope 64 cache rows, d_nope 128, d_v 128).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, lib, stream_ptr


@dataclass
class MLAConfig:
    n_heads: int = 128          # total heads (all ranks)
    dc: int = 1536              # q_lora_rank
    d_nope: int = 128
    d_rope: int = 64
    kv_lora: int = 512
    d_v: int = 128
    dim: int = 7168
    page_size: int = 64
    rope_theta: float = 10000.0
    act_round_scale: bool = False   # True: UE8M0 activation scales (scale_fmt="ue8m0")

    @property
    def softmax_scale(self) -> float:
        return (self.d_nope + self.d_rope) ** -0.5


def quantize_weight_fp8(w: torch.Tensor, e8m0: bool = False):
    """FP8 e4m3 weight with one scale per 128 x 128 block (s = amax/448).

    Weight preparation (not on the decode path).  Rows and columns must be
    multiples of 128.
    """
    R, C = w.shape
    blk = w.float().view(R // 128, 128, C // 128, 128)
    s = blk.abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0
    if e8m0:
        s = torch.exp2(torch.ceil(torch.log2(s)))
    q = (blk / s[:, None, :, None]).clamp(-448, 448).view(R, C).to(torch.float8_e4m3fn)
    return q, (s.to(torch.float8_e8m0fnu) if e8m0 else s.contiguous())


def shard_weights(cfg: MLAConfig, rank: int, world_size: int, wq_b, wq_b_scale, wkv_b,
                  wkv_b_scale, wo, wo_scale):
    """This rank's slice of the full FP8 weights and their 128x128 block scales.

    Heads are split evenly: rows of wq_b [H*(d_nope+d_rope), dc] and of wkv_b
    [H*(d_nope+d_v), kv_lora] (column-parallel, ColumnParallelLinear
    model.py:155-163), columns of wo [dim, H*d_v] (row-parallel,
    RowParallelLinear model.py:166-180, whose partial outputs are summed).
    """
    if cfg.n_heads % world_size:
        raise ValueError("n_heads must be divisible by the number of ranks")
    hl = cfg.n_heads // world_size
    dq, dkv = cfg.d_nope + cfg.d_rope, cfg.d_nope + cfg.d_v
    if (hl * dq) % 128 or (hl * dkv) % 128 or (hl * cfg.d_v) % 128:
        raise ValueError("a head shard must cover whole 128-row/column scale blocks")
    r = rank
    return (wq_b[r * hl * dq:(r + 1) * hl * dq],
            wq_b_scale[r * hl * dq // 128:(r + 1) * hl * dq // 128],
            wkv_b[r * hl * dkv:(r + 1) * hl * dkv],
            wkv_b_scale[r * hl * dkv // 128:(r + 1) * hl * dkv // 128],
            wo[:, r * hl * cfg.d_v:(r + 1) * hl * cfg.d_v],
            wo_scale[:, r * hl * cfg.d_v // 128:(r + 1) * hl * cfg.d_v // 128])


def precompute_freqs_cis(rope_dim: int, npos: int, theta: float, device) -> torch.Tensor:
    """RoPE table [npos, rope_dim/2, 2] fp32 (re, im), model.py:198-228 without YaRN."""
    freqs = 1.0 / (theta ** (torch.arange(0, rope_dim, 2, dtype=torch.float32) / rope_dim))
    t = torch.arange(npos, dtype=torch.float32)
    ang = torch.outer(t, freqs)
    return torch.view_as_real(torch.polar(torch.ones_like(ang), ang)).contiguous().to(device)


class MLADecodeLayer:
    """Holds this rank's weight shards and runs one decode step per call."""

    def __init__(self, cfg: MLAConfig, device, rank: int = 0, world_size: int = 1,
                 process_group=None, attn_split: str = "rows", exchange: str = "nccl",
                 cuda_graphs: bool = False):
        if cfg.n_heads % world_size:
            raise ValueError("n_heads must be divisible by the number of ranks")
        if attn_split not in ("heads", "context", "rows"):
            raise ValueError("attn_split must be 'heads', 'context' or 'rows'")
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.attn_split = attn_split
        self.exchange = exchange
        self._cp = None
        self._rows = None
        self._prefill = None
        self._peer = None
        # (stage name, CUDA event) marks of the split steps, recorded on the
        # compute stream when a caller sets this to a list (stage timing)
        self.stage_events = None
        # cuda_graphs: forward() replays each decode step from a CUDA graph
        # (its kernels and collectives, captured after one eager step), one
        # graph per set of tensors the step reads and writes; while
        # stage_events is set, or without an output tensor, steps run eagerly
        self.cuda_graphs = cuda_graphs
        self._graphs = {}
        self.cfg = cfg
        self.device = torch.device(device)
        self.rank, self.world_size = rank, world_size
        self.group = process_group
        self.n_local = cfg.n_heads // world_size
        self.wq_b = self.wq_b_scale = None
        self.wkv_b_bf16 = None
        self.wo = self.wo_scale = None
        self._ws = None

    # ------------------------------------------------------------ weights
    def load_weights(self, wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo, wo_scale,
                     sharded: bool = False):
        """Load FP8 weights with 128x128 block scales.

        Unsharded tensors (sharded=False) are sliced to this rank's heads:
        wq_b [H*(d_nope+d_rope), dc], wkv_b [H*(d_nope+d_v), kv_lora],
        wo [dim, H*d_v].  Scales are fp32 or float8_e8m0fnu.
        """
        if not sharded and self.world_size > 1:
            wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo, wo_scale = shard_weights(
                self.cfg, self.rank, self.world_size, wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo,
                wo_scale)
        dev = self.device
        self.wq_b = wq_b.to(dev).contiguous()
        self.wq_b_scale = wq_b_scale.to(dev).contiguous()
        self.wo = wo.to(dev).contiguous()
        self.wo_scale = wo_scale.to(dev).contiguous()
        if self.wq_b_scale.dtype != self.wo_scale.dtype:
            raise ValueError("wq_b and wo scales must share a dtype")
        wkv = wkv_b.to(dev).contiguous()
        wkv_s = wkv_b_scale.to(dev).contiguous()
        self.wkv_b_bf16 = torch.empty(wkv.shape, device=dev, dtype=torch.bfloat16)
        check(lib().qcau_dequant_fp8_weight(wkv.data_ptr(), wkv_s.data_ptr(),
                                            self._scale_code(wkv_s.dtype),
                                            self.wkv_b_bf16.data_ptr(), wkv.size(0), wkv.size(1),
                                            stream_ptr(dev)), "dequant wkv_b")

    @staticmethod
    def _scale_code(dt):
        if dt == torch.float8_e8m0fnu:
            return _lib.SCALE_E8M0
        if dt == torch.float32:
            return _lib.SCALE_F32
        raise ValueError(f"unsupported scale dtype {dt}")

    def random_weights(self, seed: int = 0, std: float = 0.02, e8m0: bool = False):
        """Random-init weights ~N(0, std) quantised to FP8 with block scales.

        Every rank draws the full (unsharded) tensors from the same seed and
        keeps its shard, so a multi-rank layer equals the single-rank one.
        Returns the full quantised tensors.
        """
        c = self.cfg
        g = torch.Generator(device=self.device).manual_seed(seed)
        H = c.n_heads
        dq, dkv = c.d_nope + c.d_rope, c.d_nope + c.d_v

        def rnd(r, k):
            return torch.randn(r, k, generator=g, device=self.device) * std

        wq, wqs = quantize_weight_fp8(rnd(H * dq, c.dc), e8m0)
        wkv, wkvs = quantize_weight_fp8(rnd(H * dkv, c.kv_lora), e8m0)
        wo, wos = quantize_weight_fp8(rnd(c.dim, H * c.d_v), e8m0)
        self.load_weights(wq, wqs, wkv, wkvs, wo, wos)
        return (wq, wqs, wkv, wkvs, wo, wos)

    # ------------------------------------------------------------ step
    def dims(self, batch: int, max_pages: int, num_pages: int, max_seqlen: int, npos: int,
             out_fp32: bool = False) -> _lib.MlaDims:
        c = self.cfg
        d = _lib.MlaDims()
        d.batch, d.n_heads, d.dc = batch, self.n_local, c.dc
        d.d_nope, d.d_rope, d.kv_lora, d.d_v, d.dim = c.d_nope, c.d_rope, c.kv_lora, c.d_v, c.dim
        d.page_size, d.max_pages, d.num_pages = c.page_size, max_pages, num_pages
        d.max_seqlen, d.npos = max_seqlen, npos
        d.softmax_scale = c.softmax_scale
        d.w_scale_dtype = self._scale_code(self.wq_b_scale.dtype)
        d.act_round_scale = int(c.act_round_scale)
        d.out_dtype = _lib.OUT_F32 if out_fp32 else _lib.OUT_BF16
        return d

    def workspace(self, d: _lib.MlaDims) -> torch.Tensor:
        need = lib().qcau_mla_decode_workspace_size(d)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), device=self.device, dtype=torch.uint8)
        return self._ws

    def forward_local(self, q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen,
                      y: Optional[torch.Tensor] = None, out_fp32: bool = False) -> torch.Tensor:
        """This rank's partial y [batch, dim] (no all-reduce)."""
        B = q_lora.size(0)
        d = self.dims(B, block_table.size(1), cache.size(0), max_seqlen, freqs.size(0), out_fp32)
        ws = self.workspace(d)
        if y is None:
            y = torch.empty(B, self.cfg.dim, device=self.device,
                            dtype=torch.float32 if out_fp32 else torch.bfloat16)
        check(lib().qcau_mla_decode(d, q_lora.data_ptr(), self.wq_b.data_ptr(),
                                    self.wq_b_scale.data_ptr(), self.wkv_b_bf16.data_ptr(),
                                    self.wo.data_ptr(), self.wo_scale.data_ptr(), cache.data_ptr(),
                                    block_table.data_ptr(), seqlens.data_ptr(),
                                    positions.data_ptr(), freqs.data_ptr(), y.data_ptr(),
                                    ws.data_ptr(), ws.numel(), stream_ptr(self.device)),
              "mla_decode")
        return y

    def forward_prefill(self, q_lora, cache, block_table, seqlens, freqs, max_seqlen,
                        y: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A prefill (or chunked-prefill) step of the layer: y [B, S, dim] bf16.

        q_lora [B, S, dc] holds the S new tokens of every sequence, whose
        latent rows are already in the cache: seqlens[b] counts them, and
        token t of sequence b attends causally over the first
        seqlens[b] - S + 1 + t cached tokens and takes RoPE at that position
        (the reference's prefill branch, model.py:517-528, on the paged
        cache).  The stages are the decode layer's (q-up + RoPE + absorb; the
        v-up and o-proj) on B * S rows, around the causal prefill attention;
        across head shards y is all-reduced as in forward().
        """
        B, S = q_lora.shape[0], q_lora.shape[1]
        rows = B * S
        c = self.cfg
        q2 = q_lora.reshape(rows, c.dc).contiguous()
        pos = (seqlens.to(torch.int64).view(B, 1) - S + 1 +
               torch.arange(S, device=self.device).view(1, S)).to(torch.int32).reshape(-1)
        # the stage workspace holds no attention partials (max_seqlen 1)
        d = self.dims(rows, block_table.size(1), cache.size(0), 1, freqs.size(0))
        w = c.kv_lora + c.d_rope
        need = lib().qcau_prefill_attn_workspace_size(B, S, self.n_local, c.kv_lora, max_seqlen)
        pf = self._prefill
        if pf is None or pf["rows"] != rows or pf["ws"].numel() < max(need, 1):
            # the stage buffers, kept across steps (and readable by tests)
            pf = self._prefill = {
                "rows": rows,
                "q_abs": torch.empty(rows, self.n_local, w, device=self.device,
                                     dtype=torch.bfloat16),
                "o_lat": torch.empty(rows, self.n_local, c.kv_lora, device=self.device,
                                     dtype=torch.bfloat16),
                "ws": torch.empty(max(need, 1), device=self.device, dtype=torch.uint8),
            }
        q_abs, o_lat, ws = pf["q_abs"], pf["o_lat"], pf["ws"]
        self._q_stage(d, q2, pos, freqs, q_abs)
        check(lib().qcau_prefill_attn_paged(
            q_abs.data_ptr(), cache.data_ptr(), block_table.data_ptr(), seqlens.data_ptr(), None,
            o_lat.data_ptr(), B, S, self.n_local, w, c.kv_lora, w, c.page_size,
            block_table.size(1), cache.size(0), max_seqlen, c.softmax_scale, ws.data_ptr(),
            need, stream_ptr(self.device)), "prefill_attn_paged")
        if y is None:
            y = torch.empty(B, S, c.dim, device=self.device, dtype=torch.bfloat16)
        self._out_stage(d, o_lat, y.view(rows, c.dim))
        if self.world_size > 1:
            dist.all_reduce(y, group=self.group)
        return y

    def forward(self, q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen,
                y: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [batch, dim] bf16, summed over the head shards."""
        if self.cuda_graphs and y is not None and self.stage_events is None:
            args = (q_lora, cache, block_table, seqlens, positions, freqs)
            key = tuple((t.data_ptr(), tuple(t.shape)) for t in args) + (y.data_ptr(),
                                                                          int(max_seqlen))
            g = self._graphs.get(key)
            if g is None:
                # one eager step sets up the stage buffers and plans; the
                # capture then records the same launches
                self._step(q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen, y)
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._step(q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen,
                               y)
                self._graphs[key] = g
            g.replay()
            return y
        return self._step(q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen, y)

    def release_graphs(self) -> None:
        """Drop the captured steps (before the process group that their
        collectives use is destroyed)."""
        self._graphs.clear()

    def _step(self, q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen,
              y: Optional[torch.Tensor] = None) -> torch.Tensor:
        rows = self.attn_split == "rows" and q_lora.size(0) % self.world_size == 0
        if self.world_size > 1 and rows:
            return self.forward_rows(q_lora, cache, block_table, seqlens, positions, freqs,
                                     max_seqlen, y)
        if self.world_size > 1 and self.attn_split in ("context", "rows"):
            # the row split needs the batch to divide by the ranks; else by context
            return self.forward_context(q_lora, cache, block_table, seqlens, positions, freqs,
                                        max_seqlen, y)
        y = self.forward_local(q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen, y)
        if self.world_size > 1:
            dist.all_reduce(y, group=self.group)
        return y

    def _mark(self, name: str) -> None:
        if self.stage_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self.stage_events.append((name, ev))

    def _rows_buffers(self, B: int, max_seqlen: int):
        """Stage buffers of the row-split step, kept across steps."""
        N, Hl, c, dev = self.world_size, self.n_local, self.cfg, self.device
        Br = B // N
        need = lib().qcau_decode_attn_workspace_size(Br, c.n_heads, c.kv_lora, max_seqlen)
        if self._rows is None or self._rows["B"] != B or self._rows["ws"].numel() < need:
            w = c.kv_lora + c.d_rope
            bf16 = torch.bfloat16
            self._rows = {
                "B": B,
                "q_local": torch.empty(B, Hl, w, device=dev, dtype=bf16),
                "q_rows": torch.empty(N, Br, Hl, w, device=dev, dtype=bf16),
                "o_rows": torch.empty(N, Br, Hl, c.kv_lora, device=dev, dtype=bf16),
                "o_lat": torch.empty(B, Hl, c.kv_lora, device=dev, dtype=bf16),
                "ws": torch.empty(max(need, 1), device=dev, dtype=torch.uint8),
            }
        return self._rows

    def forward_rows(self, q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen,
                     y: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [batch, dim] bf16 summed over the ranks, the attention split by sequences.

        Rank r attends, with all heads, over sequences [r*B/N, (r+1)*B/N):
        an all-to-all hands it their queries from every head owner, and a
        second all-to-all hands each owner its heads' outputs for every
        sequence.  With one rank the collectives are identities.
        """
        N, r = self.world_size, self.rank
        B = q_lora.size(0)
        if B % N:
            raise ValueError("attn_split='rows' needs the batch divisible by the number of ranks")
        Br = B // N
        buf = self._rows_buffers(B, max_seqlen)
        if y is None:
            y = torch.empty(B, self.cfg.dim, device=self.device, dtype=torch.bfloat16)
        d = self.dims(B, block_table.size(1), cache.size(0), max_seqlen, freqs.size(0))
        self._mark("start")
        self._q_stage(d, q_lora, positions, freqs, buf["q_local"])
        self._mark("q_up_rope_absorb")
        q_rows = buf["q_local"].view(N, Br, *buf["q_local"].shape[1:])
        if N > 1:   # block j of rank i: rows of rank j, heads of rank i
            dist.all_to_all_single(buf["q_rows"], q_rows, group=self.group)
            q_rows = buf["q_rows"]
            self._mark("q_all_to_all")
        rows = slice(r * Br, (r + 1) * Br)
        self._rows_attn_stage(q_rows, cache, block_table[rows], seqlens[rows], max_seqlen,
                              buf["o_rows"], buf["ws"])
        self._mark("attention")
        o_lat = buf["o_rows"].view(B, *buf["o_lat"].shape[1:])
        if N > 1:   # block j of rank i: heads of rank j, rows of rank i
            dist.all_to_all_single(buf["o_lat"], buf["o_rows"], group=self.group)
            o_lat = buf["o_lat"]
            self._mark("o_all_to_all")
        self._out_stage(d, o_lat, y)
        self._mark("v_up_o_proj")
        if N > 1:
            dist.all_reduce(y, group=self.group)
            self._mark("y_all_reduce")
        return y

    def _rows_attn_stage(self, q_rows, cache, table_rows, seqlens_rows, max_seqlen, o_rows, ws):
        """o_rows [N, B/N, h/N, 512]: all heads over this rank's sequences,
        from q_rows [N, B/N, h/N, 576] (both in blocks of the heads' owners)."""
        c = self.cfg
        w = c.kv_lora + c.d_rope
        Br = q_rows.size(1)
        check(lib().qcau_decode_attn_paged_blocked(
            q_rows.data_ptr(), self.n_local, cache.data_ptr(), table_rows.data_ptr(),
            seqlens_rows.data_ptr(), None, o_rows.data_ptr(), self.n_local, Br, c.n_heads, w,
            c.kv_lora, w, c.page_size, table_rows.size(1), cache.size(0), max_seqlen,
            c.softmax_scale, ws.data_ptr(), ws.numel(), stream_ptr(self.device)),
              "decode_attn_paged_blocked")

    def _cp_buffers(self, B: int):
        """Stage buffers of the context-parallel step, kept across steps."""
        if self._cp is None or self._cp["B"] != B:
            N, Hl, c, dev = self.world_size, self.n_local, self.cfg, self.device
            w = c.kv_lora + c.d_rope
            f32, bf16 = torch.float32, torch.bfloat16
            self._cp = {
                "B": B,
                "q_local": torch.empty(B, Hl, w, device=dev, dtype=bf16),
                "q_all": torch.empty(N, B, Hl, w, device=dev, dtype=bf16),
                # O partials normalised by their sum, in fp16 (half the bytes
                # to exchange, 2^-11 relative error)
                "part_o": torch.empty(N, B, Hl, c.kv_lora, device=dev, dtype=torch.float16),
                "part_ml": torch.empty(N, B, Hl, 2, device=dev, dtype=f32),
                "recv_o": torch.empty(N, B, Hl, c.kv_lora, device=dev, dtype=torch.float16),
                "recv_ml": torch.empty(N, B, Hl, 2, device=dev, dtype=f32),
                "o_lat": torch.empty(B, Hl, c.kv_lora, device=dev, dtype=bf16),
            }
        return self._cp

    def forward_context(self, q_lora, cache, block_table, seqlens, positions, freqs, max_seqlen,
                        y: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [batch, dim] bf16 summed over the ranks, the attention split by context.

        With one rank the collectives are identities and the stages run as
        one rank of one.
        """
        N = self.world_size
        B = q_lora.size(0)
        buf = self._cp_buffers(B)
        if y is None:
            y = torch.empty(B, self.cfg.dim, device=self.device, dtype=torch.bfloat16)
        d = self.dims(B, block_table.size(1), cache.size(0), max_seqlen, freqs.size(0))
        self._q_stage(d, q_lora, positions, freqs, buf["q_local"])
        q_all = buf["q_local"]
        if N > 1:   # [N, B, h/N, 576]: block j = the heads of rank j
            dist.all_gather_into_tensor(buf["q_all"].view(-1, *buf["q_local"].shape[1:]),
                                        buf["q_local"], group=self.group)
            q_all = buf["q_all"]
        if N > 1 and self.exchange == "p2p":
            # the attention kernel stores each rank's partials into that rank's
            # receive area over NVLink and raises its flags; wait for all N
            o_ptr, ml_ptr = self._peer_attn_stage(q_all, cache, block_table, seqlens, max_seqlen)
            self._combine_ptrs(o_ptr, ml_ptr, buf["o_lat"])
            self._out_stage(d, buf["o_lat"], y)
            dist.all_reduce(y, group=self.group)
            return y
        self._attn_stage(q_all, cache, block_table, seqlens, max_seqlen, buf["part_o"],
                         buf["part_ml"])
        recv_o, recv_ml = buf["part_o"], buf["part_ml"]
        if N > 1:   # block j of rank i goes to rank j, which stacks them by source
            dist.all_to_all_single(buf["recv_o"], buf["part_o"], group=self.group)
            dist.all_to_all_single(buf["recv_ml"], buf["part_ml"], group=self.group)
            recv_o, recv_ml = buf["recv_o"], buf["recv_ml"]
        self._combine_stage(recv_o, recv_ml, buf["o_lat"])
        self._out_stage(d, buf["o_lat"], y)
        if N > 1:
            dist.all_reduce(y, group=self.group)
        return y

    # ------------------------------------------------------------ stages
    def _q_stage(self, d, q_lora, positions, freqs, q_abs):
        """q_abs [B, h/N, 576] of this rank's heads."""
        ws = self.workspace(d)
        check(lib().qcau_mla_decode_q(d, q_lora.data_ptr(), self.wq_b.data_ptr(),
                                      self.wq_b_scale.data_ptr(), self.wkv_b_bf16.data_ptr(),
                                      positions.data_ptr(), freqs.data_ptr(), q_abs.data_ptr(),
                                      ws.data_ptr(), ws.numel(), stream_ptr(self.device)),
              "mla_decode_q")

    def _attn_stage(self, q_all, cache, block_table, seqlens, max_seqlen, part_o, part_ml):
        """Partials [N, B, h/N, ...] of all heads over this rank's share of the tiles."""
        c = self.cfg
        w = c.kv_lora + c.d_rope
        check(lib().qcau_decode_attn_paged_cp(q_all.data_ptr(), cache.data_ptr(),
                                              block_table.data_ptr(), seqlens.data_ptr(),
                                              part_o.data_ptr(), part_ml.data_ptr(),
                                              q_all.size(-3), c.n_heads, self.world_size,
                                              self.rank, w, c.kv_lora, w, c.page_size,
                                              block_table.size(1), cache.size(0), max_seqlen,
                                              c.softmax_scale, 1, stream_ptr(self.device)),
              "decode_attn_paged_cp")

    def _combine_stage(self, recv_o, recv_ml, o_lat):
        """o_lat [B, h/N, 512] bf16 from the N partials of this rank's heads."""
        self._combine_ptrs(recv_o.data_ptr(), recv_ml.data_ptr(), o_lat)

    def _combine_ptrs(self, o_ptr: int, ml_ptr: int, o_lat):
        check(lib().qcau_attn_combine_ranks(o_ptr, ml_ptr, None, o_lat.data_ptr(), o_lat.size(0),
                                            self.n_local, self.world_size, self.cfg.kv_lora, 1,
                                            stream_ptr(self.device)), "attn_combine_ranks")

    def _peer_attn_stage(self, q_all, cache, block_table, seqlens, max_seqlen):
        """Context-parallel attention with the exchange fused into the kernel;
        returns the (o, ml) pointers of this rank's completed receive area."""
        c, N, r = self.cfg, self.world_size, self.rank
        B = q_all.size(-3)
        if self._peer is None or self._peer.B != B:
            if self._peer is not None:
                self._peer.close()
            self._peer = PeerExchange(self.device, self.group, r, N, B, self.n_local, c.kv_lora)
        px = self._peer
        px.epoch += 1
        dst_o, dst_ml, dst_flag = px.destinations(px.epoch & 1)
        w = c.kv_lora + c.d_rope
        st = stream_ptr(self.device)
        L = lib()
        check(L.qcau_decode_attn_paged_cp_p2p(q_all.data_ptr(), cache.data_ptr(),
                                              block_table.data_ptr(), seqlens.data_ptr(), dst_o,
                                              dst_ml, dst_flag, px.epoch & 0xFFFFFFFF,
                                              px.counter.data_ptr(), B, c.n_heads, N, r, w,
                                              c.kv_lora, w, c.page_size, block_table.size(1),
                                              cache.size(0), max_seqlen, c.softmax_scale, 1, st),
              "decode_attn_paged_cp_p2p")
        check(L.qcau_wait_flags(px.flags_ptr(), N, px.epoch & 0xFFFFFFFF, st), "wait_flags")
        return px.area(px.epoch & 1)

    def close(self):
        """Release the peer receive buffers (collective: every rank calls it)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def _out_stage(self, d, o_lat, y):
        """y [B, dim], this rank's row-parallel partial."""
        ws = self.workspace(d)
        check(lib().qcau_mla_decode_out(d, o_lat.data_ptr(), self.wkv_b_bf16.data_ptr(),
                                        self.wo.data_ptr(), self.wo_scale.data_ptr(),
                                        y.data_ptr(), ws.data_ptr(), ws.numel(),
                                        stream_ptr(self.device)), "mla_decode_out")


class PeerExchange:
    """Receive areas of the fused partial exchange, shared over CUDA IPC.

    This rank's buffer (in its own GPU memory) holds two areas, used by
    alternate steps, each [N_src, B, h/N, 512] fp16 (O / sum) and [N_src, B, h/N, 2]
    fp32 (max in log2 units, sum), then one flag word per source rank.  Every
    rank opens every peer's buffer; `destinations(parity)` gives the pointers
    where this rank's partials for rank j go (its slot in rank j's area) and
    rank j's flag word for this rank.  Building it is collective.
    """

    def __init__(self, device, group, rank: int, world_size: int, batch: int, heads_local: int,
                 d_v: int):
        import ctypes
        self.device, self.rank, self.N, self.B = device, rank, world_size, batch
        align = lambda x: (x + 255) // 256 * 256   # noqa: E731
        self.slot_o = batch * heads_local * d_v * 2       # one source's o partials (fp16)
        self.slot_ml = batch * heads_local * 2 * 4
        self.area_o_bytes = align(world_size * self.slot_o)
        self.area_ml_bytes = align(world_size * self.slot_ml)
        self.area_bytes = self.area_o_bytes + self.area_ml_bytes
        self.flags_off = 2 * self.area_bytes
        total = self.flags_off + align(world_size * 4)
        L = lib()
        hsz = L.qcau_ipc_handle_size()
        handle = (ctypes.c_ubyte * hsz)()
        base = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(L.qcau_ipc_alloc(total, ctypes.byref(base), ctypes.cast(handle, ctypes.c_void_p)),
                  "ipc_alloc")
        self.base = base.value
        handles = [None] * world_size
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers = []
        for j, h in enumerate(handles):
            if j == rank:
                self.peers.append(self.base)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_ubyte * hsz).from_buffer_copy(h)
            with torch.cuda.device(device):
                check(L.qcau_ipc_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(p)),
                      "ipc_open")
            self.peers.append(p.value)
        self.counter = torch.zeros(1, device=device, dtype=torch.int32)
        self.epoch = 0
        self.group = group
        self._ptrs = ctypes.c_void_p * world_size

    def area(self, parity: int):
        """(o, ml) device pointers of this rank's receive area `parity`."""
        a = self.base + parity * self.area_bytes
        return a, a + self.area_o_bytes

    def flags_ptr(self) -> int:
        return self.base + self.flags_off

    def destinations(self, parity: int):
        """Host arrays (as void pointers) of this rank's destinations in every rank."""
        import ctypes
        r = self.rank
        off = parity * self.area_bytes
        self._keep = (self._ptrs(*[p + off + r * self.slot_o for p in self.peers]),
                      self._ptrs(*[p + off + self.area_o_bytes + r * self.slot_ml
                                   for p in self.peers]),
                      self._ptrs(*[p + self.flags_off + 4 * r for p in self.peers]))
        return tuple(ctypes.cast(a, ctypes.c_void_p) for a in self._keep)

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        L = lib()
        for j, p in enumerate(self.peers):
            if j != self.rank:
                check(L.qcau_ipc_close(p), "ipc_close")
        dist.barrier(group=self.group)
        check(L.qcau_ipc_free(self.base), "ipc_free")
        self.peers = []


def make_paged_cache(batch: int, ctx: int, page_size: int, width: int, device, seed: int = 0,
                     rms_normalise: bool = True):
    """Synthetic paged latent cache: rows ~N(0,1) RMS-normalised, pages shuffled.

    Returns (cache [batch*ctx/page, page, width] bf16, block_table [batch,
    ctx/page] int32 = a random permutation of the physical pages, seqlens).
    """
    assert ctx % page_size == 0
    pages = batch * ctx // page_size
    g = torch.Generator(device=device).manual_seed(seed)
    cache = torch.empty(pages, page_size, width, device=device, dtype=torch.bfloat16)
    chunk = max(1, (1 << 28) // (page_size * width * 4))
    for p0 in range(0, pages, chunk):
        p1 = min(pages, p0 + chunk)
        x = torch.randn(p1 - p0, page_size, width, generator=g, device=device)
        if rms_normalise:
            x = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + 1e-6)
        cache[p0:p1] = x.to(torch.bfloat16)
    perm = torch.randperm(pages, generator=g, device=device).to(torch.int32)
    table = perm.view(batch, ctx // page_size).contiguous()
    seqlens = torch.full((batch,), ctx, device=device, dtype=torch.int32)
    return cache, table, seqlens
