"""GOPU: the V4 output side of the attention block, after the QCAU output.

Replaces, in the reference Attention.forward (Deepseek_origin/inference/
model.py:536-542),

    o = o.view(bsz, seqlen, self.n_local_groups, -1)
    wo_a = self.wo_a.weight.view(self.n_local_groups, self.o_lora_rank, -1)
    o = torch.einsum("bsgd,grd->bsgr", o, wo_a)          # grouped low-rank, bf16
    x = self.wo_b(o.flatten(2))                           # RowParallelLinear, FP8

with one library call (qcau_gopu: the tcgen05 batched GEMM for wo_a, then
act_quant and the FP8 GEMM for wo_b) and, across head shards, the all-reduce
of RowParallelLinear (model.py:173-179): the bf16 partials are summed in fp32
over the process group (NCCL) and rounded back to bf16.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, lib, require_cuda, stream_ptr


class GOPU:
    """wo_a (ColumnParallelLinear over the groups, bf16) and wo_b
    (RowParallelLinear, FP8 with 128x128 block scales) of one rank.

    n_heads / n_groups / o_lora_rank / dim are the model's (V4-Flash: 64, 8,
    1024, 4096, model.py config); head_dim 512.  Ranks own n_groups /
    world_size consecutive groups and the matching columns of wo_b.
    """

    def __init__(self, n_heads: int = 64, head_dim: int = 512, n_groups: int = 8,
                 o_lora_rank: int = 1024, dim: int = 4096, device="cuda", rank: int = 0,
                 world_size: int = 1, process_group=None, act_round_scale: bool = True):
        if n_groups % world_size or n_heads % n_groups:
            raise ValueError("groups must divide over the heads and the ranks")
        self.n_heads, self.head_dim, self.n_groups = n_heads, head_dim, n_groups
        self.rank_dim, self.dim = o_lora_rank, dim
        self.rank, self.world_size, self.group = rank, world_size, process_group
        self.n_local_groups = n_groups // world_size
        self.group_dim = n_heads // n_groups * head_dim
        self.device = torch.device(device)
        self.act_round_scale = act_round_scale
        self.wo_a = self.wo_b = self.wo_b_scale = None
        self._ws = None

    def shard(self, wo_a: torch.Tensor, wo_b: torch.Tensor, wo_b_scale: torch.Tensor):
        """This rank's slices of the full weights: wo_a rows of its groups
        (ColumnParallelLinear), wo_b columns of its groups (RowParallelLinear)."""
        g0, gl, R = self.rank * self.n_local_groups, self.n_local_groups, self.rank_dim
        a = wo_a.view(self.n_groups, R, self.group_dim)[g0:g0 + gl]
        cols = slice(g0 * R, (g0 + gl) * R)
        scols = slice(g0 * R // 128, (g0 + gl) * R // 128)
        return a, wo_b[:, cols], wo_b_scale[:, scols]

    def load_weights(self, wo_a: torch.Tensor, wo_b: torch.Tensor, wo_b_scale: torch.Tensor,
                     sharded: bool = False):
        """wo_a [n_groups * o_lora_rank, group_dim] bf16, wo_b [dim, n_groups *
        o_lora_rank] e4m3, wo_b_scale [dim/128, .../128] fp32 or e8m0 (full
        tensors unless sharded=True)."""
        if not sharded:
            wo_a, wo_b, wo_b_scale = self.shard(wo_a, wo_b, wo_b_scale)
        self.wo_a = wo_a.to(self.device, torch.bfloat16).contiguous()
        self.wo_b = wo_b.to(self.device).contiguous()
        self.wo_b_scale = wo_b_scale.to(self.device).contiguous()

    def forward_local(self, o: torch.Tensor, out_fp32: bool = False) -> torch.Tensor:
        """This rank's partial output [..., dim] for o [..., local heads, head_dim]."""
        require_cuda(o)
        lead = o.shape[:-2]
        rows = o.numel() // (self.n_local_groups * self.group_dim)
        o = o.contiguous()
        y = torch.empty(*lead, self.dim, device=self.device,
                        dtype=torch.float32 if out_fp32 else torch.bfloat16)
        need = lib().qcau_gopu_workspace_size(rows, self.n_local_groups, self.rank_dim)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 1), device=self.device, dtype=torch.uint8)
        scale_code = _lib.SCALE_E8M0 if self.wo_b_scale.dtype == torch.float8_e8m0fnu else _lib.SCALE_F32
        check(lib().qcau_gopu(o.data_ptr(), self.wo_a.data_ptr(), self.wo_b.data_ptr(),
                              self.wo_b_scale.data_ptr(), scale_code, int(self.act_round_scale),
                              y.data_ptr(), _lib.OUT_F32 if out_fp32 else _lib.OUT_BF16, rows,
                              self.n_local_groups, self.group_dim, self.rank_dim, self.dim,
                              self._ws.data_ptr(), self._ws.numel(), stream_ptr(self.device)),
              "gopu")
        return y

    def forward(self, o: torch.Tensor) -> torch.Tensor:
        """y [..., dim] bf16, summed over the ranks as RowParallelLinear does:
        each rank's bf16 partial in fp32, all-reduced, back to bf16."""
        y = self.forward_local(o)
        if self.world_size > 1:
            y32 = y.float()
            dist.all_reduce(y32, group=self.group)
            y = y32.to(torch.bfloat16)
        return y
