"""The V4 output side (GOPU: wo_a grouped einsum + row-parallel wo_b,
Deepseek_origin/inference/model.py:536-542, :166-180) on CPU:

  * the oracle is bit-exact with the reference's own code
    (tests/golden/gopu.npz, made by make_golden.py from model.py's einsum and
    linear() on kernel_fallback's FP8 kernels);
  * GOPU.shard splits the weights by groups (wo_a rows, wo_b columns) so that
    the ranks' partial outputs, each rounded to bf16 and summed in fp32 by a
    world_size-2 gloo all-reduce as RowParallelLinear does, give the
    reference's sharded result.
"""
from __future__ import annotations

import os
import socket
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from qcau_b200.gopu import GOPU

GOLDEN = Path(__file__).resolve().parent / "golden"
B, S, H, D, G, R, DIM = 2, 3, 8, 512, 2, 128, 256


def _oracle(o, wo_a, wo_b, wo_b_scale):
    """y [rows, dim] fp32 of the groups the weights hold."""
    g = wo_a.shape[0] // R
    h = O.grouped_proj(o.reshape(-1, g, H // G * D), wo_a.reshape(g, R, -1))
    xq, xs = O.act_quant(h.reshape(-1, g * R), 128, True)
    return O.fp8_gemm(xq, xs, wo_b, O.e8m0_to_f32(wo_b_scale))


def test_oracle_gopu_bit_exact_with_reference_code():
    f = np.load(GOLDEN / "gopu.npz")
    h = O.grouped_proj(f["o"].reshape(B * S, G, -1), f["wo_a"].reshape(G, R, -1))
    assert np.array_equal(h.reshape(f["h"].shape), f["h"])
    y = O.f32_to_bf16(_oracle(f["o"], f["wo_a"], f["wo_b"], f["wo_b_scale"]))
    assert np.array_equal(y.reshape(f["y"].shape), f["y"])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world_size, port, out_dir):
    os.environ["OMP_NUM_THREADS"] = "2"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world_size)
    try:
        f = np.load(GOLDEN / "gopu.npz")
        m = GOPU(n_heads=H, head_dim=D, n_groups=G, o_lora_rank=R, dim=DIM, device="cpu",
                 rank=rank, world_size=world_size)
        wo_a = torch.from_numpy(f["wo_a"].view(np.int16)).view(torch.bfloat16)
        wo_b = torch.from_numpy(f["wo_b"]).view(torch.float8_e4m3fn)
        sc = torch.from_numpy(f["wo_b_scale"]).view(torch.float8_e8m0fnu)
        a, b, s = m.shard(wo_a, wo_b, sc)
        hl = H // world_size  # this rank's heads: its groups
        o = f["o"][:, :, rank * hl:(rank + 1) * hl]
        y = O.f32_to_bf16(_oracle(np.ascontiguousarray(o),
                                  a.reshape(-1, a.shape[-1]).contiguous().view(torch.int16).numpy().view(np.uint16),
                                  b.contiguous().view(torch.uint8).numpy(),
                                  s.contiguous().view(torch.uint8).numpy()))
        y32 = torch.from_numpy(O.bf16_to_f32(y))
        dist.all_reduce(y32)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y32.numpy())
    finally:
        dist.destroy_process_group()


def test_group_sharded_gopu_all_reduce(tmp_path):
    world_size = 2
    mp.start_processes(_rank_main, args=(world_size, _free_port(), str(tmp_path)),
                       nprocs=world_size, start_method="spawn", join=True)
    f = np.load(GOLDEN / "gopu.npz")
    full = _oracle(f["o"], f["wo_a"], f["wo_b"], f["wo_b_scale"])
    # the reference's sharded result: each rank's bf16 partial, summed in fp32
    parts = []
    for r in range(world_size):
        gl = G // world_size
        o = f["o"][:, :, r * H // world_size:(r + 1) * H // world_size]
        wa = f["wo_a"][r * gl * R:(r + 1) * gl * R]
        wb = f["wo_b"][:, r * gl * R:(r + 1) * gl * R]
        ws = f["wo_b_scale"][:, r * gl * R // 128:(r + 1) * gl * R // 128]
        parts.append(O.bf16_to_f32(O.f32_to_bf16(_oracle(np.ascontiguousarray(o), wa, wb, ws))))
    want = parts[0] + parts[1]
    rms = float(np.sqrt(np.mean(full.astype(np.float64) ** 2)))
    for r in range(world_size):
        y = np.load(tmp_path / f"y{r}.npy")
        assert np.array_equal(y, want), f"rank {r}"
        assert np.max(np.abs(y - full)) <= 2e-2 * rms, f"rank {r} vs unsharded"
