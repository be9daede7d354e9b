"""Head sharding of the absorbed-MLA decode layer, on CPU with gloo ranks.

The layer shards heads like the reference's tensor parallelism: wq_b / wkv_b
column-parallel, wo row-parallel followed by an all-reduce of the partial
outputs (ColumnParallelLinear / RowParallelLinear, model.py:155-180).  These
tests check the host side of that on CPU: the weight slices
(`qcau_b200.mla.shard_weights`) partition the full weights, and the oracle
layer run per rank on its slice, summed by a world_size-2 gloo all-reduce,
equals the unsharded layer.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from qcau_b200.mla import MLAConfig, precompute_freqs_cis, quantize_weight_fp8, shard_weights

CFG = MLAConfig(n_heads=4, dc=256, dim=256)
B, CTX, PAGE, WIDTH = 2, 128, 64, 576


def _bf16(x: torch.Tensor) -> np.ndarray:
    return x.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def _u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy()


def _inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    c = CFG
    H, dq, dkv = c.n_heads, c.d_nope + c.d_rope, c.d_nope + c.d_v
    w = [quantize_weight_fp8(torch.randn(r, k, generator=g) * 0.02)
         for r, k in ((H * dq, c.dc), (H * dkv, c.kv_lora), (c.dim, H * c.d_v))]
    weights = (w[0][0], w[0][1], w[1][0], w[1][1], w[2][0], w[2][1])
    q_lora = torch.randn(B, c.dc, generator=g)
    q_lora = q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))
    pages = B * CTX // PAGE
    cache = torch.randn(pages, PAGE, WIDTH, generator=g)
    cache = cache * torch.rsqrt(cache.square().mean(-1, keepdim=True))
    table = torch.randperm(pages, generator=g).to(torch.int32).view(B, CTX // PAGE)
    seqlens = np.array([CTX, 77], dtype=np.int32)
    positions = seqlens.copy()
    freqs = precompute_freqs_cis(c.d_rope, 256, c.rope_theta, "cpu").numpy()
    return weights, _bf16(q_lora), _bf16(cache), table.numpy(), seqlens, positions, freqs


def _oracle_layer(weights, q_lora, cache, table, seqlens, positions, freqs) -> np.ndarray:
    """y [B, dim] fp32 of the absorbed-MLA decode layer over the heads the
    weights hold (the full layer, or one rank's shard)."""
    c = CFG
    wq, wqs, wkv, wkvs, wo, wos = weights
    H = wq.shape[0] // (c.d_nope + c.d_rope)
    xq, xs = O.act_quant(q_lora, 128, False)
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, _u8(wq), wqs.numpy())).reshape(B, 1, H, 192)
    qr = np.stack([O.rope(q[b:b + 1], freqs, 64, int(positions[b])) for b in range(B)])[:, 0]
    qr = qr.reshape(B, H, 192)
    wkv_bf16 = O.f32_to_bf16(O.e4m3_to_f32(_u8(wkv)) *
                             np.repeat(np.repeat(wkvs.numpy(), 128, 0), 128, 1))
    q_abs = np.concatenate([O.mla_absorb(qr, wkv_bf16, 128, 128), qr[..., 128:]], axis=-1)
    o_lat = O.paged_decode_attn(q_abs, cache, table, seqlens, None, c.softmax_scale, 512)
    o_v = O.mla_vup(O.f32_to_bf16(o_lat), wkv_bf16, 128, 128).reshape(B, H * 128)
    xo, so = O.act_quant(o_v, 128, False)
    return O.fp8_gemm(xo, so, _u8(wo), wos.numpy())


def test_shard_weights_partition_the_full_weights():
    weights = _inputs()[0]
    for ws in (1, 2):
        parts = [shard_weights(CFG, r, ws, *weights) for r in range(ws)]
        for i, full in enumerate(weights):
            dim = 1 if i >= 4 else 0   # wo and its scale are split by columns
            cat = torch.cat([p[i] for p in parts], dim=dim)
            assert torch.equal(cat.view(torch.uint8) if cat.dtype == torch.float8_e4m3fn else cat,
                               full.view(torch.uint8) if full.dtype == torch.float8_e4m3fn else full)


def test_shard_weights_rejects_uneven_heads():
    with pytest.raises(ValueError, match="divisible"):
        shard_weights(CFG, 0, 3, *_inputs()[0])
    # one head per rank: 192 rows of wq_b are not whole 128-row scale blocks
    with pytest.raises(ValueError, match="scale blocks"):
        shard_weights(CFG, 0, 4, *_inputs()[0])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world_size, port, out_dir):
    os.environ["OMP_NUM_THREADS"] = "2"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world_size)
    try:
        weights, q_lora, cache, table, seqlens, positions, freqs = _inputs()
        shard = shard_weights(CFG, rank, world_size, *weights)
        y = torch.from_numpy(_oracle_layer(shard, q_lora, cache, table, seqlens, positions, freqs))
        dist.all_reduce(y)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    finally:
        dist.destroy_process_group()


def test_head_sharded_layer_all_reduce_equals_unsharded(tmp_path):
    world_size = 2
    mp.start_processes(_rank_main, args=(world_size, _free_port(), str(tmp_path)),
                       nprocs=world_size, start_method="spawn", join=True)
    ref = _oracle_layer(*_inputs())
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    for r in range(world_size):
        y = np.load(tmp_path / f"y{r}.npy")
        # the same 128-blocks summed in a different grouping: fp32 rounding only
        assert np.max(np.abs(y - ref)) <= 1e-5 * rms + 1e-7, f"rank {r}"
