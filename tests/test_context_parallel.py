"""Context-parallel attention of the head-sharded decode layer.

With `attn_split="context"` the N ranks of a head-sharded layer all-gather
their absorbed queries, each attends with all heads over 1/N of every
sequence's 128-token tiles, and an all-to-all brings each rank the partial
softmax states (unnormalised O, max in log2 units, sum) of its own heads,
which it merges before the v-up and the row-parallel o-proj.

CPU (gloo, world size 2): `MLADecodeLayer.forward_context` runs with its
four kernel stages replaced by oracle-backed stand-ins on CPU tensors, so the
orchestration itself (buffer layouts, the rank's tile range, the block order
of the exchange, the merge, the all-reduce) is checked against the unsharded
oracle layer.

GPU: the pair kernel's context-parallel mode through the C ABI, N ranks
emulated on one device (block exchange done by indexing), against the
single-rank decode attention; the staged layer at one rank against the fused
layer; and, with two or more devices, the layer over NCCL.
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
from helpers import assert_close_attn
from qcau_b200 import _lib
from qcau_b200.mla import (MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis,
                           quantize_weight_fp8, shard_weights)

LOG2E = 1.4426950408889634

# ---------------------------------------------------------------- CPU (gloo)

CFG = MLAConfig(n_heads=4, dc=256, dim=256)
B, CTX, PAGE, WIDTH = 2, 512, 64, 576
SEQLENS = np.array([CTX, 77], dtype=np.int32)   # 4 tiles, and 1 tile (one rank empty)


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
    positions = SEQLENS.copy()
    freqs = precompute_freqs_cis(c.d_rope, 1024, c.rope_theta, "cpu").numpy()
    return (weights, q_lora.to(torch.bfloat16), cache.to(torch.bfloat16), table,
            torch.from_numpy(SEQLENS.copy()), torch.from_numpy(positions), torch.from_numpy(freqs))


def _wkv_bf16(wkv, wkvs) -> np.ndarray:
    return O.f32_to_bf16(O.e4m3_to_f32(_u8(wkv)) *
                         np.repeat(np.repeat(wkvs.numpy(), 128, 0), 128, 1))


def _q_abs(wq, wqs, wkv, wkvs, q_lora_u16, positions, freqs) -> np.ndarray:
    """q_abs [B, H, 576] bf16 (uint16) of the heads the weights hold."""
    H = wq.shape[0] // 192
    xq, xs = O.act_quant(q_lora_u16, 128, False)
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, _u8(wq), wqs.numpy())).reshape(B, 1, H, 192)
    qr = np.stack([O.rope(q[b:b + 1], freqs, 64, int(positions[b])) for b in range(B)])[:, 0]
    qr = qr.reshape(B, H, 192)
    return np.concatenate([O.mla_absorb(qr, _wkv_bf16(wkv, wkvs), 128, 128), qr[..., 128:]],
                          axis=-1)


def _out(o_lat_u16, wkv, wkvs, wo, wos) -> np.ndarray:
    H = wkv.shape[0] // 256
    o_v = O.mla_vup(o_lat_u16, _wkv_bf16(wkv, wkvs), 128, 128).reshape(B, H * 128)
    xo, so = O.act_quant(o_v, 128, False)
    return O.fp8_gemm(xo, so, _u8(wo), wos.numpy())


def _oracle_layer(weights, q_lora, cache, table, seqlens, positions, freqs) -> np.ndarray:
    wq, wqs, wkv, wkvs, wo, wos = weights
    q_abs = _q_abs(wq, wqs, wkv, wkvs, _bf16(q_lora), positions.numpy(), freqs.numpy())
    o_lat = O.paged_decode_attn(q_abs, _bf16(cache), table.numpy(), seqlens.numpy(), None,
                                CFG.softmax_scale, 512)
    return _out(O.f32_to_bf16(o_lat), wkv, wkvs, wo, wos)


def rank_partials(q_all, cache, table, seqlens, rank, n, scale):
    """The context-parallel attention stage restated: all heads over rank
    `rank`'s tiles [ntiles*rank/n, ntiles*(rank+1)/n) of each sequence
    (ntiles = ceil(seqlen/128)); partials [n, B, h/n, 512] (O divided by its
    sum) and [n, B, h/n, 2] (max in log2 units, sum) with block j holding the
    heads of rank j, P rounded to bf16 for P.V and the sum over the unrounded
    P (the kernel's numerics)."""
    qa = O.bf16_to_f32(q_all)                       # [n, B, hl, 576]
    nb, bsz, hl, w = qa.shape
    q = qa.transpose(1, 0, 2, 3).reshape(bsz, nb * hl, w)
    cf = O.bf16_to_f32(cache)
    part_o = np.zeros((n, bsz, hl, 512), np.float32)
    part_ml = np.zeros((n, bsz, hl, 2), np.float32)
    for b in range(bsz):
        L = int(seqlens[b])
        nt = (L + 127) // 128
        lo, hi = 128 * (nt * rank // n), min(128 * (nt * (rank + 1) // n), L)
        toks = np.arange(lo, max(lo, hi))
        rows = cf[table[b, toks // PAGE], toks % PAGE]       # [n_tok, 576]
        if len(toks):
            x = (q[b] @ rows.T) * np.float32(scale * LOG2E)
            m = x.max(1)
            p = np.exp2(x - m[:, None]).astype(np.float32)
            l = p.sum(1)
            o = (O.bf16_to_f32(O.f32_to_bf16(p)) @ rows[:, :512]) / l[:, None]
        else:
            m = np.full(nb * hl, -np.inf, np.float32)
            l = np.zeros(nb * hl, np.float32)
            o = np.zeros((nb * hl, 512), np.float32)
        for h in range(nb * hl):
            part_o[h // hl, b, h % hl] = o[h]
            part_ml[h // hl, b, h % hl] = (m[h], l[h])
    return part_o, part_ml


def merge_partials(recv_o, recv_ml) -> np.ndarray:
    """o [B, h/n, 512] bf16 (uint16) from [n, B, h/n, ...] partials (O / sum)."""
    m = recv_ml[..., 0]
    M = m.max(0)
    wgt = np.where(np.isneginf(m), 0.0, np.exp2(m - np.where(np.isneginf(M), 0.0, M)))
    L = (recv_ml[..., 1] * wgt).sum(0)
    o = (recv_o * (wgt * recv_ml[..., 1])[..., None]).sum(0) / np.maximum(L, 1e-38)[..., None]
    return O.f32_to_bf16(o.astype(np.float32))


class OracleStagesLayer(MLADecodeLayer):
    """The layer's orchestration with its four kernel stages replaced by
    oracle-backed CPU stand-ins (CPU tensors, no CUDA)."""

    def load_weights(self, wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo, wo_scale, sharded=False):
        if not sharded and self.world_size > 1:
            wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo, wo_scale = shard_weights(
                self.cfg, self.rank, self.world_size, wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo,
                wo_scale)
        self.w = (wq_b, wq_b_scale, wkv_b, wkv_b_scale, wo, wo_scale)

    def workspace(self, d):
        return torch.empty(1, dtype=torch.uint8)

    def dims(self, *args, **kwargs):
        return None

    def _q_stage(self, d, q_lora, positions, freqs, q_abs):
        wq, wqs, wkv, wkvs, _, _ = self.w
        qa = _q_abs(wq, wqs, wkv, wkvs, _bf16(q_lora), positions.numpy(), freqs.numpy())
        q_abs.copy_(torch.from_numpy(qa.view(np.int16)).view(torch.bfloat16))

    def _attn_stage(self, q_all, cache, block_table, seqlens, max_seqlen, part_o, part_ml):
        qa = _bf16(q_all if q_all.dim() == 4 else q_all.unsqueeze(0))
        po, pml = rank_partials(qa, _bf16(cache), block_table.numpy(), seqlens.numpy(),
                                self.rank, self.world_size, self.cfg.softmax_scale)
        part_o.copy_(torch.from_numpy(po))
        part_ml.copy_(torch.from_numpy(pml))

    def _rows_attn_stage(self, q_rows, cache, table_rows, seqlens_rows, max_seqlen, o_rows, ws):
        qa = _bf16(q_rows)                                   # [N, B/N, h/N, 576]
        nb, br, hl, w = qa.shape
        q = np.ascontiguousarray(qa.transpose(1, 0, 2, 3).reshape(br, nb * hl, w))
        o = O.paged_decode_attn(q, _bf16(cache), table_rows.numpy(), seqlens_rows.numpy(), None,
                                self.cfg.softmax_scale, 512)   # [B/N, h, 512]
        ob = np.ascontiguousarray(o.reshape(br, nb, hl, 512).transpose(1, 0, 2, 3))
        o_rows.copy_(torch.from_numpy(O.f32_to_bf16(ob).view(np.int16)).view(torch.bfloat16))

    def _combine_stage(self, recv_o, recv_ml, o_lat):
        o = merge_partials(recv_o.float().numpy(), recv_ml.numpy())
        o_lat.copy_(torch.from_numpy(o.view(np.int16)).view(torch.bfloat16))

    def _out_stage(self, d, o_lat, y):
        _, _, wkv, wkvs, wo, wos = self.w
        y.copy_(torch.from_numpy(_out(_bf16(o_lat), wkv, wkvs, wo, wos)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_rank_main(rank, world_size, port, out_dir, split="context"):
    os.environ["OMP_NUM_THREADS"] = "2"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world_size)
    try:
        weights, q_lora, cache, table, seqlens, positions, freqs = _inputs()
        # the exchange through collectives (the fused peer-memory one needs GPUs)
        layer = OracleStagesLayer(CFG, "cpu", rank, world_size, attn_split=split,
                                  exchange="nccl")
        layer.load_weights(*weights)
        y = torch.empty(B, CFG.dim, dtype=torch.float32)
        layer.forward(q_lora, cache, table, seqlens, positions, freqs, CTX, y)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split", ["context", "rows"])
def test_split_attention_layer_over_gloo_equals_unsharded(tmp_path, split):
    """The context split (partial states exchanged) and the row split
    (queries and outputs exchanged, whole sequences per rank)."""
    world_size = 2
    mp.start_processes(_cp_rank_main, args=(world_size, _free_port(), str(tmp_path), split),
                       nprocs=world_size, start_method="spawn", join=True)
    ref = _oracle_layer(*_inputs())
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    for r in range(world_size):
        y = np.load(tmp_path / f"y{r}.npy")
        # P is rounded to bf16 against each rank's own maximum (and the O
        # partials are exchanged in fp16): bf16 noise in o_lat, which the FP8
        # act_quant of o_v (one e4m3 step is 1/8) can turn into a code flip of
        # single elements; a wrong block or tile order would break the cosine
        _assert_layer_close(y, ref, f"rank {r}")


def test_rank_tile_ranges_partition_every_sequence():
    """The ranks' tile ranges are disjoint and cover [0, ntiles) for any N."""
    for L in (0, 1, 127, 128, 129, 1000, 32768):
        nt = (L + 127) // 128
        for n in (1, 2, 3, 4, 8):
            got = []
            for r in range(n):
                got += list(range(nt * r // n, nt * (r + 1) // n))
            assert got == list(range(nt)), (L, n)


def test_merge_of_rank_partials_equals_one_pass():
    """Partials over disjoint token ranges, merged, equal one pass over all
    tokens (the oracle's paged decode attention), for 1, 2, 4 and 8 ranks."""
    g = torch.Generator().manual_seed(3)
    H, bsz, ctx = 8, 3, 640
    pages = bsz * ctx // PAGE
    cache = torch.randn(pages, PAGE, WIDTH, generator=g).to(torch.bfloat16)
    table = torch.randperm(pages, generator=g).to(torch.int32).view(bsz, ctx // PAGE).numpy()
    seqlens = np.array([640, 300, 1], np.int32)
    q = torch.randn(bsz, H, WIDTH, generator=g).to(torch.bfloat16)
    ref = O.bf16_to_f32(O.f32_to_bf16(O.paged_decode_attn(_bf16(q), _bf16(cache), table, seqlens,
                                                          None, 0.07, 512)))
    for n in (1, 2, 4, 8):
        hl = H // n
        q_all = _bf16(q).reshape(bsz, n, hl, WIDTH).transpose(1, 0, 2, 3).copy()
        parts = [rank_partials(q_all, _bf16(cache), table, seqlens, r, n, 0.07) for r in range(n)]
        out = []
        for dst in range(n):
            recv_o = np.stack([parts[r][0][dst] for r in range(n)])
            recv_ml = np.stack([parts[r][1][dst] for r in range(n)])
            out.append(O.bf16_to_f32(merge_partials(recv_o, recv_ml)))
        got = np.concatenate(out, axis=1)
        assert np.max(np.abs(got - ref)) <= 2e-2 * np.sqrt(np.mean(ref ** 2)), n


# ---------------------------------------------------------------- GPU


def _assert_layer_close(y: np.ndarray, ref: np.ndarray, what: str):
    """Layer outputs computed with the attention merged in a different order.
    o_lat differs by bf16 rounding; the FP8 act_quant of o_v turns that into
    one-code flips (one e4m3 step is 1/16 to 1/8 of the value) of a few per
    cent of its elements, and the o-proj sums ~16k of them: a mean error of
    1-3 % of the RMS and single elements up to ~10 %.  The bound is on the
    cosine, the mean error and the largest error."""
    y, ref = y.astype(np.float64), ref.astype(np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    cos = float((y * ref).sum() / np.sqrt((y * y).sum() * (ref * ref).sum()))
    assert cos >= 0.9995, (what, cos)
    assert float(np.mean(np.abs(y - ref))) <= 3e-2 * rms, what
    assert float(np.max(np.abs(y - ref))) <= 0.15 * rms, what


@pytest.mark.gpu
@pytest.mark.parametrize("n,f16", [(1, 1), (2, 1), (4, 0), (4, 1), (8, 1)])
def test_cp_attention_emulated_ranks_match_decode(n, f16):
    """N ranks of qcau_decode_attn_paged_cp on one device, the block exchange
    done by indexing, merged by qcau_attn_combine_ranks, equal the
    single-rank qcau_decode_attn_paged (ragged lengths, an empty sequence,
    one-token and one-tile-plus-one sequences)."""
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    H, ctx = 128, 4096
    bsz = 6
    cache, table, _ = make_paged_cache(bsz, ctx, PAGE, WIDTH, dev, seed=5)
    seqlens = torch.tensor([4096, 0, 1, 129, 3000, 2048], device=dev, dtype=torch.int32)
    g = torch.Generator(device=dev).manual_seed(6)
    q = torch.randn(bsz, H, WIDTH, device=dev, generator=g).to(torch.bfloat16)
    scale = 192 ** -0.5
    st = _lib.stream_ptr(dev)
    ref = torch.empty(bsz, H, 512, device=dev, dtype=torch.bfloat16)
    need = L.qcau_decode_attn_workspace_size(bsz, H, 512, ctx)
    ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
    _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                        seqlens.data_ptr(), None, ref.data_ptr(), bsz, H, WIDTH,
                                        512, WIDTH, PAGE, table.size(1), cache.size(0), ctx, scale,
                                        ws.data_ptr(), need, st), "decode")
    hl = H // n
    q_all = q.view(bsz, n, hl, WIDTH).transpose(0, 1).contiguous()
    odt = torch.float16 if f16 else torch.float32
    part_o = torch.empty(n, n, bsz, hl, 512, device=dev, dtype=odt)   # [rank][dest] ...
    part_ml = torch.empty(n, n, bsz, hl, 2, device=dev)
    for r in range(n):
        _lib.check(L.qcau_decode_attn_paged_cp(q_all.data_ptr(), cache.data_ptr(),
                                               table.data_ptr(), seqlens.data_ptr(),
                                               part_o[r].data_ptr(), part_ml[r].data_ptr(), bsz,
                                               H, n, r, WIDTH, 512, WIDTH, PAGE, table.size(1),
                                               cache.size(0), ctx, scale, f16, st), "cp")
    outs = []
    for dst in range(n):
        recv_o = part_o[:, dst].contiguous()
        recv_ml = part_ml[:, dst].contiguous()
        o = torch.empty(bsz, hl, 512, device=dev, dtype=torch.bfloat16)
        _lib.check(L.qcau_attn_combine_ranks(recv_o.data_ptr(), recv_ml.data_ptr(), None,
                                             o.data_ptr(), bsz, hl, n, 512, f16, st), "combine")
        outs.append(o)
    got = torch.cat(outs, dim=1)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    a, b = got.float(), ref.float()
    assert torch.all(a[1] == 0), "an empty sequence gives zeros"
    # the path's bar (max(2e-2 * rms, 1 bf16 ulp)): the two merge orders round
    # differently at large outputs
    assert_close_attn(a.cpu().numpy(), b.cpu().numpy(), f"cp {n} ranks")
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert cos >= 0.9999


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 8])
def test_cp_p2p_kernel_emulated_ranks(n):
    """qcau_decode_attn_paged_cp_p2p of N ranks on one device: each launch
    stores its partials into the (emulated) receive areas of the ranks that
    own the heads and raises their flags; after qcau_wait_flags, merging each
    area equals the single-rank decode attention.  The flags hold the epoch,
    and the done counter is back at zero after every launch."""
    import ctypes
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    H, ctx, bsz = 128, 2048, 5
    cache, table, _ = make_paged_cache(bsz, ctx, PAGE, WIDTH, dev, seed=8)
    seqlens = torch.tensor([2048, 1, 0, 1500, 700], device=dev, dtype=torch.int32)
    g = torch.Generator(device=dev).manual_seed(9)
    q = torch.randn(bsz, H, WIDTH, device=dev, generator=g).to(torch.bfloat16)
    scale = 192 ** -0.5
    st = _lib.stream_ptr(dev)
    ref = torch.empty(bsz, H, 512, device=dev, dtype=torch.bfloat16)
    need = L.qcau_decode_attn_workspace_size(bsz, H, 512, ctx)
    ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
    _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                        seqlens.data_ptr(), None, ref.data_ptr(), bsz, H, WIDTH,
                                        512, WIDTH, PAGE, table.size(1), cache.size(0), ctx, scale,
                                        ws.data_ptr(), need, st), "decode")
    hl = H // n
    q_all = q.view(bsz, n, hl, WIDTH).transpose(0, 1).contiguous()
    recv_o = torch.full((n, n, bsz, hl, 512), float("nan"), device=dev,
                        dtype=torch.float16)   # [owner][src] ...
    recv_ml = torch.full((n, n, bsz, hl, 2), float("nan"), device=dev)
    flags = torch.zeros(n, n, device=dev, dtype=torch.int32)                # [owner][src]
    counter = torch.zeros(1, device=dev, dtype=torch.int32)
    epoch = 7
    arr = ctypes.c_void_p * n
    for r in range(n):
        dst_o = arr(*[recv_o[j, r].data_ptr() for j in range(n)])
        dst_ml = arr(*[recv_ml[j, r].data_ptr() for j in range(n)])
        dst_f = arr(*[flags[j, r:].data_ptr() for j in range(n)])
        _lib.check(L.qcau_decode_attn_paged_cp_p2p(
            q_all.data_ptr(), cache.data_ptr(), table.data_ptr(), seqlens.data_ptr(),
            ctypes.cast(dst_o, ctypes.c_void_p), ctypes.cast(dst_ml, ctypes.c_void_p),
            ctypes.cast(dst_f, ctypes.c_void_p), epoch, counter.data_ptr(), bsz, H, n, r, WIDTH,
            512, WIDTH, PAGE, table.size(1), cache.size(0), ctx, scale, 1, st), "cp_p2p")
    outs = []
    for j in range(n):
        _lib.check(L.qcau_wait_flags(flags[j].data_ptr(), n, epoch, st), "wait")
        o = torch.empty(bsz, hl, 512, device=dev, dtype=torch.bfloat16)
        _lib.check(L.qcau_attn_combine_ranks(recv_o[j].data_ptr(), recv_ml[j].data_ptr(), None,
                                             o.data_ptr(), bsz, hl, n, 512, 1, st), "combine")
        outs.append(o)
    got = torch.cat(outs, dim=1)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.all(flags == epoch)
    assert int(counter.item()) == 0
    assert not torch.isnan(recv_ml).any(), "every slot was written"
    a, b = got.float(), ref.float()
    assert_close_attn(a.cpu().numpy(), b.cpu().numpy(), f"cp p2p {n} ranks")
    assert torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item() >= 0.9999


@pytest.mark.gpu
def test_wait_flags_times_out_with_status():
    """A flag that nothing raises: the wait gives up after its bound (~1 s)
    and reports QCAU_DEVERR_TIMEOUT; the context stays usable."""
    L = _lib.lib()
    flags = torch.zeros(4, device="cuda", dtype=torch.int32)
    flags[:3] = 5
    _lib.check(L.qcau_wait_flags(flags.data_ptr(), 4, 5, _lib.stream_ptr()), "wait")
    assert _lib.device_error() == _lib.DEVERR_TIMEOUT
    flags[3] = 5
    _lib.check(L.qcau_wait_flags(flags.data_ptr(), 4, 5, _lib.stream_ptr()), "wait")
    assert _lib.device_error() == 0


@pytest.mark.gpu
def test_cp_rejects_unsupported_head_blocks():
    L = _lib.lib()
    z = torch.zeros(16, device="cuda", dtype=torch.int32)
    # 128 heads over 3 ranks: not divisible
    rc = L.qcau_decode_attn_paged_cp(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(),
                                     z.data_ptr(), z.data_ptr(), 1, 128, 3, 0, 576, 512, 576, 64,
                                     1, 1, 64, 0.1, 0, _lib.stream_ptr())
    assert rc == _lib.QCAU_ERR_INVALID
    # 128 heads over 16 ranks: blocks of 8 heads are allowed; 48 heads are not a multiple of 128
    rc = L.qcau_decode_attn_paged_cp(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(),
                                     z.data_ptr(), z.data_ptr(), 1, 48, 2, 0, 576, 512, 576, 64,
                                     1, 1, 64, 0.1, 0, _lib.stream_ptr())
    assert rc == _lib.QCAU_ERR_UNSUPPORTED


@pytest.mark.gpu
@pytest.mark.parametrize("hb", [16, 32, 64, 128])
def test_blocked_decode_equals_plain_decode(hb):
    """qcau_decode_attn_paged_blocked with q and o in head blocks gives the
    same bits as qcau_decode_attn_paged (same kernel and splits)."""
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    H, ctx, bsz = 128, 2048, 6
    cache, table, _ = make_paged_cache(bsz, ctx, PAGE, WIDTH, dev, seed=11)
    seqlens = torch.tensor([2048, 0, 1, 129, 1500, 640], device=dev, dtype=torch.int32)
    g = torch.Generator(device=dev).manual_seed(12)
    q = torch.randn(bsz, H, WIDTH, device=dev, generator=g).to(torch.bfloat16)
    st = _lib.stream_ptr(dev)
    need = L.qcau_decode_attn_workspace_size(bsz, H, 512, ctx)
    ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
    ref = torch.empty(bsz, H, 512, device=dev, dtype=torch.bfloat16)
    _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                        seqlens.data_ptr(), None, ref.data_ptr(), bsz, H, WIDTH,
                                        512, WIDTH, PAGE, table.size(1), cache.size(0), ctx,
                                        0.07, ws.data_ptr(), need, st), "decode")
    qb = q.view(bsz, H // hb, hb, WIDTH).transpose(0, 1).contiguous()
    ob = torch.empty(H // hb, bsz, hb, 512, device=dev, dtype=torch.bfloat16)
    _lib.check(L.qcau_decode_attn_paged_blocked(qb.data_ptr(), hb, cache.data_ptr(),
                                                table.data_ptr(), seqlens.data_ptr(), None,
                                                ob.data_ptr(), hb, bsz, H, WIDTH, 512, WIDTH, PAGE,
                                                table.size(1), cache.size(0), ctx, 0.07,
                                                ws.data_ptr(), need, st), "blocked")
    got = ob.transpose(0, 1).reshape(bsz, H, 512)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(got, ref)


@pytest.mark.gpu
def test_row_split_stages_one_rank_match_fused_layer():
    """forward_rows at one rank (q stage, blocked attention, out stage)
    gives the bits of the fused qcau_mla_decode."""
    dev = torch.device("cuda", 0)
    cfg = MLAConfig(n_heads=128)
    layer = MLADecodeLayer(cfg, dev, attn_split="rows")
    layer.random_weights(seed=1)
    bsz, ctx = 8, 2048
    cache, table, seqlens = make_paged_cache(bsz, ctx, PAGE, WIDTH, dev, seed=2)
    seqlens[3] = 1000
    g = torch.Generator(device=dev).manual_seed(3)
    q_lora = torch.randn(bsz, cfg.dc, device=dev, generator=g)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    freqs = precompute_freqs_cis(cfg.d_rope, ctx + 1, cfg.rope_theta, dev)
    positions = seqlens.clone()
    y_fused = layer.forward_local(q_lora, cache, table, seqlens, positions, freqs, ctx).clone()
    y_rows = layer.forward_rows(q_lora, cache, table, seqlens, positions, freqs, ctx)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(y_rows, y_fused)


@pytest.mark.gpu
def test_staged_layer_one_rank_matches_fused_layer():
    """forward_context at one rank (q stage, cp attention, combine, out stage)
    equals the fused qcau_mla_decode."""
    dev = torch.device("cuda", 0)
    cfg = MLAConfig(n_heads=128)
    layer = MLADecodeLayer(cfg, dev, attn_split="context")
    layer.random_weights(seed=1)
    bsz, ctx = 8, 2048
    cache, table, seqlens = make_paged_cache(bsz, ctx, PAGE, WIDTH, dev, seed=2)
    seqlens[3] = 1000
    g = torch.Generator(device=dev).manual_seed(3)
    q_lora = torch.randn(bsz, cfg.dc, device=dev, generator=g)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    freqs = precompute_freqs_cis(cfg.d_rope, ctx + 1, cfg.rope_theta, dev)
    positions = seqlens.clone()
    y_fused = layer.forward_local(q_lora, cache, table, seqlens, positions, freqs, ctx)
    y_fused = y_fused.clone()
    y_cp = layer.forward_context(q_lora, cache, table, seqlens, positions, freqs, ctx)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    a, b = y_cp.float(), y_fused.float()
    _assert_layer_close(a.cpu().numpy(), b.cpu().numpy(), "staged vs fused")


def _nccl_rank_main(rank, world_size, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world_size, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        cfg = MLAConfig(n_heads=128)
        bsz, ctx = 16, 4096
        cache, table, seqlens = make_paged_cache(bsz, ctx, PAGE, WIDTH, dev, seed=2)
        g = torch.Generator(device=dev).manual_seed(3)
        q_lora = torch.randn(bsz, cfg.dc, device=dev, generator=g)
        q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
        freqs = precompute_freqs_cis(cfg.d_rope, ctx + 1, cfg.rope_theta, dev)
        positions = seqlens.clone()
        ys = {}
        for name, mode, ex in (("p2p", "context", "p2p"), ("nccl", "context", "nccl"),
                               ("rows", "rows", "nccl"), ("heads", "heads", "nccl")):
            layer = MLADecodeLayer(cfg, dev, rank, world_size, attn_split=mode, exchange=ex)
            layer.random_weights(seed=1)
            for _ in range(3):   # steps alternate the receive areas
                y = layer.forward(q_lora, cache, table, seqlens, positions, freqs, ctx)
            ys[name] = y.clone()
            layer.close()
        if rank == 0:
            full = MLADecodeLayer(cfg, dev)
            full.random_weights(seed=1)
            ys["one"] = full.forward(q_lora, cache, table, seqlens, positions, freqs, ctx).clone()
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        for k, v in ys.items():
            np.save(os.path.join(out_dir, f"{k}{rank}.npy"), v.float().cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_cp_layer_over_nccl_two_gpus(tmp_path):
    """Two ranks: the context-split layer with the exchange fused into the
    attention kernel (peer memory) and with an NCCL all-to-all, the
    row-split layer and the head-split layer, all equal the one-GPU layer."""
    world_size = 2
    mp.start_processes(_nccl_rank_main, args=(world_size, _free_port(), str(tmp_path)),
                       nprocs=world_size, start_method="spawn", join=True)
    ref = np.load(tmp_path / "one0.npy")
    for mode in ("p2p", "nccl", "rows", "heads"):
        for r in range(world_size):
            _assert_layer_close(np.load(tmp_path / f"{mode}{r}.npy"), ref, f"{mode} rank {r}")


def test_row_split_falls_back_to_context_split_for_uneven_batch():
    """attn_split="rows" (the default) runs the row split when the batch
    divides by the ranks and the context split when it does not."""
    called = []

    class Probe(MLADecodeLayer):
        def forward_rows(self, *a, **k):
            called.append("rows")

        def forward_context(self, *a, **k):
            called.append("context")

    layer = Probe(CFG, "cpu", rank=0, world_size=2)
    assert layer.attn_split == "rows"
    for bsz in (2, 3):
        layer.forward(torch.zeros(bsz, CFG.dc), None, None, None, None, None, 0)
    assert called == ["rows", "context"]
