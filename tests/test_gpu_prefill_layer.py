"""The absorbed-MLA layer's prefill step (MLADecodeLayer.forward_prefill)
against the oracle, stage by stage: every new token of every sequence is a
decode row of the oracle layer over the cached prefix up to its own position,
with RoPE at that position (the reference's prefill branch,
Deepseek_origin/inference/model.py:517-528, is the causal attention of the new
tokens over the cache).  Each stage is fed the GPU's previous-stage output,
since one bf16 ulp upstream can flip an FP8 code of the o-proj's input.
"""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_close_attn, f32, n_bf16, n_u8
from test_gpu_parity import _mla_ws_views

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200.mla import MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis


@pytest.mark.parametrize("heads,seqlens,S", [(16, [200, 48], 48), (128, [130, 64], 32)])
def test_prefill_layer_stagewise_vs_oracle(heads, seqlens, S):
    cfg = MLAConfig(n_heads=heads)
    layer = MLADecodeLayer(cfg, "cuda")
    wq, wqs, wkv, wkvs, wo, wos = [t.cpu() for t in layer.random_weights(seed=11)]
    B, ctx, H = len(seqlens), 256, heads
    rows = B * S
    cache, table, _ = make_paged_cache(B, ctx, 64, 576, "cuda", seed=12)
    sl = torch.tensor(seqlens, device="cuda", dtype=torch.int32)
    freqs = precompute_freqs_cis(64, 1024, cfg.rope_theta, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(13)
    q_lora = torch.randn(B, S, cfg.dc, device="cuda", generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    y = layer.forward_prefill(q_lora, cache, table, sl, freqs, ctx)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert y.shape == (B, S, cfg.dim)
    v = _mla_ws_views(layer, rows)
    q_abs, o_lat = layer._prefill["q_abs"], layer._prefill["o_lat"]
    # token t of sequence b: position and visible length seqlens[b] - S + 1 + t
    row_len = np.array([seqlens[b] - S + 1 + t for b in range(B) for t in range(S)], np.int32)
    row_tb = np.repeat(table.cpu().numpy(), S, axis=0)
    fr = freqs.cpu().numpy()
    # q-up + RoPE at each row's position
    xq, xs = O.act_quant(n_bf16(q_lora.reshape(rows, cfg.dc)), 128, False)
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, n_u8(wq), wqs.numpy())).reshape(rows, 1, H, 192)
    q = np.stack([O.rope(q[r:r + 1], fr, 64, int(row_len[r])) for r in range(rows)])[:, 0, 0]
    assert_close_attn(f32(n_bf16(v["q"])), f32(q), f"prefill h{H} q-up + rope")
    # absorb from the GPU's q
    wkv_bf16 = O.f32_to_bf16(O.e4m3_to_f32(n_u8(wkv)) *
                             np.repeat(np.repeat(wkvs.numpy(), 128, 0), 128, 1))
    qg = n_bf16(v["q"])
    ref_abs = np.concatenate([O.mla_absorb(qg, wkv_bf16, 128, 128), qg[..., 128:]], axis=-1)
    assert_close_attn(f32(n_bf16(q_abs)), f32(ref_abs), f"prefill h{H} absorb")
    # causal attention from the GPU's q_abs: row r over its first row_len[r] tokens
    ref_o = O.paged_decode_attn(n_bf16(q_abs), n_bf16(cache), row_tb, row_len, None,
                                cfg.softmax_scale, 512)
    assert_close_attn(f32(n_bf16(o_lat)), f32(O.f32_to_bf16(ref_o)), f"prefill h{H} attention")
    # v-up from the GPU's o_lat; act_quant of the GPU's o_v bit-exact; o-proj
    ref_ov = O.mla_vup(n_bf16(o_lat), wkv_bf16, 128, 128).reshape(rows, H * 128)
    assert_close_attn(f32(n_bf16(v["ov"])), f32(ref_ov), f"prefill h{H} v-up")
    xo, so = O.act_quant(n_bf16(v["ov"]), 128, False)
    assert np.array_equal(n_u8(v["xo"]), xo)
    assert np.array_equal(v["so"].cpu().numpy(), so)
    ref_y = O.f32_to_bf16(O.fp8_gemm(xo, so, n_u8(wo), wos.numpy()))
    assert_close_attn(f32(n_bf16(y.reshape(rows, cfg.dim))), f32(ref_y), f"prefill h{H} o-proj")
