"""GPU parity at the sizes the decode configurations are measured on.

  * the benchmarked decode step: batch 128, 128 heads, 32768 cached tokens per
    sequence (every sequence full length), the paged cache and block table
    built exactly as the benchmark builds them, 4 KV splits; the whole batch
    runs in one launch and sampled sequences (all 128 heads) are compared
    with the oracle;
  * the one-GPU decode configuration: batch 32, 128 heads, a contiguous
    [32, 4096, 576] bf16 cache (an identity block table over 64-token pages),
    one new token per sequence at position 4096, the whole layer stage by
    stage against the oracle.

The benchmarked step (the layer's own query) is held to the strict bar:
every element within 2e-2 * RMS of the oracle, no ulp allowance.  With a
~N(0,1) query (a sharper softmax, outputs up to ~10x their RMS) and at the
one-GPU configuration, a few elements above ~3x RMS land one bf16 ulp from
the oracle's bf16 value (fp32 sums in another order round the other way);
those cases use the one-ulp allowance and the count is reported.
"""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_close_attn, f32, n_bf16, n_u8

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200.mla import MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis

SAMPLED = [0, 37, 90, 127]


def _compact_pages(cache, table_rows):
    """The pages of the sampled sequences gathered into a small cache, and
    their block table remapped onto it (the oracle reads only those)."""
    pages = np.unique(table_rows)
    remap = np.full(int(pages.max()) + 1, -1, dtype=np.int64)
    remap[pages] = np.arange(pages.size)
    sub = cache[torch.from_numpy(pages).to(cache.device).long()]
    return n_bf16(sub), remap[table_rows].astype(np.int32)


def _bench_inputs():
    """The decode benchmark's layer and cache (same seeds and shapes)."""
    B, H, ctx = 128, 128, 32768
    cfg = MLAConfig(n_heads=H)
    layer = MLADecodeLayer(cfg, "cuda")
    layer.random_weights(seed=0)
    cache, table, seqlens = make_paged_cache(B, ctx, 64, 576, "cuda", seed=0)
    freqs = precompute_freqs_cis(64, ctx + 1, cfg.rope_theta, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(1)
    q_lora = torch.randn(B, cfg.dc, device="cuda", generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    return cfg, layer, cache, table, seqlens, freqs, q_lora, gen


@pytest.mark.parametrize("q_kind", ["layer", "randn"])
def test_decode_bench_workload_vs_oracle(q_kind):
    """128 x 32768 full-length sequences, 128 heads, in one launch (the split
    count the library picks for this shape: 4); q is the layer's absorbed
    query of the benchmarked step, or ~N(0,1) as the attention-only timing
    uses (sharper softmax)."""
    cfg, layer, cache, table, seqlens, freqs, q_lora, gen = _bench_inputs()
    B, H, ctx = 128, 128, 32768
    if q_kind == "layer":
        q = torch.empty(B, H, 576, device="cuda", dtype=torch.bfloat16)
        d = layer.dims(B, table.size(1), cache.size(0), ctx, freqs.size(0))
        layer._q_stage(d, q_lora, seqlens.clone(), freqs, q)
    else:
        q = torch.randn(B, H, 576, device="cuda", generator=gen).to(torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_decode_attn_workspace_size(B, H, 512, ctx)
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    o = torch.empty(B, H, 512, device="cuda", dtype=torch.bfloat16)
    _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                        seqlens.data_ptr(), None, o.data_ptr(), B, H, 576, 512,
                                        576, 64, table.size(1), cache.size(0), ctx,
                                        cfg.softmax_scale, ws.data_ptr(), need,
                                        _lib.stream_ptr()), "decode_attn_paged")
    assert _lib.device_error() == 0
    # 4 splits: partials for 128 x 4 x 128 rows of 512 fp16 + (max, sum)
    assert need >= B * 4 * H * (512 * 2 + 8)
    sub, tsub = _compact_pages(cache, table.cpu().numpy()[SAMPLED])
    ref = O.paged_decode_attn(n_bf16(q[SAMPLED]), sub, tsub, np.full(len(SAMPLED), ctx, np.int32),
                              None, cfg.softmax_scale, 512)
    assert_close_attn(f32(n_bf16(o[SAMPLED])), f32(O.f32_to_bf16(ref)),
                      f"bench workload ({q_kind} q)", strict=q_kind == "layer")


def test_decode_one_gpu_config_layer_stagewise():
    """Batch 32, 128 heads, contiguous 4096-token cache per sequence, new
    token at position 4096: each stage of the layer against the oracle fed
    with the GPU's previous stage; the attention over all 32 sequences."""
    from test_gpu_parity import _mla_ws_views

    B, H, ctx = 32, 128, 4096
    cfg = MLAConfig(n_heads=H)
    layer = MLADecodeLayer(cfg, "cuda")
    wq, wqs, wkv, wkvs, wo, wos = [t.cpu() for t in layer.random_weights(seed=0)]
    gen = torch.Generator(device="cuda").manual_seed(11)
    rows = torch.randn(B, ctx, 576, device="cuda", generator=gen)
    rows = (rows * torch.rsqrt(rows.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    cache = rows.view(B * ctx // 64, 64, 576)            # the contiguous cache as pages
    table = torch.arange(B * ctx // 64, device="cuda", dtype=torch.int32).view(B, ctx // 64)
    seqlens = torch.full((B,), ctx, device="cuda", dtype=torch.int32)
    positions = seqlens.clone()
    freqs = precompute_freqs_cis(64, ctx + 1, cfg.rope_theta, "cuda")
    q_lora = torch.randn(B, cfg.dc, device="cuda", generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    y = layer.forward(q_lora, cache, table, seqlens, positions, freqs, ctx)
    assert _lib.device_error() == 0
    v = _mla_ws_views(layer, B)
    xq, xs = O.act_quant(n_bf16(q_lora), 128, False)
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, n_u8(wq), wqs.numpy())).reshape(B, 1, H, 192)
    fr = freqs.cpu().numpy()
    q = np.stack([O.rope(q[b:b + 1], fr, 64, int(positions[b])) for b in range(B)])[:, 0, 0]
    assert_close_attn(f32(n_bf16(v["q"])), f32(q), "cfg1 q-up + rope")
    wkv_bf16 = O.f32_to_bf16(O.e4m3_to_f32(n_u8(wkv)) *
                             np.repeat(np.repeat(wkvs.numpy(), 128, 0), 128, 1))
    qg = n_bf16(v["q"])
    q_abs = np.concatenate([O.mla_absorb(qg, wkv_bf16, 128, 128), qg[..., 128:]], axis=-1)
    assert_close_attn(f32(n_bf16(v["qabs"])), f32(q_abs), "cfg1 absorb")
    o_lat = O.paged_decode_attn(n_bf16(v["qabs"]), n_bf16(cache), table.cpu().numpy(),
                                seqlens.cpu().numpy(), None, cfg.softmax_scale, 512)
    assert_close_attn(f32(n_bf16(v["olat"])), f32(O.f32_to_bf16(o_lat)), "cfg1 attention")
    o_v = O.mla_vup(n_bf16(v["olat"]), wkv_bf16, 128, 128).reshape(B, H * 128)
    assert_close_attn(f32(n_bf16(v["ov"])), f32(o_v), "cfg1 v-up")
    xo, so = O.act_quant(n_bf16(v["ov"]), 128, False)
    assert np.array_equal(n_u8(v["xo"]), xo)
    assert np.array_equal(v["so"].cpu().numpy(), so)
    ref = O.f32_to_bf16(O.fp8_gemm(xo, so, n_u8(wo), wos.numpy()))
    assert_close_attn(f32(n_bf16(y)), f32(ref), "cfg1 o-proj")
