"""GPU parity of the sm_100a kernels against the oracle and the reference's
golden vectors.  Every call goes through the C ABI of libqcau_b200.so (via the
qcau_b200 drop-ins).  Tolerances are those of tests/helpers.py."""

import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_close_attn, cosine, f32, n_bf16, n_u8, t_bf16, t_u8

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import qcau_b200
    from qcau_b200 import _lib, kernel
    from qcau_b200.mla import MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis


def _no_device_error():
    assert _lib.device_error() == 0


# ------------------------------------------------------------------ act_quant

def test_act_quant_36_goldens_bitwise(golden_dir):
    g = np.load(golden_dir / "act_quant_goldens.npz")
    for c in g["cases"]:
        x = t_bf16(g[f"{c}/c_q"])
        y, s = kernel.act_quant(x, 128, "ue8m0", torch.float8_e8m0fnu)
        assert np.array_equal(n_u8(y), g[f"{c}/x"]), c
        assert np.array_equal(n_u8(s), g[f"{c}/s"]), c
    _no_device_error()


def test_act_quant_modes_bitwise(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    x = t_bf16(g["aq/x"])
    y, s = kernel.act_quant(x, 128, None, torch.float32)
    assert np.array_equal(n_u8(y), g["aq/y_f32"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), g["aq/s_f32"].view(np.uint32))
    y, s = kernel.act_quant(x, 128, "ue8m0", torch.float8_e8m0fnu)
    assert np.array_equal(n_u8(y), g["aq/y_ue8m0"])
    assert np.array_equal(n_u8(s), g["aq/s_ue8m0"])
    kv = x[:, :448].clone()
    kernel.act_quant(kv, 64, "ue8m0", torch.float8_e8m0fnu, inplace=True)
    assert np.array_equal(n_bf16(kv), g["aq/inplace64"])


def test_act_quant_prefill_size_bitwise():
    """The prefill activation size [16384, 1536] against the oracle."""
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.randn(16384, 1536, device="cuda", generator=gen) * 4).to(torch.bfloat16)
    x[7, :128] = 0
    y, s = kernel.act_quant(x, 128, None, torch.float32)
    yo, so = O.act_quant(n_bf16(x), 128, False)
    assert np.array_equal(n_u8(y), yo)
    assert np.array_equal(s.cpu().numpy(), so)


# ------------------------------------------------------------------ fp8_gemm

def test_fp8_gemm_matches_reference(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        c = kernel.fp8_gemm(t_u8(g["gemm/a"]), torch.from_numpy(g["gemm/sa"]).cuda(),
                            t_u8(g["gemm/b"]), torch.from_numpy(g["gemm/sb"]).cuda())
    finally:
        torch.set_default_dtype(prev)
    got = f32(n_bf16(c))
    ref = f32(g["gemm/c_bf16"])
    assert np.mean(got == ref) > 0.99
    assert cosine(got, ref) > 0.99999
    assert np.abs(got - ref).max() <= 2 ** -7 * np.abs(ref).max()


@pytest.mark.parametrize("m", [1, 32, 128, 200])
@pytest.mark.parametrize("e8m0", [False, True])
def test_fp8_gemm_shapes(m, e8m0):
    gen = torch.Generator(device="cuda").manual_seed(m)
    n, k = 384, 1536
    a = (torch.randn(m, k, device="cuda", generator=gen) * 2).to(torch.bfloat16)
    w = torch.randn(n, k, device="cuda", generator=gen) * 0.02
    sdt = torch.float8_e8m0fnu if e8m0 else torch.float32
    aq, asc = kernel.act_quant(a, 128, "ue8m0" if e8m0 else None, sdt)
    wq, wsc = qcau_b200.mla.quantize_weight_fp8(w, e8m0)
    c = kernel.fp8_gemm(aq, asc, wq, wsc, sdt)  # default dtype fp32 -> fp32 output
    assert c.dtype == torch.float32
    sa = asc.float().cpu().numpy() if not e8m0 else O.e8m0_to_f32(n_u8(asc))
    sb = wsc.float().cpu().numpy() if not e8m0 else O.e8m0_to_f32(n_u8(wsc))
    ref = O.fp8_gemm(n_u8(aq), sa, n_u8(wq), sb)
    got = c.cpu().numpy()
    assert cosine(got, ref) > 0.99999
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-6


# ------------------------------------------------------------------ attention

def _sparse_attn_abi(q, kv, sink, idx, scale, inv_rope=False, freqs=None, pos0=0):
    B, S, H, D = q.shape
    o = torch.empty_like(q)
    f = freqs if freqs is not None else None
    _lib.check(_lib.lib().qcau_sparse_attn(
        q.data_ptr(), kv.data_ptr(), None if sink is None else sink.data_ptr(), idx.data_ptr(),
        o.data_ptr(), B, S, H, D, D, kv.size(-1), kv.size(1), idx.size(-1), float(scale),
        int(inv_rope), None if f is None else f.data_ptr(), 64, 0 if f is None else f.size(0),
        pos0, _lib.stream_ptr()), "sparse_attn")
    return o


def test_sparse_attn_inverse_rope_36_goldens(golden_dir):
    g = np.load(golden_dir / "attn_goldens.npz")
    exact = total = 0
    for c in g["cases"]:
        q = t_bf16(g[f"{c}/q"])
        kv = t_bf16(g[f"{c}/kv"])
        idx = torch.from_numpy(g[f"{c}/idx"]).cuda()
        sink = torch.from_numpy(g[f"{c}/sink"]).cuda()
        freqs = torch.from_numpy(g[f"{c}/freqs"]).cuda()
        o = _sparse_attn_abi(q, kv, sink, idx, float(g[f"{c}/scale"]), True, freqs)
        got = n_bf16(o)
        ref = g[f"{c}/qcau_o"]
        exact += int(np.sum(got == ref))
        total += got.size
        assert_close_attn(f32(got), f32(ref), c)
    # most values are bit-identical with the TileLang golden output
    assert exact / total > 0.8
    _no_device_error()


def test_sparse_attn_matches_reference_edge_cases(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    o = kernel.sparse_attn(t_bf16(g["attn/q"]), t_bf16(g["attn/kv"]),
                           torch.from_numpy(g["attn/sink"]).cuda(),
                           torch.from_numpy(g["attn/idx"]).cuda(), float(g["attn/scale"]))
    assert_close_attn(f32(n_bf16(o)), f32(g["attn/o"]), "synthetic")


@pytest.mark.parametrize("h,topk,n", [(1, 1, 5), (3, 63, 70), (17, 64, 64), (16, 65, 300),
                                      (64, 200, 1000), (5, 130, 40)])
def test_sparse_attn_shapes_vs_oracle(h, topk, n):
    gen = torch.Generator(device="cuda").manual_seed(h * 1000 + topk)
    B, S, D = 2, 3, 512
    q = torch.randn(B, S, h, D, device="cuda", generator=gen).to(torch.bfloat16)
    kv = torch.randn(B, n, D, device="cuda", generator=gen).to(torch.bfloat16)
    idx = torch.randint(-1, n + 2, (B, S, topk), device="cuda", generator=gen, dtype=torch.int32)
    idx[0, 0, :] = -1  # a query with no valid key -> zeros
    sink = torch.randn(h, device="cuda", generator=gen)
    o = kernel.sparse_attn(q, kv, sink, idx, D ** -0.5)
    ref = O.sparse_attn(n_bf16(q), n_bf16(kv), sink.cpu().numpy(), idx.cpu().numpy(), D ** -0.5)
    got = f32(n_bf16(o))
    assert np.all(got[0, 0] == 0)
    assert_close_attn(got, f32(O.f32_to_bf16(ref)), f"h{h} k{topk}")


# ------------------------------------------------------------------ FP8 latent cache (top-k gather)

def _fp8_cache(B, N, gen, device="cuda"):
    """Random FP8 latent cache: e4m3 codes (no NaN code), one fp32 scale per
    row, bf16 rope part."""
    mag = torch.randint(0, 0x7F, (B, N, 512), device=device, generator=gen, dtype=torch.uint8)
    sign = torch.randint(0, 2, (B, N, 512), device=device, generator=gen, dtype=torch.uint8) << 7
    codes = (mag | sign).contiguous()
    scale = (torch.rand(B, N, device=device, generator=gen) * 0.01 + 1e-3).contiguous()
    rope = torch.randn(B, N, 64, device=device, generator=gen).to(torch.bfloat16).contiguous()
    return codes, scale, rope


def _fp8_rows_bf16(codes_u8, scale, rope_u16):
    """The rows' values as the kernel sees them: bf16(e4m3 * scale) ‖ rope."""
    lat = O.f32_to_bf16(O.e4m3_to_f32(codes_u8) * scale[..., None].astype(np.float32))
    return np.concatenate([lat, rope_u16], axis=-1)


def _sparse_fp8_abi(q, codes, scale, rope, sink, idx, sm_scale):
    B, S, H, _ = q.shape
    o = torch.empty(B, S, H, 512, device="cuda", dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_sparse_attn_fp8_workspace_size(B, S, H, idx.size(-1))
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    _lib.check(L.qcau_sparse_attn_fp8(q.data_ptr(), codes.data_ptr(), scale.data_ptr(),
                                      rope.data_ptr(), None if sink is None else sink.data_ptr(),
                                      idx.data_ptr(), o.data_ptr(), B, S, H, codes.size(1),
                                      idx.size(-1), float(sm_scale), ws.data_ptr(), need,
                                      _lib.stream_ptr()), "sparse_attn_fp8")
    return o


@pytest.mark.parametrize("h", [16, 128])
def test_sparse_attn_fp8_vs_oracle(h):
    gen = torch.Generator(device="cuda").manual_seed(77 + h)
    B, S, N, K = 2, 2, 5000, 2048
    codes, scale, rope = _fp8_cache(B, N, gen)
    q = torch.randn(B, S, h, 576, device="cuda", generator=gen).to(torch.bfloat16)
    idx = torch.randint(-1, N, (B, S, K), device="cuda", generator=gen, dtype=torch.int32)
    idx[1, 1, :] = -1  # a query with no valid key -> zeros
    sink = torch.randn(h, device="cuda", generator=gen)
    o = _sparse_fp8_abi(q, codes, scale, rope, sink, idx, 192 ** -0.5)
    assert _lib.device_error() == 0
    kv = _fp8_rows_bf16(n_u8(codes), scale.cpu().numpy(), n_bf16(rope))
    ref = O.sparse_attn(n_bf16(q), kv, sink.cpu().numpy(), idx.cpu().numpy(), 192 ** -0.5, 512)
    got = f32(n_bf16(o))
    assert np.all(got[1, 1] == 0)
    assert_close_attn(got, f32(O.f32_to_bf16(ref)), f"fp8 sparse h{h}")


def test_sparse_attn_fp8_long_context_sampled():
    """The long-context sparse decode configuration at its per-rank shape of
    an 8-GPU head shard: batch 64, 131072 cached rows per sequence (FP8
    latent + fp32 row scale + bf16 rope), top-2048 indices drawn without
    replacement, 16 heads; sampled sequences against the oracle."""
    gen = torch.Generator(device="cuda").manual_seed(131072)
    B, N, K, H = 64, 131072, 2048, 16
    codes, scale, rope = _fp8_cache(B, N, gen)
    q = torch.randn(B, 1, H, 576, device="cuda", generator=gen)
    q = (q * torch.rsqrt(q.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(N, device="cuda", generator=gen)[:K] for _ in range(B)])
    idx = idx.to(torch.int32).view(B, 1, K).contiguous()
    sink = torch.randn(H, device="cuda", generator=gen)
    o = _sparse_fp8_abi(q, codes, scale, rope, sink, idx, 192 ** -0.5)
    assert _lib.device_error() == 0
    assert bool(torch.isfinite(o.float()).all())
    for b in (0, 31, 63):
        rows = idx[b, 0].long()
        kv = _fp8_rows_bf16(n_u8(codes[b, rows]), scale[b, rows].cpu().numpy(),
                            n_bf16(rope[b, rows]))[None]
        local = np.arange(K, dtype=np.int32).reshape(1, 1, K)
        ref = O.sparse_attn(n_bf16(q[b:b + 1]), kv, sink.cpu().numpy(), local, 192 ** -0.5, 512)
        assert_close_attn(f32(n_bf16(o[b:b + 1])), f32(O.f32_to_bf16(ref)), f"long ctx b{b}")


def test_sparse_attn_reference_fp8_roundtrip_cache():
    """The reference's own FP8 cache: the 512 non-rope values of each row go
    through act_quant(block 64, UE8M0, inplace) and stay bf16 (model.py:505);
    sparse_attn then reads that bf16 cache."""
    gen = torch.Generator(device="cuda").manual_seed(505)
    B, S, N, K, H = 2, 1, 3000, 512, 64
    kv = torch.randn(B, N, 576, device="cuda", generator=gen).to(torch.bfloat16)
    kv0 = n_bf16(kv).copy()
    lat = kv[..., :512].contiguous()
    kernel.act_quant(lat, 64, "ue8m0", torch.float8_e8m0fnu, inplace=True)
    kv[..., :512] = lat
    q = torch.randn(B, S, H, 576, device="cuda", generator=gen).to(torch.bfloat16)
    idx = torch.randint(-1, N, (B, S, K), device="cuda", generator=gen, dtype=torch.int32)
    sink = torch.randn(H, device="cuda", generator=gen)
    o = torch.empty(B, S, H, 512, device="cuda", dtype=torch.bfloat16)
    _lib.check(_lib.lib().qcau_sparse_attn(
        q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(), o.data_ptr(), B, S, H, 576,
        512, 576, N, K, float(192 ** -0.5), 0, None, 64, 0, 0, _lib.stream_ptr()), "sparse_attn")
    kv_ref = kv0.copy()
    kv_ref[..., :512] = O.act_quant_inplace(kv0[..., :512].copy(), 64, True)
    assert np.array_equal(kv_ref, n_bf16(kv))  # the round trip is bit-exact
    ref = O.sparse_attn(n_bf16(q), kv_ref, sink.cpu().numpy(), idx.cpu().numpy(), 192 ** -0.5, 512)
    assert_close_attn(f32(n_bf16(o)), f32(O.f32_to_bf16(ref)), "reference fp8 cache")


# ------------------------------------------------------------------ QCAU block

def _qcau_inputs(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    w = t_u8(g["qcau/w"])
    w.scale = t_u8(g["qcau/w_scale_e8m0"], torch.float8_e8m0fnu)
    freqs = torch.view_as_complex(torch.from_numpy(g["qcau/freqs"]).contiguous()).cuda()
    return g, w, freqs


def test_qcau_fused_matches_reference(golden_dir):
    g, w, freqs = _qcau_inputs(golden_dir)
    o = qcau_b200.QCAU(c_q=t_bf16(g["qcau/c_q"]), w_uq=w, kv=t_bf16(g["qcau/kv"]),
                       topk_idxs=torch.from_numpy(g["qcau/idx"]).cuda(),
                       attn_sink=torch.from_numpy(g["qcau/sink"]).cuda(), freqs_cis=freqs,
                       n_local_heads=g["qcau/sink"].shape[0])
    assert_close_attn(f32(n_bf16(o)), f32(g["qcau/o"]), "QCAU fused")
    _no_device_error()


def test_qcau_callable_projector_matches_reference(golden_dir):
    g, w, freqs = _qcau_inputs(golden_dir)

    def projector(x):
        xq, xs = kernel.act_quant(x, 128, "ue8m0", torch.float8_e8m0fnu)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            return kernel.fp8_gemm(xq, xs, w, w.scale, torch.float8_e8m0fnu)
        finally:
            torch.set_default_dtype(prev)

    o = qcau_b200.QCAU(c_q=t_bf16(g["qcau/c_q"]), w_uq=projector, kv=t_bf16(g["qcau/kv"]),
                       topk_idxs=torch.from_numpy(g["qcau/idx"]).cuda(),
                       attn_sink=torch.from_numpy(g["qcau/sink"]).cuda(), freqs_cis=freqs)
    assert_close_attn(f32(n_bf16(o)), f32(g["qcau/o"]), "QCAU callable")


def test_qcau_validation_messages(golden_dir):
    g, w, freqs = _qcau_inputs(golden_dir)
    with pytest.raises(ValueError, match="attn_sink must match"):
        qcau_b200.QCAU(c_q=t_bf16(g["qcau/c_q"]), w_uq=w, kv=t_bf16(g["qcau/kv"]),
                       topk_idxs=torch.from_numpy(g["qcau/idx"]).cuda(),
                       attn_sink=torch.zeros(5, device="cuda"), freqs_cis=freqs)
    with pytest.raises(ValueError, match="freqs_cis does not cover"):
        qcau_b200.QCAU(c_q=t_bf16(g["qcau/c_q"]), w_uq=w, kv=t_bf16(g["qcau/kv"]),
                       topk_idxs=torch.from_numpy(g["qcau/idx"]).cuda(),
                       attn_sink=torch.from_numpy(g["qcau/sink"]).cuda(), freqs_cis=freqs[:1],
                       start_pos=3)


# ------------------------------------------------------------------ paged decode

def _decode_abi(q, cache, table, seqlens, sink, scale, d_v, max_seqlen):
    B, H, dqk = q.shape
    o = torch.empty(B, H, d_v, device="cuda", dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_decode_attn_workspace_size(B, H, d_v, max_seqlen)
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                        seqlens.data_ptr(), None if sink is None else sink.data_ptr(),
                                        o.data_ptr(), B, H, dqk, d_v, cache.size(-1),
                                        cache.size(1), table.size(1), cache.size(0), max_seqlen,
                                        float(scale), ws.data_ptr(), need, _lib.stream_ptr()),
               "decode_attn_paged")
    return o


# 8 and 48 heads run the tcgen05 gather kernel (paged mode), 128 the tcgen05 pair kernel
@pytest.mark.parametrize("h,seqlens", [(8, [1, 100, 1000]), (128, [4096, 64, 777]),
                                       (48, [0, 2000, 513])])
def test_decode_paged_vs_oracle(h, seqlens):
    gen = torch.Generator(device="cuda").manual_seed(h)
    B, page, width = len(seqlens), 64, 576
    max_pages = (max(seqlens) + page - 1) // page
    pages = B * max_pages + 3
    cache = torch.randn(pages, page, width, device="cuda", generator=gen).to(torch.bfloat16)
    table = torch.randperm(pages, device="cuda", generator=gen)[:B * max_pages]
    table = table.view(B, max_pages).to(torch.int32).contiguous()
    sl = torch.tensor(seqlens, device="cuda", dtype=torch.int32)
    q = torch.randn(B, h, width, device="cuda", generator=gen).to(torch.bfloat16)
    sink = torch.randn(h, device="cuda", generator=gen)
    scale = 192 ** -0.5
    o = _decode_abi(q, cache, table, sl, sink, scale, 512, max(seqlens))
    ref = O.paged_decode_attn(n_bf16(q), n_bf16(cache), table.cpu().numpy(), sl.cpu().numpy(),
                              sink.cpu().numpy(), scale, 512)
    assert_close_attn(f32(n_bf16(o)), f32(O.f32_to_bf16(ref)), f"decode h{h}")
    _no_device_error()


# ------------------------------------------------------------------ absorbed decode layer

def _oracle_layer(layer, weights, q_lora, cache, table, seqlens, positions, freqs):
    c = layer.cfg
    wq, wqs, wkv, wkvs, wo, wos = [t.cpu() for t in weights]
    B, H = q_lora.shape[0], c.n_heads
    xq, xs = O.act_quant(n_bf16(q_lora), 128, False)
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, n_u8(wq), wqs.numpy()))
    q = q.reshape(B, 1, H, 192)
    # RoPE of q_rope at each sequence's position
    qr = np.stack([O.rope(q[b:b + 1], freqs, 64, int(positions[b])) for b in range(B)])[:, 0]
    qr = qr.reshape(B, H, 192)
    wkv_bf16 = O.f32_to_bf16(O.e4m3_to_f32(n_u8(wkv)) *
                             np.repeat(np.repeat(wkvs.numpy(), 128, 0), 128, 1))
    q_lat = O.mla_absorb(qr, wkv_bf16, 128, 128)
    q_abs = np.concatenate([q_lat, qr[..., 128:]], axis=-1)
    o_lat = O.paged_decode_attn(q_abs, n_bf16(cache), table, seqlens, None, c.softmax_scale, 512)
    o_v = O.mla_vup(O.f32_to_bf16(o_lat), wkv_bf16, 128, 128).reshape(B, H * 128)
    xo, so = O.act_quant(o_v, 128, False)
    return O.fp8_gemm(xo, so, n_u8(wo), wos.numpy())


def test_mla_decode_layer_vs_oracle():
    cfg = MLAConfig(n_heads=16)
    layer = MLADecodeLayer(cfg, "cuda")
    weights = layer.random_weights(seed=1)
    B, ctx = 4, 256
    cache, table, seqlens = make_paged_cache(B, ctx, 64, 576, "cuda", seed=2)
    seqlens = torch.tensor([256, 1, 130, 64], device="cuda", dtype=torch.int32)
    positions = seqlens.clone()
    freqs = precompute_freqs_cis(64, 1024, cfg.rope_theta, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    q_lora = torch.randn(B, cfg.dc, device="cuda", generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    y = layer.forward(q_lora, cache, table, seqlens, positions, freqs, ctx)
    ref = _oracle_layer(layer, weights, q_lora, cache, table.cpu().numpy(),
                        seqlens.cpu().numpy(), positions.cpu().numpy(), freqs.cpu().numpy())
    assert_close_attn(f32(n_bf16(y)), f32(O.f32_to_bf16(ref)), "mla decode layer")
    _no_device_error()


# ------------------------------------------------------------------ tcgen05 two-CTA decode kernel

@pytest.mark.parametrize("h,seqlens", [(128, [4096, 64, 777, 1]), (128, [0, 130, 2000]),
                                       (256, [513, 128, 3000]), (64, [1000, 1, 3000, 256]),
                                       (32, [513, 0, 2048]), (16, [77, 4096])])
def test_decode_paged_two_cta_vs_oracle(h, seqlens):
    """h a multiple of 128 (or a head shard of 64, 32 or 16) with 576/512
    widths and 64-token pages runs the tcgen05 pair kernel."""
    gen = torch.Generator(device="cuda").manual_seed(7 + h + len(seqlens))
    B, page, width = len(seqlens), 64, 576
    max_pages = (max(seqlens) + page - 1) // page
    pages = B * max_pages + 5
    cache = torch.randn(pages, page, width, device="cuda", generator=gen)
    cache = (cache * torch.rsqrt(cache.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    table = torch.randperm(pages, device="cuda", generator=gen)[:B * max_pages]
    table = table.view(B, max_pages).to(torch.int32).contiguous()
    sl = torch.tensor(seqlens, device="cuda", dtype=torch.int32)
    q = torch.randn(B, h, width, device="cuda", generator=gen).to(torch.bfloat16)
    scale = 192 ** -0.5
    o = _decode_abi(q, cache, table, sl, None, scale, 512, max(seqlens))
    assert _lib.device_error() == 0
    ref = O.paged_decode_attn(n_bf16(q), n_bf16(cache), table.cpu().numpy(), sl.cpu().numpy(),
                              None, scale, 512)
    assert_close_attn(f32(n_bf16(o)), f32(O.f32_to_bf16(ref)), f"two-cta h{h} {seqlens}")


def _ragged_decode_case(h, B, max_len, seed, full=False):
    """Paged decode inputs with ragged lengths: empty sequences, one token,
    page and tile edges, and sequences with fewer tiles than splits; with
    `full`, lengths within 5 % of max_len (page and tile edges below it)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    page, width = 64, 576
    if full:
        special = [max(max_len - d, 1) for d in (129, 128, 127, 64, 63, 1, 0)]
        low = max_len - max_len // 20
    else:
        special = [0, 1, 63, 64, 127, 128, 129, max_len]
        low = 0
    if B <= len(special):  # the longest ones
        sl_l = special[len(special) - B:]
    else:
        sl_l = special + torch.randint(low, max_len + 1, (B - len(special),), generator=gen,
                                       device="cuda").tolist()
    max_pages = (max_len + page - 1) // page
    pages = B * max_pages + 3
    cache = torch.randn(pages, page, width, device="cuda", generator=gen)
    cache = (cache * torch.rsqrt(cache.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    table = torch.randperm(pages, device="cuda", generator=gen)[:B * max_pages]
    table = table.view(B, max_pages).to(torch.int32).contiguous()
    sl = torch.tensor(sl_l, device="cuda", dtype=torch.int32)
    q = torch.randn(B, h, width, device="cuda", generator=gen).to(torch.bfloat16)
    sink = torch.randn(h, device="cuda", generator=gen)
    return q, cache, table, sl, sink


# More (row, head group, split) units than CTA pairs fit at once, so each
# pair runs several in turn: 100 x 128 heads to 8192 tokens in 2 splits, 80
# short sequences in one, 16 sequences in 4 splits, one sequence in 16, and
# 256 heads (two head groups a row).  Lengths spread from 0 to max_seqlen,
# or all within 5 % of it (`full`: long softmax sums, where a page's weight
# missing from a denominator shows as ~0.8 % on the largest outputs; a
# schedule that cut rows into uneven pieces failed exactly that way).
@pytest.mark.parametrize("h,B,max_len,full", [
    (128, 100, 8192, True), (128, 100, 8192, False), (128, 80, 600, True),
    (128, 80, 600, False), (128, 16, 8192, True), (128, 16, 8192, False),
    (128, 1, 8192, True), (256, 24, 4096, True), (256, 24, 4096, False)])
def test_decode_paged_two_cta_more_units_than_pairs(h, B, max_len, full):
    """Ragged sequences (empty, one token, page and tile edges, full
    length) against the oracle."""
    q, cache, table, sl, sink = _ragged_decode_case(h, B, max_len, 1000 + h + B, full)
    scale = 192 ** -0.5
    o = _decode_abi(q, cache, table, sl, sink, scale, 512, max_len)
    assert _lib.device_error() == 0
    ref = O.paged_decode_attn(n_bf16(q), n_bf16(cache), table.cpu().numpy(), sl.cpu().numpy(),
                              sink.cpu().numpy(), scale, 512)
    assert_close_attn(f32(n_bf16(o)), f32(O.f32_to_bf16(ref)), f"units > pairs h{h} B{B}")


# (batch, sub-batch, max_len): 100 rows in 2 splits (200 units) against 4 x 25
# rows (50 units each); 150 rows in one split against 3 x 50 rows.  The split
# count of the full batch and of its sub-batches is the same.
@pytest.mark.parametrize("h", [128, 16])
@pytest.mark.parametrize("B,sub,max_len", [(100, 25, 2048), (150, 50, 600)])
def test_decode_paged_units_loop_bit_exact(h, B, sub, max_len):
    """A pair that runs several units in turn gives the same bits as one pair
    per unit: the batch in one launch (more units than resident pairs) against
    its sub-batches in separate launches (fewer units than pairs)."""
    q, cache, table, sl, sink = _ragged_decode_case(h, B, max_len, 2000 + h + B)
    scale = 192 ** -0.5
    whole = _decode_abi(q, cache, table, sl, sink, scale, 512, max_len)
    parts = torch.cat([_decode_abi(q[i:i + sub], cache, table[i:i + sub], sl[i:i + sub], sink,
                                   scale, 512, max_len) for i in range(0, B, sub)])
    assert _lib.device_error() == 0
    assert torch.equal(whole, parts), "the unit loop changed the result"
    assert bool(torch.isfinite(whole.float()).all())


# ------------------------------------------------------------------ causal prefill (paged)

def _prefill_abi(q, cache, table, seqlens, sink, scale, max_seqlen):
    B, S, H, dqk = q.shape
    o = torch.empty(B, S, H, 512, device="cuda", dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_prefill_attn_workspace_size(B, S, H, 512, max_seqlen)
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    _lib.check(L.qcau_prefill_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                         seqlens.data_ptr(),
                                         None if sink is None else sink.data_ptr(), o.data_ptr(),
                                         B, S, H, dqk, 512, cache.size(-1), cache.size(1),
                                         table.size(1), cache.size(0), max_seqlen, float(scale),
                                         ws.data_ptr(), need, _lib.stream_ptr()),
               "prefill_attn_paged")
    return o


def _prefill_oracle(q, cache, table, seqlens, sink, scale, rows):
    """Oracle of query rows [(b, t)]: row (b, t) is a decode row over the
    first seqlens[b] - S + 1 + t cached tokens of sequence b."""
    S = q.shape[1]
    qn = n_bf16(q)
    tb, sl = table.cpu().numpy(), seqlens.cpu().numpy()
    q_rows = np.stack([qn[b, t] for b, t in rows])
    t_rows = np.stack([tb[b] for b, _ in rows]).astype(np.int32)
    l_rows = np.array([sl[b] - (S - 1 - t) for b, t in rows], dtype=np.int32)
    return O.paged_decode_attn(q_rows, n_bf16(cache), t_rows, l_rows,
                               None if sink is None else sink.cpu().numpy(), scale, 512)


# 128 heads run the tcgen05 pair kernel, 48 the tcgen05 gather kernel (paged mode)
@pytest.mark.parametrize("h", [128, 48])
def test_prefill_paged_vs_oracle(h):
    """Causal prefill of 200 new tokens: sequence 0 holds only them, sequence
    1 has 100 tokens already cached before them."""
    gen = torch.Generator(device="cuda").manual_seed(31 + h)
    B, S, page, width = 2, 200, 64, 576
    seqlens_l = [200, 300]
    max_pages = (max(seqlens_l) + page - 1) // page
    pages = B * max_pages + 2
    cache = torch.randn(pages, page, width, device="cuda", generator=gen)
    cache = (cache * torch.rsqrt(cache.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    table = torch.randperm(pages, device="cuda", generator=gen)[:B * max_pages]
    table = table.view(B, max_pages).to(torch.int32).contiguous()
    sl = torch.tensor(seqlens_l, device="cuda", dtype=torch.int32)
    q = torch.randn(B, S, h, width, device="cuda", generator=gen).to(torch.bfloat16)
    sink = torch.randn(h, device="cuda", generator=gen)
    scale = 192 ** -0.5
    o = _prefill_abi(q, cache, table, sl, sink, scale, max(seqlens_l))
    assert _lib.device_error() == 0
    rows = [(b, t) for b in range(B) for t in range(S)]
    ref = _prefill_oracle(q, cache, table, sl, sink, scale, rows)
    got = f32(n_bf16(o)).reshape(B * S, h, 512)
    assert_close_attn(got, f32(O.f32_to_bf16(ref)), f"prefill h{h}")


def test_prefill_full_size_sampled_rows():
    """The causal prefill configuration at full size (batch 4 x 4096 tokens x
    128 heads, 576-wide paged cache): every output row is finite and sampled
    rows (first token, tile edges, last token) match the oracle."""
    gen = torch.Generator(device="cuda").manual_seed(4096)
    B, S, H, page, width = 4, 4096, 128, 64, 576
    from qcau_b200.mla import make_paged_cache
    cache, table, sl = make_paged_cache(B, S, page, width, "cuda", seed=9)
    q = torch.randn(B, S, H, width, device="cuda", generator=gen)
    q = (q * torch.rsqrt(q.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    sink = torch.randn(H, device="cuda", generator=gen)
    scale = 192 ** -0.5
    o = _prefill_abi(q, cache, table, sl, sink, scale, S)
    assert _lib.device_error() == 0
    assert bool(torch.isfinite(o.float()).all())
    rows = [(0, 0), (0, 255), (1, 256), (2, 2047), (3, 4095), (1, 3000)]
    ref = _prefill_oracle(q, cache, table, sl, sink, scale, rows)
    got = np.stack([f32(n_bf16(o[b, t])) for b, t in rows])
    assert_close_attn(got, f32(O.f32_to_bf16(ref)), "prefill full size")


def _mla_ws_views(layer, B):
    """Views of the decode layer's intermediates inside its workspace (the
    layout of qcau_mla_decode: x_q, s_q, q, q_abs, o_lat, o_v, x_o, s_o, ...)."""
    H = layer.n_local
    c = layer.cfg
    al = lambda n: (n + 255) // 256 * 256
    sizes = [("xq", B * c.dc), ("sq", B * (c.dc // 128) * 4), ("q", B * H * 192 * 2),
             ("qabs", B * H * 576 * 2), ("olat", B * H * 512 * 2), ("ov", B * H * 128 * 2),
             ("xo", B * H * 128), ("so", B * H * 4)]
    off, views = 0, {}
    for name, n in sizes:
        views[name] = layer._ws[off:off + n]
        off += al(n)
    return {
        "q": views["q"].view(torch.bfloat16).view(B, H, 192),
        "qabs": views["qabs"].view(torch.bfloat16).view(B, H, 576),
        "olat": views["olat"].view(torch.bfloat16).view(B, H, 512),
        "ov": views["ov"].view(torch.bfloat16).view(B, H * 128),
        "xo": views["xo"].view(torch.float8_e4m3fn).view(B, H * 128),
        "so": views["so"].view(torch.float32).view(B, H),
    }


def test_mla_decode_layer_128_heads_stagewise():
    """Each stage of the 128-head layer against the oracle fed with the GPU's
    previous-stage output (a bf16 ulp upstream can flip an FP8 code of o_v,
    so stages are compared one at a time)."""
    cfg = MLAConfig(n_heads=128)
    layer = MLADecodeLayer(cfg, "cuda")
    wq, wqs, wkv, wkvs, wo, wos = [t.cpu() for t in layer.random_weights(seed=3)]
    B, ctx = 2, 640
    cache, table, _ = make_paged_cache(B, ctx, 64, 576, "cuda", seed=4)
    seqlens = torch.tensor([640, 300], device="cuda", dtype=torch.int32)
    positions = seqlens.clone()
    freqs = precompute_freqs_cis(64, 1024, cfg.rope_theta, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(6)
    q_lora = torch.randn(B, cfg.dc, device="cuda", generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    y = layer.forward(q_lora, cache, table, seqlens, positions, freqs, ctx)
    assert _lib.device_error() == 0
    v = _mla_ws_views(layer, B)
    H = 128
    # q-up + RoPE
    xq, xs = O.act_quant(n_bf16(q_lora), 128, False)
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, n_u8(wq), wqs.numpy())).reshape(B, 1, H, 192)
    fr = freqs.cpu().numpy()
    q = np.stack([O.rope(q[b:b + 1], fr, 64, int(positions[b])) for b in range(B)])[:, 0, 0]
    assert_close_attn(f32(n_bf16(v["q"])), f32(q), "q-up + rope")
    # absorb from the GPU's q
    wkv_bf16 = O.f32_to_bf16(O.e4m3_to_f32(n_u8(wkv)) *
                             np.repeat(np.repeat(wkvs.numpy(), 128, 0), 128, 1))
    qg = n_bf16(v["q"])
    q_abs = np.concatenate([O.mla_absorb(qg, wkv_bf16, 128, 128), qg[..., 128:]], axis=-1)
    assert_close_attn(f32(n_bf16(v["qabs"])), f32(q_abs), "absorb")
    # attention from the GPU's q_abs (two-CTA tcgen05 kernel)
    o_lat = O.paged_decode_attn(n_bf16(v["qabs"]), n_bf16(cache), table.cpu().numpy(),
                                seqlens.cpu().numpy(), None, cfg.softmax_scale, 512)
    assert_close_attn(f32(n_bf16(v["olat"])), f32(O.f32_to_bf16(o_lat)), "attention")
    # v-up from the GPU's o_lat
    o_v = O.mla_vup(n_bf16(v["olat"]), wkv_bf16, 128, 128).reshape(B, H * 128)
    assert_close_attn(f32(n_bf16(v["ov"])), f32(o_v), "v-up")
    # act_quant of the GPU's o_v is bit-exact; o-proj from those codes
    xo, so = O.act_quant(n_bf16(v["ov"]), 128, False)
    assert np.array_equal(n_u8(v["xo"]), xo)
    assert np.array_equal(v["so"].cpu().numpy(), so)
    ref = O.f32_to_bf16(O.fp8_gemm(xo, so, n_u8(wo), wos.numpy()))
    assert_close_attn(f32(n_bf16(y)), f32(ref), "o-proj")


@pytest.mark.parametrize("round_scale", [False, True])
def test_mla_vup_fused_act_quant_bit_exact(round_scale):
    """The v-up's epilogue quantises its own bf16 output (1 x 128 blocks, one
    head's d_v values a block): codes and scales are bit for bit the
    reference act_quant of the o_v it wrote, with fp32 and UE8M0 scales."""
    import dataclasses
    cfg = dataclasses.replace(MLAConfig(n_heads=16), act_round_scale=round_scale)
    layer = MLADecodeLayer(cfg, "cuda")
    layer.random_weights(seed=9, e8m0=round_scale)
    B, ctx = 70, 256
    cache, table, seqlens = make_paged_cache(B, ctx, 64, 576, "cuda", seed=10)
    freqs = precompute_freqs_cis(64, 512, cfg.rope_theta, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(11)
    q_lora = torch.randn(B, cfg.dc, device="cuda", generator=gen).to(torch.bfloat16)
    layer.forward(q_lora, cache, table, seqlens, seqlens.clone(), freqs, ctx)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    v = _mla_ws_views(layer, B)
    H = layer.n_local
    xo, so = O.act_quant(n_bf16(v["ov"]), 128, round_scale)
    assert np.array_equal(n_u8(v["xo"]), xo)
    if round_scale:
        got = layer._ws[_ws_offset(layer, B, "so"):][:B * H].cpu().numpy().reshape(B, H)
        assert np.array_equal(np.ldexp(1.0, got.astype(np.int32) - 127).astype(np.float32), so)
    else:
        assert np.array_equal(v["so"].cpu().numpy(), so)


def _ws_offset(layer, B, name):
    """Byte offset of one intermediate in the decode layer's workspace."""
    H, c = layer.n_local, layer.cfg
    al = lambda n: (n + 255) // 256 * 256
    sizes = [("xq", B * c.dc), ("sq", B * (c.dc // 128) * 4), ("q", B * H * 192 * 2),
             ("qabs", B * H * 576 * 2), ("olat", B * H * 512 * 2), ("ov", B * H * 128 * 2),
             ("xo", B * H * 128), ("so", B * H * 4)]
    off = 0
    for n_, sz in sizes:
        if n_ == name:
            return off
        off += al(sz)
    raise KeyError(name)
