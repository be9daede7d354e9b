"""Pins the CPU oracle to the reference before it is trusted as the checker.

* act_quant: bit-exact against all 36 reference golden cases (TileLang GPU
  output of linear() -> act_quant(c_q, 128, "ue8m0")) and against the
  reference's PyTorch path (kernel_fallback.act_quant) in fp32-scale, UE8M0 and
  in-place block-64 modes.
* fp8_gemm, attention, RoPE and the whole V4 QCAU chain: against the
  reference's PyTorch path on seeded inputs and against the 36 golden
  attention outputs, within one bf16 ulp / cosine >= 0.9999.
* the attention core against the reference's own qcau_c C++ build.
"""
import numpy as np
import pytest

import oracle as O


def _cos(a, b):
    a = a.ravel().astype(np.float64)
    b = b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def test_act_quant_matches_36_goldens_bitwise(golden_dir):
    g = np.load(golden_dir / "act_quant_goldens.npz")
    assert len(g["cases"]) == 36
    for c in g["cases"]:
        y, s = O.act_quant(g[f"{c}/c_q"], 128, True)
        assert np.array_equal(y, g[f"{c}/x"]), c
        assert np.array_equal(O.f32_pow2_to_e8m0(s), g[f"{c}/s"]), c


def test_act_quant_matches_reference_pytorch_bitwise(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    x = g["aq/x"]
    y, s = O.act_quant(x, 128, False)
    assert np.array_equal(y, g["aq/y_f32"])
    assert np.array_equal(s.view(np.uint32), g["aq/s_f32"].view(np.uint32))
    y, s = O.act_quant(x, 128, True)
    assert np.array_equal(y, g["aq/y_ue8m0"])
    assert np.array_equal(O.f32_pow2_to_e8m0(s), g["aq/s_ue8m0"])
    ip = O.act_quant_inplace(x[:, :448], 64, True)
    assert np.array_equal(ip, g["aq/inplace64"])


def test_fp8_gemm_matches_reference_pytorch(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    c = O.fp8_gemm(g["gemm/a"], g["gemm/sa"], g["gemm/b"], g["gemm/sb"])
    ref = O.bf16_to_f32(g["gemm/c_bf16"])
    got = O.bf16_to_f32(O.f32_to_bf16(c))
    # fp32 summation order differs; the bf16 results agree to one ulp
    assert np.mean(got == ref) > 0.999
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2 ** -7 + 1e-6)


def test_attention_matches_reference_pytorch(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    o = O.sparse_attn(g["attn/q"], g["attn/kv"], g["attn/sink"], g["attn/idx"],
                      float(g["attn/scale"]))
    got = O.bf16_to_f32(O.f32_to_bf16(o))
    ref = O.bf16_to_f32(g["attn/o"])
    assert np.mean(got == ref) > 0.995
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2 ** -7 + 1e-3)


def test_attention_and_inverse_rope_match_36_goldens(golden_dir):
    g = np.load(golden_dir / "attn_goldens.npz")
    for c in g["cases"]:
        o = O.sparse_attn(g[f"{c}/q"], g[f"{c}/kv"], g[f"{c}/sink"], g[f"{c}/idx"],
                          float(g[f"{c}/scale"]))
        ob = O.f32_to_bf16(o)
        tail = O.bf16_to_f32(ob[..., -64:])
        ref_tail = O.bf16_to_f32(g[f"{c}/sparse_o_tail"])
        assert np.abs(tail - ref_tail).max() <= 2 ** -7 * max(1.0, np.abs(ref_tail).max()), c
        out = O.bf16_to_f32(O.rope(ob, g[f"{c}/freqs"], 64, 0, inverse=True))
        ref = O.bf16_to_f32(g[f"{c}/qcau_o"])
        rms = float(np.sqrt(np.mean(ref ** 2)))
        assert _cos(out, ref) >= 0.9999, c
        assert np.abs(out - ref).max() <= 2e-2 * rms, c


def test_inverse_rope_matches_goldens(golden_dir):
    """qcau_o = inverse RoPE of the bf16 sparse_o (QCAU.py:313-319)."""
    g = np.load(golden_dir / "attn_goldens.npz")
    exact = total = 0
    for c in g["cases"]:
        tail = g[f"{c}/sparse_o_tail"]
        ref = g[f"{c}/qcau_o"][..., -64:]
        got = O.rope(tail, g[f"{c}/freqs"], 64, 0, inverse=True)
        exact += int(np.sum(got == ref))
        total += got.size
        assert np.abs(O.bf16_to_f32(got) - O.bf16_to_f32(ref)).max() <= 2 ** -6, c
    # the reference's freqs are decimal text, so a few values differ by an ulp
    assert exact / total > 0.99


def test_qcau_chain_matches_reference_pytorch(golden_dir):
    g = np.load(golden_dir / "ref_synthetic.npz")
    cq = g["qcau/c_q"][0]
    S = cq.shape[0]
    xq, xs = O.act_quant(cq, 128, True)
    ws = O.e8m0_to_f32(g["qcau/w_scale_e8m0"])
    q = O.f32_to_bf16(O.fp8_gemm(xq, xs, g["qcau/w"], ws))
    H = g["qcau/sink"].shape[0]
    q = q.reshape(1, S, H, 512)
    q = O.head_rms_norm(q, 1e-6)
    q = O.rope(q, g["qcau/freqs"], 64, 0)
    o = O.f32_to_bf16(O.sparse_attn(q, g["qcau/kv"], g["qcau/sink"], g["qcau/idx"], 512 ** -0.5))
    o = O.rope(o, g["qcau/freqs"], 64, 0, inverse=True)
    got = O.bf16_to_f32(o)
    ref = O.bf16_to_f32(g["qcau/o"])
    assert _cos(got, ref) >= 0.9999
    assert np.abs(got - ref).max() <= 2e-2 * float(np.sqrt(np.mean(ref ** 2)))


@pytest.mark.skipif(not O.ref_available(), reason="qcau_c reference build missing")
def test_attention_matches_reference_cpp(golden_dir):
    """Oracle vs the reference's own C++ port (qcau.cpp sparse_attention)."""
    g = np.load(golden_dir / "attn_goldens.npz")
    c = "hardware_seq4_layer2"
    q = g[f"{c}/q"][0]
    kv = g[f"{c}/kv"][0]
    idx = g[f"{c}/idx"][0]
    sink = g[f"{c}/sink"]
    ref = O.bf16_to_f32(O.ref_sparse_attention(q, kv, idx, sink))
    got = O.bf16_to_f32(O.f32_to_bf16(O.sparse_attn(q[None], kv[None], sink, idx[None],
                                                    512 ** -0.5)))[0]
    assert _cos(got, ref) >= 0.9999
    assert np.abs(got - ref).max() <= 2e-2 * float(np.sqrt(np.mean(ref ** 2)))
