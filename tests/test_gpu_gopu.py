"""GPU parity of the V4 output side (qcau_gopu via qcau_b200.gopu.GOPU):
the grouped wo_a projection on the tcgen05 batched GEMM, act_quant and the
FP8 wo_b GEMM, against the reference's own output (tests/golden/gopu.npz)
and stage by stage against the oracle fed with the GPU's previous stage."""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from helpers import assert_close_attn, f32, n_bf16, n_u8, t_bf16, t_u8

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200.gopu import GOPU

GOLDEN = Path(__file__).resolve().parent / "golden"
B, S, H, D, G, R, DIM = 2, 3, 8, 512, 2, 128, 256


def _gopu(f):
    m = GOPU(n_heads=H, head_dim=D, n_groups=G, o_lora_rank=R, dim=DIM, device="cuda")
    m.load_weights(t_bf16(f["wo_a"]), t_u8(f["wo_b"]), t_u8(f["wo_b_scale"], torch.float8_e8m0fnu))
    return m


def test_gopu_vs_reference_and_stages():
    f = np.load(GOLDEN / "gopu.npz")
    m = _gopu(f)
    y = m.forward(t_bf16(f["o"]))
    assert y.shape == (B, S, DIM)
    assert _lib.device_error() == 0
    assert_close_attn(f32(n_bf16(y)), f32(f["y"]), "gopu vs reference")
    # stages: the workspace holds h [rows, G, R] bf16, then its codes and scales
    rows = B * S
    h = m._ws[:rows * G * R * 2].view(torch.bfloat16).view(rows, G, R)
    hg = n_bf16(h)
    assert_close_attn(f32(hg), f32(f["h"].reshape(rows, G, R)), "wo_a")
    off = (rows * G * R * 2 + 255) // 256 * 256
    codes = m._ws[off:off + rows * G * R].view(rows, G * R)
    xq, xs = O.act_quant(hg.reshape(rows, G * R), 128, True)
    assert np.array_equal(n_u8(codes), xq)
    ref = O.f32_to_bf16(O.fp8_gemm(xq, xs, f["wo_b"], O.e8m0_to_f32(f["wo_b_scale"])))
    assert_close_attn(f32(n_bf16(y)).reshape(rows, DIM), f32(ref), "wo_b")


def test_gopu_v4_flash_widths_vs_oracle():
    """The model's widths: 64 heads of 512 in 8 groups, o_lora_rank 1024,
    dim 4096 (V4-Flash config), 4 tokens."""
    gen = torch.Generator(device="cuda").manual_seed(9)
    Hh, Gg, Rr, Dm, rows = 64, 8, 1024, 4096, 4
    o = torch.randn(rows, Hh, 512, device="cuda", generator=gen).to(torch.bfloat16)
    wo_a = (torch.randn(Gg * Rr, Hh * 512 // Gg, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    from qcau_b200.mla import quantize_weight_fp8
    wb, wbs = quantize_weight_fp8(torch.randn(Dm, Gg * Rr, device="cuda", generator=gen) * 0.02, True)
    m = GOPU(device="cuda")
    m.load_weights(wo_a, wb, wbs)
    y = m.forward(o)
    assert _lib.device_error() == 0
    h = O.grouped_proj(n_bf16(o).reshape(rows, Gg, -1), n_bf16(wo_a).reshape(Gg, Rr, -1))
    hg = n_bf16(m._ws[:rows * Gg * Rr * 2].view(torch.bfloat16).view(rows, Gg, Rr))
    assert_close_attn(f32(hg), f32(h), "wo_a v4 widths")
    xq, xs = O.act_quant(hg.reshape(rows, Gg * Rr), 128, True)
    ref = O.f32_to_bf16(O.fp8_gemm(xq, xs, n_u8(wb), O.e8m0_to_f32(n_u8(wbs))))
    assert_close_attn(f32(n_bf16(y)), f32(ref), "wo_b v4 widths")
