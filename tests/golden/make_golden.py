"""Generate the committed golden fixtures under tests/golden/.

Run where the reference checkout is readable; its root is taken from
QCAU_REFERENCE_ROOT, else a directory named `reference` beside this
repository's parent:

    QCAU_REFERENCE_ROOT=<reference root> python tests/golden/make_golden.py

Outputs (compressed .npz, raw bit patterns: bf16 as uint16, fp8/e8m0 as uint8):

* act_quant_goldens.npz -- all 36 reference golden cases
  (QCAU/QCAU_inference/framework/test_vectors/*): c_q and the FP8 codes / E8M0
  scales that linear() -> act_quant(c_q, 128, "ue8m0") produced on the GPU
  (model.py:117; the TileLang kernel kernel.py:40-102).
* attn_goldens.npz -- the same 36 cases' attention inputs (q after query-up,
  kv, topk_idxs, attn_sink, freqs_cis) and TileLang outputs
  (qcau_o_after_inverse_rope, and the rope tail of sparse_o_before_inverse_rope).
  To keep the fixture small, sequence-length-4 cases keep 16 of the 64 heads
  and sequence-length-16 cases keep 4 (heads are independent in the MQA core,
  kernel.py:301-343, so a head subset is an exact sub-problem); length-1 cases
  keep all 64.
* kv_build.npz -- the reference's KV build (model.py RMSNorm, RoPE with the
  YaRN freqs of a compressed layer, kernel_fallback.act_quant in place, block
  64, UE8M0) on seeded rows.
* indexer.npz -- the index-list producers (window / compressed lists, the
  Hadamard rotation, and Indexer.forward of a small seeded indexer) run by
  the QCAU package's model.py on kernel_fallback.
* attention_trace.npz -- every call the reference's Attention.forward
  (Deepseek_origin/inference/model.py) makes into its `kernel` module, with
  arguments as passed and results, on a small seeded V4-width layer run with
  kernel_fallback as that module.
* compressor.npz -- the reference's Compressor (gated pooling, norm, RoPE,
  FP8 or Hadamard) over prefill and decode steps, with its projections,
  outputs, cache and state.
* gopu.npz -- the reference's output side (the wo_a einsum and wo_b through
  linear() on kernel_fallback's FP8 kernels) on seeded tensors.
* ref_synthetic.npz -- seeded synthetic inputs run through the reference's
  own PyTorch CPU path, imported here by file path:
  kernel_fallback.act_quant / fp8_gemm (QCAU/QCAU_inference/inference/
  kernel_fallback.py:48-113) and check/QCAU.py (_sparse_attention_online with
  prob_dtype=bf16, and the whole QCAU() with a callable FP8 Linear).
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

REF = Path(os.environ.get("QCAU_REFERENCE_ROOT") or
           Path(__file__).resolve().parents[3] / "reference")
FW = REF / "QCAU/QCAU_inference/framework"
VEC = FW / "test_vectors"
INF = REF / "QCAU/QCAU_inference/inference"
OUT = Path(__file__).resolve().parent


def load_module(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "deepseek-v4-flash_b200"))
from qcau_b200.golden_io import read_shape, read_tensor  # noqa: E402  (the library's reader)


def read_hex(case: Path, fname: str, dtype) -> np.ndarray:
    return read_tensor(case, fname.split(".")[0]).ravel().astype(dtype)


def read_text(case: Path, fname: str, dtype) -> np.ndarray:
    return read_tensor(case, fname.split(".")[0]).ravel().astype(dtype)


def head_subset(seq: int, n_heads: int) -> np.ndarray:
    if seq == 1:
        return np.arange(n_heads)
    if seq == 4:
        return np.arange(0, n_heads, n_heads // 16)
    return np.arange(0, n_heads, n_heads // 4)


def goldens():
    manifest = json.loads((FW / "manifest.json").read_text())
    cases = manifest["cases"]
    aq = {}
    at = {}
    for name in cases:
        case = VEC / name
        meta = json.loads((case / "metadata.json").read_text())
        S = meta["seq_len"]
        H = meta["n_local_heads"]
        D = meta["head_dim"]
        cq = read_hex(case, "c_q.bf16_hex.txt", np.uint16).reshape(read_shape(case, "c_q"))
        x = read_hex(case, "linear_x_after_act_quant.fp8_e4m3_hex.txt", np.uint8)
        s = read_hex(case, "linear_s_after_act_quant.e8m0_hex.txt", np.uint8)
        aq[f"{name}/c_q"] = cq.reshape(S, -1)
        aq[f"{name}/x"] = x.reshape(S, -1)
        aq[f"{name}/s"] = s.reshape(S, -1)

        hs = head_subset(S, H)
        q = read_hex(case, "q_after_query_up_rope.bf16_hex.txt", np.uint16).reshape(1, S, H, D)
        kv_shape = read_shape(case, "kv_after_rope_quant_compress")
        kv = read_hex(case, "kv_after_rope_quant_compress.bf16_hex.txt", np.uint16).reshape(kv_shape)
        idx = np.loadtxt(case / "topk_idxs.int.txt", dtype=np.int64).astype(np.int32)
        idx = idx.reshape(read_shape(case, "topk_idxs"))
        sink = read_text(case, "attn_sink.fp32.txt", np.float32)
        fr = read_text(case, "freqs_cis_real.fp32.txt", np.float32).reshape(S, -1)
        fi = read_text(case, "freqs_cis_imag.fp32.txt", np.float32).reshape(S, -1)
        o = read_hex(case, "qcau_o_after_inverse_rope.bf16_hex.txt", np.uint16).reshape(1, S, H, D)
        so = read_hex(case, "sparse_o_before_inverse_rope.bf16_hex.txt", np.uint16).reshape(1, S, H, D)
        at[f"{name}/heads"] = hs.astype(np.int32)
        at[f"{name}/q"] = np.ascontiguousarray(q[:, :, hs])
        at[f"{name}/kv"] = kv
        at[f"{name}/idx"] = idx
        at[f"{name}/sink"] = sink[hs]
        at[f"{name}/freqs"] = np.stack([fr, fi], axis=-1).astype(np.float32)
        at[f"{name}/qcau_o"] = np.ascontiguousarray(o[:, :, hs])
        at[f"{name}/sparse_o_tail"] = np.ascontiguousarray(so[:, :, hs, D - 64:])
        at[f"{name}/scale"] = np.float32(meta["softmax_scale"])
    aq["cases"] = np.asarray(cases)
    at["cases"] = np.asarray(cases)
    np.savez_compressed(OUT / "act_quant_goldens.npz", **aq)
    np.savez_compressed(OUT / "attn_goldens.npz", **at)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy()


def synthetic():
    fb = load_module("ref_kernel_fallback", INF / "kernel_fallback.py")
    cq_mod = load_module("ref_check_qcau", INF / "check" / "QCAU.py")
    g = torch.Generator().manual_seed(0)
    out = {}

    # act_quant: fp32 scales (scale_fmt=None), UE8M0 scales, and the in-place
    # block-64 UE8M0 round trip used on the KV rows (model.py:506).
    x = (torch.randn(64, 1536, generator=g) * torch.logspace(-3, 2, 64).unsqueeze(1)).bfloat16()
    x[3, 128:256] = 0  # all-zero block -> amax floor 1e-4
    y32, s32 = fb.act_quant(x, 128, None, torch.float32)
    y8, s8 = fb.act_quant(x, 128, "ue8m0", torch.float8_e8m0fnu)
    kvx = x[:, :448].clone()
    fb.act_quant(kvx, 64, "ue8m0", torch.float8_e8m0fnu, inplace=True)
    out["aq/x"] = u16(x)
    out["aq/y_f32"] = u8(y32)
    out["aq/s_f32"] = s32.numpy()
    out["aq/y_ue8m0"] = u8(y8)
    out["aq/s_ue8m0"] = u8(s8)
    out["aq/inplace64"] = u16(kvx)

    # fp8_gemm with fp32 block scales, output in the model's default dtype bf16
    torch.set_default_dtype(torch.bfloat16)
    try:
        a = (torch.randn(32, 1536, generator=g) * 3).bfloat16()
        aq_, as_ = fb.act_quant(a, 128, None, torch.float32)
        w = torch.randn(384, 1536, generator=g) * 0.02
        # weight scales are per 128x128 block
        wblk = w.view(3, 128, 12, 128).abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0
        wq_ = (w.view(3, 128, 12, 128) / wblk[:, None, :, None]).clamp(-448, 448).view(384, 1536)
        wq_ = wq_.to(torch.float8_e4m3fn)
        c = fb.fp8_gemm(aq_, as_, wq_, wblk.float())
        out["gemm/a"] = u8(aq_)
        out["gemm/sa"] = as_.numpy()
        out["gemm/b"] = u8(wq_)
        out["gemm/sb"] = wblk.float().numpy()
        out["gemm/c_bf16"] = u16(c)
    finally:
        torch.set_default_dtype(torch.float32)

    # attention core (bf16 P), V4 widths, with -1 holes, an all-invalid tile
    # and an out-of-range index
    B, S, H, D, N, K = 1, 3, 16, 512, 300, 200
    q = torch.randn(B, S, H, D, generator=g).bfloat16()
    kv = torch.randn(B, N, D, generator=g).bfloat16()
    idx = torch.randint(0, N, (B, S, K), generator=g, dtype=torch.int64)
    idx[:, :, 5::7] = -1
    idx[:, 1, 64:128] = -1
    idx[:, 2, 0] = N + 5
    sink = torch.randn(H, generator=g)
    scale = D ** -0.5
    o = cq_mod._sparse_attention_online(q, kv, sink, idx, scale, 64, torch.bfloat16)
    out["attn/q"] = u16(q)
    out["attn/kv"] = u16(kv)
    out["attn/idx"] = idx.int().numpy()
    out["attn/sink"] = sink.numpy()
    out["attn/scale"] = np.float32(scale)
    out["attn/o"] = u16(o)

    # whole QCAU (V4 mode) with a callable FP8 projector: act_quant(ue8m0) ->
    # fp8_gemm, per-head RMSNorm (bf16), RoPE, attention, inverse RoPE
    Dc, H2, S2, N2, K2 = 1024, 2, 2, 96, 80
    c_q = torch.randn(1, S2, Dc, generator=g).bfloat16()
    w2 = torch.randn(H2 * D, Dc, generator=g) * 0.02
    blk = w2.view(H2 * D // 128, 128, Dc // 128, 128).abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0
    blk = torch.exp2(torch.ceil(torch.log2(blk)))
    w2q = (w2.view(H2 * D // 128, 128, Dc // 128, 128) / blk[:, None, :, None]).clamp(-448, 448)
    w2q = w2q.view(H2 * D, Dc).to(torch.float8_e4m3fn)

    def projector(x):
        xq, xs = fb.act_quant(x, 128, "ue8m0", torch.float8_e8m0fnu)
        return fb.fp8_gemm(xq, xs, w2q, blk.to(torch.float8_e8m0fnu), torch.float8_e8m0fnu)

    kv2 = torch.randn(1, N2, D, generator=g).bfloat16()
    idx2 = torch.randint(0, N2, (1, S2, K2), generator=g, dtype=torch.int64)
    idx2[:, :, 3::5] = -1
    sink2 = torch.randn(H2, generator=g)
    ang = torch.randn(S2, 32, generator=g)
    freqs = torch.polar(torch.ones_like(ang), ang)
    torch.set_default_dtype(torch.bfloat16)
    try:
        o2 = cq_mod.QCAU(c_q=c_q, w_uq=projector, kv=kv2, topk_idxs=idx2, attn_sink=sink2,
                         freqs_cis=freqs, n_local_heads=H2, head_dim=D, rope_head_dim=64,
                         prob_dtype=torch.bfloat16)
    finally:
        torch.set_default_dtype(torch.float32)
    out["qcau/c_q"] = u16(c_q)
    out["qcau/w"] = u8(w2q)
    out["qcau/w_scale_e8m0"] = u8(blk.to(torch.float8_e8m0fnu))
    out["qcau/kv"] = u16(kv2)
    out["qcau/idx"] = idx2.int().numpy()
    out["qcau/sink"] = sink2.numpy()
    out["qcau/freqs"] = torch.view_as_real(freqs).numpy().astype(np.float32)
    out["qcau/o"] = u16(o2)
    np.savez_compressed(OUT / "ref_synthetic.npz", **out)


def kv_build_fixture():
    """kv_build.npz: the reference's KV build (Deepseek_origin/inference/
    model.py:502-505) run by its own code on seeded rows: RMSNorm
    (model.py:182-195), apply_rotary_emb of the last 64 values (:231-243) with
    the YaRN freqs_cis of a compressed layer (precompute_freqs_cis :198-228),
    then kernel_fallback.act_quant(kv[..., :-64], 64, "ue8m0", inplace=True)
    (the QCAU package's CPU kernels standing in for kernel.py)."""
    kf = load_module("kernel_fallback_kv", INF / "kernel_fallback.py")
    sys.modules["kernel"] = kf
    model = load_module("ref_model_v4", REF / "Deepseek_origin/inference/model.py")
    g = torch.Generator().manual_seed(11)
    rows, d, rd = 96, 512, 64
    x = (torch.randn(rows, d, generator=g) * 3.0).to(torch.bfloat16)
    w = 1.0 + 0.1 * torch.randn(d, generator=g)
    pos = torch.randint(0, 8192, (rows,), generator=g)
    freqs = model.precompute_freqs_cis(rd, 8192, 65536, 160000.0, 16.0, 32, 1)
    # the table rows the positions use, so the fixture stays small: row r of
    # "freqs" is freqs_cis[positions[r]] (the kernel reads it at position r)
    out = {"x": u16(x), "weight": w.numpy().astype(np.float32),
           "positions": pos.numpy().astype(np.int32),
           "freqs": torch.view_as_real(freqs[pos]).numpy().astype(np.float32)}
    norm = model.RMSNorm(d, 1e-6)
    with torch.no_grad():
        norm.weight.copy_(w)
        kv = norm(x.unsqueeze(0))                         # [1, rows, 512] bf16
        model.apply_rotary_emb(kv[..., -rd:], freqs[pos])
        out["after_norm_rope"] = u16(kv[0].clone())
        kf.act_quant(kv[..., :-rd], 64, "ue8m0", torch.float8_e8m0fnu, True)
    out["kv"] = u16(kv[0])
    np.savez_compressed(OUT / "kv_build.npz", **out)


def gopu_fixture():
    """gopu.npz: the reference's output side (model.py:536-542) run by its own
    code on seeded tensors at reduced widths (8 heads of 512 in 2 groups,
    o_lora_rank 128, dim 256): the bf16 einsum with wo_a, then wo_b through
    linear() (model.py:108-120) on kernel_fallback's act_quant / fp8_gemm with
    UE8M0 scales."""
    kf = load_module("kernel_fallback_gopu", INF / "kernel_fallback.py")
    sys.modules["kernel"] = kf
    model = load_module("ref_model_v4_gopu", REF / "Deepseek_origin/inference/model.py")
    model.scale_fmt, model.scale_dtype = "ue8m0", torch.float8_e8m0fnu
    g = torch.Generator().manual_seed(13)
    B, S, H, D, G, R, dim = 2, 3, 8, 512, 2, 128, 256
    o = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    wo_a = (torch.randn(G * R, H * D // G, generator=g) * 0.02).to(torch.bfloat16)
    w = torch.randn(dim, G * R, generator=g) * 0.02
    blk = w.view(dim // 128, 128, G * R // 128, 128)
    sc = torch.exp2(torch.ceil(torch.log2(blk.abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0)))
    wq = (blk / sc[:, None, :, None]).clamp(-448, 448).view(dim, G * R).to(torch.float8_e4m3fn)
    wq.scale = sc.to(torch.float8_e8m0fnu)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)  # the model's (generate.py), fp8_gemm's out dtype
    try:
        with torch.no_grad():
            h = torch.einsum("bsgd,grd->bsgr", o.view(B, S, G, -1), wo_a.view(G, R, -1))
            y = model.linear(h.flatten(2), wq)
    finally:
        torch.set_default_dtype(prev)
    out = {"o": u16(o), "wo_a": u16(wo_a), "wo_b": wq.view(torch.uint8).numpy(),
           "wo_b_scale": wq.scale.view(torch.uint8).numpy(), "h": u16(h), "y": u16(y)}
    np.savez_compressed(OUT / "gopu.npz", **out)


def load_qcau_inference_model():
    """QCAU/QCAU_inference/inference/model.py imported as a package module
    whose `.kernel` is kernel_fallback.py (the TileLang kernels need a GPU);
    its rotate_activation then runs its own fp32 Hadamard restatement, since
    fast_hadamard_transform is not installed."""
    import types

    name = "qcau_ref_inference"
    if f"{name}.model" in sys.modules:
        return sys.modules[f"{name}.model"]
    pkg = types.ModuleType(name)
    pkg.__path__ = [str(INF)]
    sys.modules[name] = pkg

    def load(sub):
        spec = importlib.util.spec_from_file_location(f"{name}.{sub}", INF / f"{sub}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        return mod

    sys.modules[f"{name}.kernel"] = load("kernel_fallback")
    return load("model")


def indexer_fixture():
    """indexer.npz: the index-list producers run by the reference's own code
    (QCAU/QCAU_inference/inference/model.py):

    * lists/<i>: get_window_topk_idxs and get_compress_topk_idxs concatenated
      as Attention.forward does (model.py:614-624), for the (window, ratio,
      bsz, seqlen, start_pos, offset) of list_params[i];
    * rot_x / rot_y: rotate_activation on seeded rows (its fp32 restatement);
    * step<i>/...: Indexer.forward (model.py:500-534) of a seeded small
      indexer (8 heads of 128, index_topk 8, ratio 4, bf16 projections) over
      a 64-token prefill of 2 sequences and 4 decode steps: the queries before
      rotation (q_pre) and as the einsum reads them (q), the compressed keys
      (kv = kv_cache[:b, :end_pos // 4]), the head weights (w), the masked
      score rows (score, recomputed from those tensors by the same expressions)
      and the returned topk_idxs (idx).  kernel_fallback's fp4_act_quant does
      not round to FP4, so q equals rotate_activation(q_pre) here."""
    model = load_qcau_inference_model()
    out = {}
    params = []
    cases = [(8, 4, 2, 5, 0, 5), (8, 4, 2, 21, 0, 21), (128, 4, 1, 300, 0, 300),
             (128, 128, 2, 300, 0, 300), (128, 0, 2, 130, 0, 0), (8, 4, 3, 1, 3, 8),
             (8, 4, 3, 1, 7, 8), (8, 4, 3, 1, 8, 8), (8, 4, 2, 1, 22, 8),
             (128, 4, 2, 1, 131, 128), (128, 128, 2, 1, 1000, 128), (128, 128, 2, 1, 127, 128),
             (128, 4, 1, 1, 126, 128), (128, 0, 2, 1, 200, 128)]
    for i, (win, ratio, bsz, seqlen, sp, off) in enumerate(cases):
        w = model.get_window_topk_idxs(win, bsz, seqlen, sp)
        if ratio:
            c = model.get_compress_topk_idxs(ratio, bsz, seqlen, sp, off)
            w = torch.cat([w, c], dim=-1)
        out[f"lists/{i}"] = w.int().numpy()
        params.append((win, ratio, bsz, seqlen, sp, off))
    out["list_params"] = np.array(params, dtype=np.int64)

    g = torch.Generator().manual_seed(17)
    x = (torch.randn(64, 128, generator=g) * 2).to(torch.bfloat16)
    out["rot_x"] = u16(x)
    out["rot_y"] = u16(model.rotate_activation(x))

    args = model.ModelArgs(max_batch_size=2, max_seq_len=256, dim=256, q_lora_rank=128,
                           index_n_heads=8, index_head_dim=128, index_topk=8)
    torch.manual_seed(19)
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)  # the model's (generate.py): bf16 kv_cache buffers
    idx = model.Indexer(args, 4)
    with torch.no_grad():
        for n, p in idx.named_parameters():
            if n.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            elif n.endswith("ape"):
                p.copy_(0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_((torch.randn(p.shape, generator=g) / p.shape[-1] ** 0.5).to(p.dtype))
    idx.freqs_cis = model.precompute_freqs_cis(64, 256, 0, 10000.0, 40, 32, 1)
    rec = {}
    real_rot, real_fp4 = model.rotate_activation, model.fp4_act_quant

    def rot(t):
        y = real_rot(t)
        if t.dim() == 4:
            rec["q_pre"] = t.clone()
        return y

    def fp4(t, block, inplace=False):
        y = real_fp4(t, block, inplace)
        if t.dim() == 4:
            rec["q"] = t.clone()
        return y

    model.rotate_activation, model.fp4_act_quant = rot, fp4
    idx.weights_proj.register_forward_hook(lambda m, a, o: rec.__setitem__("w_proj", o.clone()))
    try:
        B, S = 2, 64
        steps = [(0, S)] + [(S + i, 1) for i in range(4)]
        for i, (sp, sl) in enumerate(steps):
            x = torch.randn(B, sl, 256, generator=g).to(torch.bfloat16)
            qr = torch.randn(B, sl, 128, generator=g).to(torch.bfloat16)
            offset = sl if sp == 0 else 128  # Attention.forward: kv.size(1) at prefill, else win
            with torch.no_grad():
                topk_idxs = idx(x, qr, sp, offset)
                end = sp + sl
                kv = idx.kv_cache[:B, :end // 4]
                w = rec["w_proj"] * (idx.softmax_scale * idx.n_heads ** -0.5)
                sc = torch.einsum("bshd,btd->bsht", rec["q"], kv)
                sc = (sc.relu_() * w.unsqueeze(-1)).sum(dim=2)
                if sp == 0:
                    mask = torch.arange(sl // 4).repeat(sl, 1) >= torch.arange(1, sl + 1).unsqueeze(1) // 4
                    sc += torch.where(mask, float("-inf"), 0)
            out[f"step{i}/meta"] = np.array([sp, sl, offset], dtype=np.int64)
            out[f"step{i}/q_pre"] = u16(rec["q_pre"])
            out[f"step{i}/q"] = u16(rec["q"])
            out[f"step{i}/kv"] = u16(kv.contiguous())
            out[f"step{i}/w"] = u16(w)
            out[f"step{i}/score"] = sc.float().numpy()
            out[f"step{i}/idx"] = topk_idxs.int().numpy()
    finally:
        model.rotate_activation, model.fp4_act_quant = real_rot, real_fp4
        torch.set_default_dtype(prev_dtype)
    np.savez_compressed(OUT / "indexer.npz", **out)


_TRACE_DTYPES = {torch.bfloat16: "bf16", torch.float32: "fp32", torch.float8_e4m3fn: "e4m3",
                 torch.float8_e8m0fnu: "e8m0", torch.int32: "int32", torch.int64: "int64"}


class _TraceWriter:
    """Records the calls a reference module makes into its `kernel` module:
    every tensor argument as its base tensor's bits plus the view (size,
    stride, offset) the call saw, the results, and for in-place calls the base
    tensor after the call.  Identical arrays (the weights, read every step)
    are stored once."""

    def __init__(self):
        self.arrays, self.calls, self._by_hash = {}, [], {}

    def _store(self, t: torch.Tensor) -> str:
        raw = t.detach().contiguous().view(-1)
        if t.dtype in (torch.bfloat16,):
            a = raw.view(torch.int16).numpy().view(np.uint16)
        elif t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu):
            a = raw.view(torch.uint8).numpy()
        else:
            a = raw.numpy()
        key = (a.dtype.str, a.tobytes())
        h = hash(key)
        if h not in self._by_hash:
            name = f"a{len(self.arrays)}"
            self.arrays[name] = a.copy()
            self._by_hash[h] = name
        return self._by_hash[h]

    def spec(self, v):
        if isinstance(v, torch.Tensor):
            base = v._base if v._base is not None else v
            return {"t": self._store(base), "dtype": _TRACE_DTYPES[v.dtype],
                    "base_size": list(base.shape), "size": list(v.shape), "stride": list(v.stride()),
                    "offset": v.storage_offset() - base.storage_offset()}
        if isinstance(v, torch.dtype):
            return {"dtype_arg": _TRACE_DTYPES[v]}
        if isinstance(v, (tuple, list)):
            return {"seq": [self.spec(x) for x in v]}
        return {"v": v}

    def wrap(self, fn_name, fn):
        def call(*args, **kwargs):
            rec = {"fn": fn_name, "args": [self.spec(a) for a in args],
                   "kwargs": {k: self.spec(v) for k, v in kwargs.items()},
                   "default_dtype": _TRACE_DTYPES[torch.get_default_dtype()]}
            out = fn(*args, **kwargs)
            rec["out"] = self.spec(out)
            if isinstance(out, torch.Tensor) and out._base is not None:  # in place on a view
                rec["out_base_after"] = self.spec(out._base)
            self.calls.append(rec)
            return out
        return call


def attention_trace_fixture():
    """attention_trace.npz: the calls the reference's own Attention.forward
    (Deepseek_origin/inference/model.py:484-543, the module that does
    `from kernel import ...`, model.py:12) makes into its kernel module, run on
    the CPU with kernel_fallback as that module: a seeded V4-width layer
    (4 heads of 512, rope 64, q_lora_rank 128, FP8 weights with UE8M0 scales,
    window 16, compress ratio 4 with the Lightning indexer: 4 heads of 128,
    index_topk 8) over a 24-token prefill of 2 sequences and 2 decode steps.
    rotate_activation is the QCAU package's fp32 restatement (model.py:302-
    323 there; fast_hadamard_transform is not installed).  Each call keeps its
    arguments as the call site passed them (views included), its results, and
    the layer outputs are kept as out/<step>."""
    load_qcau_inference_model()  # kernel_fallback inside its package: sparse_attn imports .QCAU
    kf = sys.modules["qcau_ref_inference.kernel_fallback"]
    tw = _TraceWriter()
    shim = type(sys)("kernel")
    for n in ("act_quant", "fp8_gemm", "sparse_attn", "fp4_act_quant", "fp4_gemm",
              "hc_split_sinkhorn"):
        setattr(shim, n, tw.wrap(n, getattr(kf, n)))
    sys.modules["kernel"] = shim
    model = load_module("ref_model_v4_trace", REF / "Deepseek_origin/inference/model.py")
    model.rotate_activation = load_qcau_inference_model().rotate_activation
    model.scale_fmt, model.scale_dtype = "ue8m0", torch.float8_e8m0fnu
    model.default_dtype = torch.float8_e4m3fn
    args = model.ModelArgs(max_batch_size=2, max_seq_len=64, dim=256, n_heads=4, q_lora_rank=128,
                           head_dim=512, rope_head_dim=64, o_groups=2, o_lora_rank=128,
                           window_size=16, compress_ratios=(4,), index_n_heads=4,
                           index_head_dim=128, index_topk=8, original_seq_len=0)
    g = torch.Generator().manual_seed(23)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    out = {}
    try:
        attn = model.Attention(0, args)
        with torch.no_grad():
            for name, p in attn.named_parameters():
                if p.dtype == torch.float8_e4m3fn:
                    n_out, n_in = p.shape
                    w = torch.randn(n_out, n_in, generator=g) / n_in ** 0.5
                    blk = w.view(n_out // 128, 128, n_in // 128, 128)
                    sc = torch.exp2(torch.ceil(torch.log2(
                        blk.abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0)))
                    p.copy_((blk / sc[:, None, :, None]).clamp(-448, 448).view(n_out, n_in)
                            .to(torch.float8_e4m3fn))
                    p.scale.copy_(sc.to(torch.float8_e8m0fnu))
                elif name.endswith("scale"):
                    continue
                elif name.endswith("norm.weight"):
                    p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
                elif name.endswith("ape") or name.endswith("attn_sink"):
                    p.copy_(0.5 * torch.randn(p.shape, generator=g))
                else:
                    p.copy_((torch.randn(p.shape, generator=g) / p.shape[-1] ** 0.5).to(p.dtype))
            steps = [(0, 24), (24, 1), (25, 1)]
            for i, (sp, sl) in enumerate(steps):
                x = torch.randn(2, sl, 256, generator=g).to(torch.bfloat16)
                first = len(tw.calls)
                y = attn(x, sp)
                for c in tw.calls[first:]:
                    c["step"] = i
                out[f"out/{i}"] = u16(y)
    finally:
        torch.set_default_dtype(prev)
    out.update(tw.arrays)
    out["calls"] = np.array(json.dumps(tw.calls))
    np.savez_compressed(OUT / "attention_trace.npz", **out)


def compressor_fixture():
    """compressor.npz: the reference's Compressor.forward (QCAU/QCAU_inference/
    inference/model.py:415-476) run by its own code on seeded projections:
    c4 = the attention's compressor (ratio 4, overlapping windows, 512 wide,
    FP8 round trip with UE8M0 scales), c8 = a non-overlapping one (ratio 8),
    i4 = the indexer's (ratio 4, 128 wide, Hadamard rotation; kernel_fallback's
    fp4_act_quant leaves the rotated values unchanged).  Each case is a prefill
    and decode steps past two group boundaries; per step the projections the
    compressor computed (kv, score: the wkv / wgate outputs), the rows it
    returned (out, absent when it returned None) and the rows given to
    rotate_activation (pre_rot, i4); the cache and the state after the
    prefill and after the last step."""
    model = load_qcau_inference_model()
    model.scale_fmt, model.scale_dtype = "ue8m0", torch.float8_e8m0fnu
    g = torch.Generator().manual_seed(29)
    out = {}
    cases = {"c4": (4, 512, False, 10, 6), "c8": (8, 512, False, 19, 5), "i4": (4, 128, True, 10, 6)}
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    real_rot = model.rotate_activation
    rec = {}

    def rot(t):
        rec["pre_rot"] = t.clone()
        return real_rot(t)

    model.rotate_activation = rot
    try:
        for name, (ratio, d, rotate, s0, ndec) in cases.items():
            args = model.ModelArgs(max_batch_size=2, max_seq_len=64, dim=128, rope_head_dim=64)
            comp = model.Compressor(args, ratio, d, rotate)
            with torch.no_grad():
                comp.ape.copy_(0.5 * torch.randn(comp.ape.shape, generator=g))
                comp.norm.weight.copy_(1.0 + 0.1 * torch.randn(d, generator=g))
                for lin in (comp.wkv, comp.wgate):
                    lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) / 128 ** 0.5)
            comp.kv_cache = torch.zeros(2, 64 // ratio, d, dtype=torch.bfloat16)
            comp.freqs_cis = model.precompute_freqs_cis(64, 64, 0, 10000.0, 40, 32, 1)
            comp.wkv.register_forward_hook(lambda m, a, o: rec.__setitem__("kv", o.clone()))
            comp.wgate.register_forward_hook(lambda m, a, o: rec.__setitem__("score", o.clone()))
            out[f"{name}/ape"] = comp.ape.detach().numpy().copy()
            out[f"{name}/norm"] = comp.norm.weight.detach().numpy().copy()
            out[f"{name}/freqs"] = torch.view_as_real(comp.freqs_cis).numpy().astype(np.float32)
            steps = [(0, s0)] + [(s0 + i, 1) for i in range(ndec)]
            for i, (sp, sl) in enumerate(steps):
                x = torch.randn(2, sl, 128, generator=g).to(torch.bfloat16)
                rec.pop("pre_rot", None)
                with torch.no_grad():
                    y = comp(x, sp)
                k = f"{name}/step{i}"
                out[f"{k}/meta"] = np.array([sp, sl], dtype=np.int64)
                out[f"{k}/kv"] = rec["kv"].numpy().copy()
                out[f"{k}/score"] = rec["score"].numpy().copy()
                if y is not None:
                    out[f"{k}/out"] = u16(y.contiguous())
                if "pre_rot" in rec:
                    out[f"{k}/pre_rot"] = u16(rec["pre_rot"].contiguous())
                if i in (0, len(steps) - 1):  # after the prefill and at the end
                    out[f"{k}/cache"] = u16(comp.kv_cache.clone())
                    out[f"{k}/kv_state"] = comp.kv_state[:2].numpy().copy()
                    out[f"{k}/score_state"] = comp.score_state[:2].numpy().copy()
    finally:
        model.rotate_activation = real_rot
        torch.set_default_dtype(prev)
    np.savez_compressed(OUT / "compressor.npz", **out)


if __name__ == "__main__":
    if not VEC.exists():
        sys.exit(f"reference test vectors not found under {REF} (set QCAU_REFERENCE_ROOT)")
    goldens()
    synthetic()
    kv_build_fixture()
    gopu_fixture()
    indexer_fixture()
    attention_trace_fixture()
    compressor_fixture()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)
