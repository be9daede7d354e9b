"""GPU parity of the KV build (qcau_kv_build through qcau_b200.cache) against
the reference's own computation, the oracle and the reference's golden cache
rows, and its cache writes (window ring and paged cache)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from helpers import f32, n_bf16, t_bf16

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200.cache import PagedKVCache, kv_build, window_slots

GOLDEN = Path(__file__).resolve().parent / "golden"


def _fixture():
    g = np.load(GOLDEN / "kv_build.npz")
    rows = g["x"].shape[0]
    return g, torch.from_numpy(g["freqs"]).cuda(), torch.arange(rows, dtype=torch.int32).cuda()


def test_fp8_round_trip_bit_exact_with_reference_act_quant():
    """The FP8 stage alone, on the reference's own normalised and rotated rows:
    the codes and scales of kernel_fallback.act_quant(kv[..., :-64], 64,
    "ue8m0", inplace=True), bit for bit."""
    g, freqs, pos = _fixture()
    y = kv_build(t_bf16(g["after_norm_rope"]), None, freqs, pos, rope_dim=0, norm_dim=0,
                 quant_dims=448, scale_fmt="ue8m0")
    assert np.array_equal(n_bf16(y), g["kv"])
    assert _lib.device_error() == 0


def test_kv_build_chain_vs_reference_and_oracle():
    """RMSNorm (weight), YaRN RoPE at each row's position, FP8 round trip: the
    whole chain against the reference's output and the oracle.  The RMSNorm
    mean is summed in another order than torch's, so a value at a rounding
    boundary may move by one bf16 ulp before the quantisation."""
    g, freqs, pos = _fixture()
    w = torch.from_numpy(g["weight"]).cuda()
    y = n_bf16(kv_build(t_bf16(g["x"]), w, freqs, pos))
    ref = O.kv_build(g["x"], g["weight"], 512, 1e-6, g["freqs"], np.arange(len(g["x"]), dtype=np.int32),
                     64, 448, True)
    for name, want in (("reference", g["kv"]), ("oracle", ref)):
        bad = int(np.sum(y != want))
        assert bad <= y.size // 1000, f"{name}: {bad} values differ"
        d = np.abs(f32(y) - f32(want))
        assert float(d.max()) <= 0.05 * float(np.abs(f32(want)).max()), name
    assert _lib.device_error() == 0


def test_fp8_round_trip_fixed_point_on_golden_cache_rows(golden_dir):
    """The reference's cache rows (kv_after_rope_quant_compress of the 36
    golden cases) have been through the UE8M0 FP8 round trip already; a power
    of two scale makes it idempotent, so the kernel returns them unchanged."""
    a = np.load(golden_dir / "attn_goldens.npz")
    for c in a["cases"]:
        kv = a[f"{c}/kv"].reshape(-1, 512)
        pos = torch.zeros(kv.shape[0], dtype=torch.int32, device="cuda")
        freqs = torch.zeros(1, 32, 2, device="cuda")
        y = kv_build(t_bf16(kv), None, freqs, pos, rope_dim=0, norm_dim=0, quant_dims=448)
        assert np.array_equal(n_bf16(y), kv), c
    assert _lib.device_error() == 0


def test_window_ring_cache_writes():
    """Prefill of 21 tokens into 8-token rings of 3 sequences: only the last 8
    of each land, at position % 8; rows outside the rings stay untouched."""
    bsz, seqlen, win, ring = 3, 21, 8, 13
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.randn(bsz * seqlen, 512, device="cuda", generator=gen) * 2).to(torch.bfloat16)
    freqs = torch.view_as_real(torch.polar(torch.ones(64, 32), torch.rand(64, 32) * 6)).cuda()
    positions = torch.arange(seqlen, dtype=torch.int32, device="cuda").repeat(bsz)
    cache = torch.full((bsz * ring, 512), 7.0, device="cuda", dtype=torch.bfloat16)
    slots = window_slots(bsz, seqlen, 0, win, ring, "cuda")
    y = kv_build(x, None, freqs, positions, cache=cache, slots=slots)
    torch.cuda.synchronize()
    sl = slots.cpu().numpy()
    yc, cc = y.cpu(), cache.cpu()
    written = set()
    for r, s in enumerate(sl):
        if s >= 0:
            assert torch.equal(cc[s], yc[r])
            written.add(int(s))
    assert len(written) == bsz * win
    for s in range(bsz * ring):
        if s not in written:
            assert bool((cc[s] == 7.0).all())
    assert _lib.device_error() == 0


def test_paged_cache_absorbed_rows_vs_oracle():
    """Absorbed-MLA cache rows (576 = 512 latent + 64 rope): RMSNorm of the
    latent part, RoPE of the rope part, no FP8 round trip, appended through
    PagedKVCache and read back from the rows it returned."""
    pc = PagedKVCache(num_pages=16, max_seqs=4, max_pages=6, width=576, device="cuda")
    seqs, counts = [0, 2, 3], [70, 1, 129]
    slots = pc.append(seqs, counts)
    positions = pc.positions(seqs, counts)
    n = sum(counts)
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(n, 576, device="cuda", generator=gen).to(torch.bfloat16)
    w = 1.0 + 0.1 * torch.randn(512, device="cuda", generator=gen)
    freqs = torch.view_as_real(torch.polar(torch.ones(256, 32), torch.rand(256, 32) * 6)).cuda()
    kv_build(x, w, freqs, positions, norm_dim=512, rope_dim=64, quant_dims=0, cache=pc.cache,
             slots=slots, return_rows=False)
    torch.cuda.synchronize()
    got = pc.cache.view(-1, 576)[slots.long()]
    ref = O.kv_build(n_bf16(x), w.cpu().numpy(), 512, 1e-6, freqs.cpu().numpy(),
                     positions.cpu().numpy(), 64, 0, False)
    g = n_bf16(got)
    assert int(np.sum(g != ref)) <= g.size // 1000
    assert float(np.abs(f32(g) - f32(ref)).max()) <= 0.02 * float(np.abs(f32(ref)).max())
    # the block table and lengths are what the decode attention reads
    assert pc.seqlens.tolist() == [70, 0, 1, 129]
    assert _lib.device_error() == 0


def test_slot_out_of_range_is_skipped_and_flagged():
    x = torch.ones(4, 512, device="cuda", dtype=torch.bfloat16)
    cache = torch.zeros(8, 512, device="cuda", dtype=torch.bfloat16)
    slots = torch.tensor([0, 9, -1, 3], dtype=torch.int32, device="cuda")
    freqs = torch.zeros(4, 32, 2, device="cuda")
    pos = torch.zeros(4, dtype=torch.int32, device="cuda")
    kv_build(x, None, freqs, pos, rope_dim=0, quant_dims=0, cache=cache, slots=slots)
    assert _lib.device_error() == _lib.DEVERR_INDEX
    c = cache.float().cpu()
    assert bool((c[0] != 0).all()) and bool((c[3] != 0).all())
    assert bool((c[[1, 2, 4, 5, 6, 7]] == 0).all())
