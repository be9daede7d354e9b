"""GPU parity of the index-list producers (qcau_b200.indexer through the C
ABI) against the reference's outputs (tests/golden/indexer.npz, made from the
QCAU package's model.py) and the oracle (oracle/indexer_oracle.py).

Bars: the Hadamard rotation, the FP4 round trip, the weighted head sum, the
top-k selection and the index lists are bit-exact against the oracle on the
same inputs; the raw q . k scores (the tcgen05 GEMM) are within one bf16 ulp
of the exact dot product rounded once; against the reference's own
Indexer.forward the selected positions carry the same scores (equal scores
may be listed in another order) and are identical where a row has no ties.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import indexer_oracle as IO
import oracle as O
from helpers import n_bf16, t_bf16

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200 import indexer as I

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "indexer.npz")


def _steps(g):
    i = 0
    while f"step{i}/meta" in g.files:
        yield i
        i += 1


def _ok():
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_rotate_activation_bit_exact_with_reference(g):
    assert np.array_equal(n_bf16(I.rotate_activation(t_bf16(g["rot_x"]))), g["rot_y"])
    for i in _steps(g):
        q = I.rotate_activation(t_bf16(g[f"step{i}/q_pre"]))
        assert np.array_equal(n_bf16(q), g[f"step{i}/q"]), i
    _ok()


@pytest.mark.parametrize("scale", [1e-30, 1e-3, 1.0, 37.0, 3e4])
def test_fp4_and_rotate_fp4_bit_exact_with_oracle(scale):
    gen = torch.Generator(device="cuda").manual_seed(int(scale * 7) % 1000)
    x = (torch.randn(1000, 128, device="cuda", generator=gen) * scale).to(torch.bfloat16)
    x[3, :32] = 0
    x[4, :32] = torch.tensor([6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5] * 4, device="cuda")
    x[5, :32] = -x[4, :32]
    xn = n_bf16(x)
    y = I.fp4_act_quant(x.clone(), 32, inplace=True)
    assert np.array_equal(n_bf16(y), IO.fp4_quant(xn))
    z = I.rotate_fp4_(x.clone())
    assert np.array_equal(n_bf16(z), IO.fp4_quant(IO.hadamard_rotate(xn)))
    _ok()


def test_index_lists_bit_exact_with_reference(g):
    for i, (win, ratio, bsz, seqlen, sp, off) in enumerate(g["list_params"]):
        want = g[f"lists/{i}"]
        got = I.index_lists(int(win), int(ratio), int(bsz), int(seqlen), int(sp), int(off))
        assert np.array_equal(got.cpu().numpy(), want), i
        w = I.get_window_topk_idxs(int(win), int(bsz), int(seqlen), int(sp))
        assert np.array_equal(w.cpu().numpy(), IO.window_topk_idxs(int(win), int(bsz), int(seqlen), int(sp)))
        if ratio:
            c = I.get_compress_topk_idxs(int(ratio), int(bsz), int(seqlen), int(sp), int(off))
            assert np.array_equal(c.cpu().numpy(),
                                  IO.compress_topk_idxs(int(ratio), int(bsz), int(seqlen), int(sp), int(off)))
    # the indexer's selection in place of the compressed positions
    sel = torch.randint(-1, 500, (2, 1, 7), dtype=torch.int32, device="cuda")
    got = I.index_lists(128, 4, 2, 1, 300, 128, selected=sel).cpu().numpy()
    assert np.array_equal(got, IO.index_lists(128, 4, 2, 1, 300, 128, sel.cpu().numpy()))
    _ok()


def _raw(q, kv, t):
    """The einsum the indexer's fused score pass keeps on chip, from the
    separate raw-score entry (the tcgen05 bmm): the scores below are checked
    against the oracle's head sum of exactly these values."""
    return n_bf16(I.raw_scores(q, kv, t).contiguous())


def _check_topk_rows(got, want, score):
    for r in range(got.shape[0]):
        gv, wv = got[r], want[r]
        assert np.array_equal(gv < 0, wv < 0), r
        sel = gv >= 0
        assert np.array_equal(score[r][gv[sel]], score[r][wv[sel]]), r
        if len(np.unique(score[r][wv[sel]])) == sel.sum():
            assert np.array_equal(gv, wv), r


def test_indexer_forward_vs_reference_steps(g):
    """The reference's prefill and decode steps: the same inputs the
    reference's einsum read, our scores within an ulp of its scores, our
    selection the oracle's on our scores bit for bit, and the reference's
    up to the order of equal scores."""
    ix = I.Indexer(n_heads=8, head_dim=128, index_topk=8, compress_ratio=4)
    for i in _steps(g):
        sp, sl, off = (int(v) for v in g[f"step{i}/meta"])
        q, kv, w = g[f"step{i}/q"], g[f"step{i}/kv"], g[f"step{i}/w"]
        b, s, h, _ = q.shape
        t = kv.shape[1]
        # a cache with more rows than the step reads (the reference slices its buffer)
        cache = torch.zeros(b, t + 9, 128, dtype=torch.bfloat16, device="cuda")
        cache[:, :t] = t_bf16(kv)
        got = ix.forward(t_bf16(q), cache, t_bf16(w), sp, off, rotate=False)
        torch.cuda.synchronize()
        got = got.cpu().numpy()
        want = g[f"step{i}/idx"]
        assert got.shape == want.shape
        raw = _raw(t_bf16(q), cache, t)
        ref_raw = IO.raw_scores(q, kv)
        d = np.abs(O.bf16_to_f32(raw) - O.bf16_to_f32(ref_raw))
        assert np.all(d <= np.spacing(np.abs(O.bf16_to_f32(ref_raw))) * 65536 + 0), i
        score = IO.index_scores(raw, w)
        sel = IO.topk(score.reshape(b * s, t), want.shape[-1], off, s, 4 if sp == 0 else 0)
        assert np.array_equal(got.reshape(b * s, -1), sel), i
        ref_score = g[f"step{i}/score"].reshape(b * s, t)
        rel = lambda a: np.where(a >= 0, a - off, -1)
        _check_topk_rows(rel(got.reshape(b * s, -1)), rel(want.reshape(b * s, -1)), ref_score)
    _ok()


@pytest.mark.parametrize("b,s,start_pos,t,k", [
    (4, 1, 32767, 8192, 512),     # decode at 32k context, ratio 4
    (2, 1, 511, 128, 512),        # k above the candidates: all of them, then -1
    (1, 256, 0, 64, 512),         # prefill: the mask leaves rows short of k
    (1, 1024, 0, 256, 128),       # prefill, k below the candidates for later rows
])
def test_indexer_chain_bit_exact_with_oracle(b, s, start_pos, t, k):
    h = 64
    gen = torch.Generator(device="cuda").manual_seed(b * 1000 + s + t)
    q = torch.randn(b, s, h, 128, device="cuda", generator=gen).to(torch.bfloat16)
    kv = torch.randn(b, t, 128, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(b, s, h, device="cuda", generator=gen) * 0.01).to(torch.bfloat16)
    ix = I.Indexer(n_heads=h, head_dim=128, index_topk=k, compress_ratio=4)
    assert (start_pos + s) // 4 == t
    got = ix.forward(q, kv, w, start_pos, 1000, rotate=True)
    torch.cuda.synchronize()
    kk = min(k, t)
    assert got.shape == (b, s, kk)
    qr = IO.fp4_quant(IO.hadamard_rotate(n_bf16(q)))
    raw = _raw(I.rotate_fp4_(q.clone()), kv, t)
    ref_raw = IO.raw_scores(qr, n_bf16(kv))
    rf, gf = O.bf16_to_f32(ref_raw), O.bf16_to_f32(raw)
    assert np.all(np.abs(rf - gf) <= np.spacing(np.abs(rf)) * 65536)
    assert int(np.sum(rf != gf)) <= rf.size // 200
    score = IO.index_scores(raw, n_bf16(w)).reshape(b * s, t)
    want = IO.topk(score, kk, 1000, s, 4 if start_pos == 0 else 0)
    assert np.array_equal(got.cpu().numpy().reshape(b * s, kk), want)
    _ok()


@pytest.mark.parametrize("rows,t,k,levels", [(8, 16384, 2048, 7), (64, 4096, 512, 3),
                                             (3, 100, 37, 1), (5, 3000, 2048, 50)])
def test_topk_ties_and_infinities_bit_exact(rows, t, k, levels):
    """Score rows with few distinct values (ties across the k-th place) and
    -inf entries: the selection is the lowest indices among equal scores."""
    gen = torch.Generator(device="cuda").manual_seed(rows * t)
    sc = torch.randint(0, levels, (rows, t), device="cuda", generator=gen).float() * 0.5 - 1
    sc[torch.rand(rows, t, device="cuda", generator=gen) < 0.1] = float("-inf")
    sc[0, : t // 2] = float("-inf")
    got = I.topk(sc, k, offset=7)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), IO.topk(sc.cpu().numpy(), k, 7))
    _ok()


def test_topk_prefill_mask_and_empty_rows():
    sc = torch.randn(2 * 33, 8, device="cuda")
    got = I.topk(sc, 8, 5, seqlen=33, mask_ratio=4)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), IO.topk(sc.cpu().numpy(), 8, 5, 33, 4))
    assert I.topk(torch.empty(3, 0, device="cuda"), 4).cpu().tolist() == [[-1] * 4] * 3
    _ok()


@pytest.mark.parametrize("b,s,h,t,kv_rows", [
    (128, 1, 64, 8192, 8192),    # the decode batch of 128 sequences at 32768 tokens (ratio 4)
    (3, 1, 8, 300, 333),         # one rank of eight (64 heads / 8), ragged last tile, longer rows
    (2, 5, 16, 129, 129),        # several query rows a sequence, one key past a tile
    (2, 3, 48, 1000, 1024),      # heads padded to 64 in the MMA
    (1, 2, 128, 640, 700),       # 128 heads a rank
])
def test_fused_score_rows_bit_exact_with_oracle(b, s, h, t, kv_rows):
    """qcau_indexer_scores (one pass: the einsum in TMEM, ReLU x weight and the
    head sum in the epilogue) against the oracle's head sum of the einsum's
    bf16 values, bit for bit, on every row (sampled sequences at the decode
    batch)."""
    gen = torch.Generator(device="cuda").manual_seed(b * 7 + s * 5 + h + t)
    q = torch.randn(b, s, h, 128, device="cuda", generator=gen).to(torch.bfloat16)
    kv = torch.randn(b, kv_rows, 128, device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn(b, s, h, device="cuda", generator=gen) * 0.01).to(torch.bfloat16)
    score = torch.full((b * s, t), float("nan"), device="cuda")
    L = _lib.lib()
    _lib.check(L.qcau_indexer_scores(q.data_ptr(), kv.data_ptr(), w.data_ptr(), score.data_ptr(),
                                     b, s, h, 128, t, kv_rows, None, 0,
                                     _lib.stream_ptr(q.device)), "indexer_scores")
    raw = I.raw_scores(q, kv, t)
    _ok()
    seqs = range(b) if b <= 8 else [0, 1, 37, 64, 100, 126, 127]
    got = score.view(b, s, t)
    for bi in seqs:
        want = IO.index_scores(n_bf16(raw[bi].contiguous()), n_bf16(w[bi]))
        assert np.array_equal(got[bi].cpu().numpy(), want.astype(np.float32)), bi
