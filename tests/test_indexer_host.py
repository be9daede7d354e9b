"""The index-list producers' oracle against the reference's own code, and the
library's argument checks, without a GPU.

tests/golden/indexer.npz was made by make_golden.py from the QCAU package's
model.py (get_window_topk_idxs, get_compress_topk_idxs, rotate_activation and
Indexer.forward on kernel_fallback); see that script for the cases.
"""
from pathlib import Path

import numpy as np
import pytest

import indexer_oracle as IO
import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "indexer.npz")


def _steps(g):
    i = 0
    while f"step{i}/meta" in g.files:
        yield i
        i += 1


def test_index_lists_match_reference(g):
    for i, (win, ratio, bsz, seqlen, sp, off) in enumerate(g["list_params"]):
        want = g[f"lists/{i}"]
        got = IO.index_lists(int(win), int(ratio), int(bsz), int(seqlen), int(sp), int(off))
        assert got.shape == want.shape, (i, got.shape, want.shape)
        assert np.array_equal(got, want), i


def test_hadamard_matches_reference_bit_for_bit(g):
    assert np.array_equal(IO.hadamard_rotate(g["rot_x"]), g["rot_y"])
    for i in _steps(g):
        # kernel_fallback's fp4_act_quant leaves the rotated values unchanged
        assert np.array_equal(IO.hadamard_rotate(g[f"step{i}/q_pre"]), g[f"step{i}/q"]), i


def test_hadamard_is_its_own_inverse_up_to_rounding():
    rng = np.random.default_rng(0)
    x = O.f32_to_bf16(rng.standard_normal((16, 128)).astype(np.float32))
    back = O.bf16_to_f32(IO.hadamard_rotate(IO.hadamard_rotate(x)))
    assert np.max(np.abs(back - O.bf16_to_f32(x))) <= 0.02 * np.max(np.abs(O.bf16_to_f32(x)))


def test_fp4_known_values_and_ties():
    # a block with amax 6 has scale 1: the values are rounded to e2m1 directly
    vals = np.array([6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5, -0.25, -0.3, -5.5, 0.74] + [0] * 20,
                    dtype=np.float32)
    y = O.bf16_to_f32(IO.fp4_quant(O.f32_to_bf16(vals[None])))[0]
    assert y[:12].tolist() == [6, 0, 1, 1, 2, 2, 4, 4, -0.0, -0.5, -6, 0.5]
    assert np.signbit(y[8])  # -0.25 rounds to -0
    # amax 3 -> scale 2^ceil(log2(0.5)) = 0.5: codes times 0.5
    v2 = np.array([3, 0.3, 1.1] + [0] * 29, dtype=np.float32)
    y2 = O.bf16_to_f32(IO.fp4_quant(O.f32_to_bf16(v2[None])))[0]
    assert y2[:3].tolist() == [3, 0.25, 1.0]
    # a zero block takes the floor scale and stays zero
    assert not O.bf16_to_f32(IO.fp4_quant(np.zeros((1, 32), np.uint16))).any()


def test_fp4_idempotent_and_on_grid():
    rng = np.random.default_rng(1)
    x = O.f32_to_bf16((rng.standard_normal((64, 128)) * 3).astype(np.float32))
    y = IO.fp4_quant(x)
    assert np.array_equal(IO.fp4_quant(y), y)
    yb = O.bf16_to_f32(y).reshape(-1, 32)
    amax = np.abs(O.bf16_to_f32(x)).reshape(-1, 32).max(1)
    s = np.exp2(np.ceil(np.log2(amax / 6)))
    codes = np.abs(yb / s[:, None])
    assert np.all(np.isin(codes, [0, 0.5, 1, 1.5, 2, 3, 4, 6]))


def _ulp_close(a, b):
    d = np.abs(a - b)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32)) * 65536
    return (d <= ulp) | (a == b)


def test_index_scores_vs_reference(g):
    """Exact dot products rounded once against torch's bf16 einsum on the
    CPU (fp32 partial sums): a score may move by one bf16 ulp."""
    for i in _steps(g):
        sp, sl, off = (int(v) for v in g[f"step{i}/meta"])
        raw = IO.raw_scores(g[f"step{i}/q"], g[f"step{i}/kv"])
        sc = IO.index_scores(raw, g[f"step{i}/w"])
        if sp == 0:
            t = sc.shape[-1]
            mask = np.arange(t)[None, :] >= (np.arange(1, sl + 1)[:, None] // 4)
            sc = np.where(mask[None], -np.inf, sc)
        ref = g[f"step{i}/score"]
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(sc), fin)
        ok = _ulp_close(sc[fin], ref[fin])
        assert ok.all(), i
        assert int(np.sum(sc[fin] != ref[fin])) <= max(2, fin.sum() // 50), i


def _check_topk_rows(got, want, score, k):
    """got / want [R, k] index lists over the same score rows: the same -1
    pattern and, position by position, the same scores (the reference's
    order among equal scores is unspecified); identical where a row's
    selected scores are all distinct."""
    for r in range(got.shape[0]):
        gv, wv = got[r], want[r]
        assert np.array_equal(gv < 0, wv < 0), r
        sel = gv >= 0
        assert np.array_equal(score[r][gv[sel]], score[r][wv[sel]]), r
        if len(np.unique(score[r][wv[sel]])) == sel.sum():
            assert np.array_equal(gv, wv), r


def test_topk_vs_reference_on_reference_scores(g):
    for i in _steps(g):
        sp, sl, off = (int(v) for v in g[f"step{i}/meta"])
        ref = g[f"step{i}/score"]
        want = g[f"step{i}/idx"]
        b, s, t = ref.shape
        k = want.shape[-1]
        got = IO.topk(ref.reshape(b * s, t), k, off, s, 4 if sp == 0 else 0).reshape(b, s, k)
        sel_want = np.where(want >= 0, want - off, -1).reshape(b * s, k)
        sel_got = np.where(got >= 0, got - off, -1).reshape(b * s, k)
        _check_topk_rows(sel_got, sel_want, ref.reshape(b * s, t), k)


def test_topk_tie_order_and_mask():
    score = np.array([[1, 3, 3, -np.inf, 3, 2, 0.5, 3]], dtype=np.float32)
    assert IO.topk(score, 4).tolist() == [[1, 2, 4, 7]]
    assert IO.topk(score, 7, offset=10).tolist() == [[11, 12, 14, 17, 15, 10, 16]]
    assert IO.topk(score, 8).tolist()[0][-1] == -1
    # prefill mask: row r of a 3-token sequence sees positions < (r + 1) // 1
    sc = np.tile(np.array([[5, 4, 3]], dtype=np.float32), (3, 1))
    assert IO.topk(sc, 3, 0, 3, 1).tolist() == [[0, -1, -1], [0, 1, -1], [0, 1, 2]]


def test_library_rejects_bad_indexer_arguments():
    torch = pytest.importorskip("torch")
    from qcau_b200 import _lib

    lib = _lib.lib()
    assert lib.qcau_topk(None, None, 1, 8, 4, 0, 0, 0, None) == _lib.QCAU_ERR_INVALID
    assert lib.qcau_rotate_fp4(8, 1, 64, 1, 1, None) == _lib.QCAU_ERR_INVALID
    buf = 256
    assert lib.qcau_topk(buf, buf, 1, 8, 4096, 0, 0, 0, None) == _lib.QCAU_ERR_INVALID
    assert lib.qcau_topk(buf, buf, 1, 8, 4, 0, 4, 0, None) == _lib.QCAU_ERR_INVALID  # mask, no seqlen
    need = lib.qcau_indexer_topk_workspace_size(2, 3, 8, 17)
    assert need >= 2 * 3 * 17 * 4
    assert lib.qcau_indexer_scores_workspace_size(2, 3, 8, 17) == 0
    # the fused score pass: head_dim 128 and up to 128 heads a rank
    assert lib.qcau_indexer_scores(buf, buf, buf, buf, 1, 1, 129, 128, 8, 8, None, 0,
                                   None) == _lib.QCAU_ERR_INVALID
    assert lib.qcau_indexer_scores(buf, buf, buf, buf, 1, 1, 8, 64, 8, 8, None, 0,
                                   None) == _lib.QCAU_ERR_INVALID
    rc = lib.qcau_indexer_topk(buf, buf, buf, buf, 2, 3, 8, 128, 17, 17, 8, 0, 4, 0, buf, need - 1,
                               None)
    assert rc == _lib.QCAU_ERR_WORKSPACE
    assert lib.qcau_index_lists_width(300, 0, 128, 4, 0) == 128 + 75
    assert lib.qcau_index_lists_width(1, 131, 128, 4, 0) == 128 + 33
    assert lib.qcau_index_lists_width(1, 131, 128, 4, 512) == 128 + 512
    assert lib.qcau_index_lists(buf, 1, 4, 5, 8, 4, 0, None, 0, None) == _lib.QCAU_ERR_INVALID
    del torch
