"""The KV compressor's oracle against the reference's own Compressor.forward
(tests/golden/compressor.npz, made by make_golden.py from the QCAU package's
model.py on kernel_fallback), without a GPU.

The reference's softmax exponent is torch's and the oracle's numpy's, so a
pooled value can round to the neighbouring bf16; the norm and the FP8 round
trip after it then move that row's values slightly.  The bar: the decode
state bit-exact (copies and one fp32 add), and the finished rows equal in
>= 99 % of values, every value within 2 % of the row's largest.
"""
from pathlib import Path

import numpy as np
import pytest

import compressor_oracle as CO
import indexer_oracle as IO
import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = {"c4": (4, 512, False), "c8": (8, 512, False), "i4": (4, 128, True)}


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "compressor.npz")


def close_rows(got, want, what):
    got, want = O.bf16_to_f32(got).reshape(-1, got.shape[-1]), O.bf16_to_f32(want).reshape(-1, want.shape[-1])
    assert got.shape == want.shape, what
    assert np.mean(got == want) >= 0.99, (what, float(np.mean(got == want)))
    scale = np.abs(want).max(axis=1, keepdims=True)
    assert np.all(np.abs(got - want) <= 0.02 * scale), what


def run_oracle(g, name):
    """The oracle over the case's steps: [(step, out rows or None, states)]."""
    ratio, d, rotate = CASES[name]
    overlap = ratio == 4
    ks, ss = CO.new_state(2, ratio, d, overlap)
    ape, norm, freqs = g[f"{name}/ape"], g[f"{name}/norm"], g[f"{name}/freqs"]
    res = []
    i = 0
    while f"{name}/step{i}/meta" in g.files:
        sp, sl = (int(v) for v in g[f"{name}/step{i}/meta"])
        kv, sc = g[f"{name}/step{i}/kv"], g[f"{name}/step{i}/score"]
        if sp == 0:
            pooled = CO.prefill(kv, sc, ape, ratio, overlap, ks, ss)
            pos = np.tile(np.arange(pooled.shape[1]) * ratio, 2)
        else:
            pooled = CO.decode(kv, sc, ape, ratio, overlap, ks, ss, sp)
            pos = np.full(2, sp + 1 - ratio)
        rows = None
        if pooled is not None and pooled.shape[1]:
            rows = CO.finish(pooled.reshape(-1, d), norm, freqs, pos, rotate).reshape(2, -1, d)
        res.append((i, sp, rows, ks.copy(), ss.copy()))
        i += 1
    return res


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_reference_compressor(g, name):
    ratio, d, rotate = CASES[name]
    outs = 0
    for i, sp, rows, ks, ss in run_oracle(g, name):
        k = f"{name}/step{i}"
        assert (rows is not None) == (f"{k}/out" in g.files), k
        if rows is not None:
            want = g[f"{k}/out"]
            if rotate:
                # kernel_fallback's fp4_act_quant does not round: compare the
                # rotation, then the FP4 stage on the reference's own rows
                want = IO.fp4_quant(want)
            close_rows(rows, want, k)
            outs += 1
        if f"{k}/kv_state" in g.files:
            assert np.array_equal(ks, g[f"{k}/kv_state"]), k
            assert np.array_equal(ss, g[f"{k}/score_state"]), k
    assert outs >= 2  # the prefill and at least one decode boundary


def test_oracle_pooling_edge_cases():
    """A window whose scores are equal averages it; one score far above the
    others selects its value; the first group's overlap half (score -inf)
    takes no weight."""
    b, ratio, d = 1, 4, 2
    kv = np.arange(b * 8 * 2 * d, dtype=np.float32).reshape(b, 8, 2 * d)
    sc = np.zeros_like(kv)
    ape = np.zeros((ratio, 2 * d), dtype=np.float32)
    ks, ss = CO.new_state(b, ratio, d, True)
    out = O.bf16_to_f32(CO.prefill(kv, sc, ape, ratio, True, ks, ss))
    # group 0: the mean of its own tokens' second-half channels
    assert np.allclose(out[0, 0], kv[0, :4, d:].mean(0), rtol=1e-2)
    # group 1: the mean over the previous group's first half and its own second half
    assert np.allclose(out[0, 1], np.concatenate([kv[0, :4, :d], kv[0, 4:, d:]]).mean(0), rtol=1e-2)
    sc2 = sc.copy()
    sc2[0, 5, d:] = 100.0
    ks, ss = CO.new_state(b, ratio, d, True)
    out2 = O.bf16_to_f32(CO.prefill(kv, sc2, ape, ratio, True, ks, ss))
    assert np.allclose(out2[0, 1], kv[0, 5, d:], rtol=1e-2)
