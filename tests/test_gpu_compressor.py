"""GPU parity of the KV compressor (qcau_compress + qcau_kv_build /
qcau_rotate_fp4 through qcau_b200.cache.Compressor) against the reference's
own Compressor.forward (tests/golden/compressor.npz) and the oracle.

Bars: the decode state bit-exact; the compressed rows and the cache equal to
the reference's in >= 99 % of values, each within 2 % of its row's largest
(the softmax exponent is CUDA's expf against torch's, so a pooled value can
round to the neighbouring bf16 before the norm and quantisation).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import indexer_oracle as IO
from helpers import n_bf16
from test_compressor_host import CASES, close_rows, run_oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qcau_b200 import _lib
    from qcau_b200.cache import Compressor

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "compressor.npz")


@pytest.mark.parametrize("name", list(CASES))
def test_compressor_vs_reference_and_oracle(g, name):
    ratio, d, rotate = CASES[name]
    comp = Compressor(d, ratio, rotate=rotate, max_batch=2)
    comp.ape.copy_(torch.from_numpy(g[f"{name}/ape"]))
    comp.norm_weight.copy_(torch.from_numpy(g[f"{name}/norm"]))
    comp.kv_cache = torch.zeros(2, 64 // ratio, d, dtype=torch.bfloat16, device="cuda")
    comp.freqs_cis = torch.view_as_complex(torch.from_numpy(g[f"{name}/freqs"]).contiguous()).cuda()
    oracle = {i: (rows, ks, ss) for i, _, rows, ks, ss in run_oracle(g, name)}
    i = 0
    outs = 0
    while f"{name}/step{i}/meta" in g.files:
        k = f"{name}/step{i}"
        sp, _ = (int(v) for v in g[f"{k}/meta"])
        y = comp(torch.from_numpy(g[f"{k}/kv"]).cuda(), torch.from_numpy(g[f"{k}/score"]).cuda(), sp)
        torch.cuda.synchronize()
        assert (y is not None) == (f"{k}/out" in g.files), k
        if y is not None:
            want = g[f"{k}/out"]
            if rotate:  # kernel_fallback's fp4_act_quant does not round to FP4
                want = IO.fp4_quant(want)
            close_rows(n_bf16(y), want, f"{k} vs reference")
            close_rows(n_bf16(y), oracle[i][0], f"{k} vs oracle")
            outs += 1
        ks = comp.kv_state[:2].cpu().numpy()
        ss = comp.score_state[:2].cpu().numpy()
        assert np.array_equal(ks, oracle[i][1]) and np.array_equal(ss, oracle[i][2]), k
        if f"{k}/kv_state" in g.files:
            assert np.array_equal(ks, g[f"{k}/kv_state"]), k
            assert np.array_equal(ss, g[f"{k}/score_state"]), k
            want_cache = g[f"{k}/cache"]
            got_cache = n_bf16(comp.kv_cache)
            written = np.any(want_cache != 0, axis=-1)
            assert np.array_equal(np.any(got_cache != 0, axis=-1), written), k
            if rotate:
                want_cache = IO.fp4_quant(want_cache)
            close_rows(got_cache[written], want_cache[written], f"{k} cache")
        i += 1
    assert outs >= 2
    assert _lib.device_error() == 0


def test_compressor_rejects_bad_shapes():
    comp = Compressor(512, 4, max_batch=2)
    comp.kv_cache = torch.zeros(2, 16, 512, dtype=torch.bfloat16, device="cuda")
    comp.freqs_cis = torch.ones(64, 32, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError):
        comp(torch.zeros(2, 4, 512, device="cuda"), torch.zeros(2, 4, 512, device="cuda"), 0)
    with pytest.raises(ValueError):
        comp(torch.zeros(2, 2, 1024, device="cuda"), torch.zeros(2, 2, 1024, device="cuda"), 5)
    # a prefill shorter than the ratio compresses nothing but keeps its tokens
    assert comp(torch.ones(2, 3, 1024, device="cuda"), torch.zeros(2, 3, 1024, device="cuda"), 0) is None
    assert bool((comp.kv_state[:2, 4:7] == 1).all())
