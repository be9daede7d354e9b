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


def _unfused_step(comp, kv, score, start_pos, state):
    """The same compressor step composed from qcau_compress, kv_build with
    explicit positions and slots, and rotate_fp4: what qcau_compressor_step
    computes on the device in one call."""
    from qcau_b200.cache import kv_build
    from qcau_b200.indexer import rotate_fp4_
    b, s, _ = kv.shape
    ratio, d = comp.ratio, comp.d
    ks, ss = state
    n = s // ratio if start_pos == 0 else int((start_pos + 1) % ratio == 0)
    first = 0 if start_pos == 0 else start_pos // ratio
    pooled = torch.empty(b, max(n, 1), d, device="cuda", dtype=torch.bfloat16)
    _lib.check(_lib.lib().qcau_compress(kv.data_ptr(), score.data_ptr(), comp.ape.data_ptr(),
                                        ks.data_ptr(), ss.data_ptr(), pooled.data_ptr(), b, s, d,
                                        ratio, int(comp.overlap), start_pos,
                                        _lib.stream_ptr(kv.device)), "compress")
    if n == 0:
        return None
    rows_per_seq = comp.kv_cache.size(1)
    i = torch.arange(n, device="cuda", dtype=torch.int32)
    slots = (torch.arange(b, device="cuda", dtype=torch.int32).view(b, 1) * rows_per_seq
             + comp.cache_offset + first + i.view(1, n)).reshape(-1)
    pos = ((first + i) * ratio).repeat(b)
    cache = comp.kv_cache.clone()
    if not comp.rotate:
        out = kv_build(pooled[:, :n].reshape(-1, d), comp.norm_weight, comp.freqs_cis, pos,
                       rope_dim=comp.rd, quant_dims=d - comp.rd, cache=cache, slots=slots)
    else:
        out = kv_build(pooled[:, :n].reshape(-1, d), comp.norm_weight, comp.freqs_cis, pos,
                       rope_dim=comp.rd, quant_dims=0)
        rotate_fp4_(out)
        cache.view(-1, d).index_copy_(0, slots.long(), out)
    return out.view(b, n, d), cache


@pytest.mark.parametrize("d,rotate,b,s,start_pos", [
    (512, False, 4, 1024, 0),      # attention compressor, prefill
    (512, False, 128, 1, 4095),    # decode step closing a group, bench batch
    (512, False, 128, 1, 4093),    # decode step closing none: state only
    (128, True, 8, 512, 0),        # indexer compressor (rotated), prefill
    (128, True, 64, 1, 2047),      # indexer compressor, decode
])
def test_compressor_step_equals_unfused_chain(d, rotate, b, s, start_pos):
    """qcau_compressor_step (one call: pooling, norm, RoPE, FP8 or rotation
    and FP4, cache rows computed on the device) against the chain of the
    separate entry points, bit for bit, cache included."""
    gen = torch.Generator(device="cuda").manual_seed(d + b + s)
    comp = Compressor(d, 4, 64, rotate=rotate, max_batch=b)
    comp.ape.copy_(torch.randn(comp.ape.shape, device="cuda", generator=gen) * 0.1)
    comp.norm_weight.copy_(1 + 0.1 * torch.randn(d, device="cuda", generator=gen))
    comp.kv_cache = torch.zeros(b, 1200, d, dtype=torch.bfloat16, device="cuda")
    comp.cache_offset = 128
    comp.freqs_cis = torch.polar(torch.ones(8192, 32), torch.rand(8192, 32) * 6).cuda()
    comp.kv_state.normal_(generator=gen)
    comp.score_state.normal_(generator=gen)
    kv = torch.randn(b, s, 2 * d, device="cuda", generator=gen)
    sc = torch.randn(b, s, 2 * d, device="cuda", generator=gen)
    state = (comp.kv_state[:b].clone(), comp.score_state[:b].clone())
    want = _unfused_step(comp, kv, sc, start_pos, state)
    got = comp(kv, sc, start_pos)
    torch.cuda.synchronize()
    assert torch.equal(comp.kv_state[:b], state[0]) and torch.equal(comp.score_state[:b], state[1])
    if want is None:
        assert got is None
    else:
        assert torch.equal(got, want[0])
        assert torch.equal(comp.kv_cache, want[1])
    assert _lib.device_error() == 0
