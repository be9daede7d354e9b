"""C ABI checks that need no GPU: the library loads, exports exactly what the
header declares, and rejects bad arguments with the reference's error kinds
before touching the device.

The pointer arguments are real host buffers.  With a CUDA device present
the argument checks are left to the GPU tests, which pass real device
buffers: a call that reached a launch here would hand a kernel host memory.
"""
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from qcau_b200 import _lib

# eight 1 MiB host buffers standing for the calls' tensors
_HOST = [np.zeros(1 << 20, dtype=np.uint8) for _ in range(8)]
P = [int(a.ctypes.data) for a in _HOST]

no_device = pytest.mark.skipif(torch.cuda.is_available(),
                               reason="argument checks with host buffers run without a device")

HEADER = Path(__file__).resolve().parent.parent / "include" / "qcau_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qcau_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"{n} declared in qcau_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_empty_error():
    assert _lib.lib().qcau_version() == 100


def _expect(rc, exc):
    with pytest.raises(exc):
        _lib.check(rc, "call")


@no_device
def test_act_quant_rejects_bad_block():
    L = _lib.lib()
    rc = L.qcau_act_quant(P[0], P[1], P[2], 4, 100, 128, 0, 0, 0, None)
    _expect(rc, ValueError)
    assert b"divisible" in L.qcau_last_error()
    rc = L.qcau_act_quant(P[0], P[1], P[2], 4, 128, 96, 0, 0, 0, None)
    _expect(rc, ValueError)
    rc = L.qcau_act_quant(P[0], P[1], P[2], 4, 128, 128, 0, 1, 0, None)  # e8m0 needs round_scale
    _expect(rc, ValueError)


@no_device
def test_fp8_gemm_rejects_bad_k():
    L = _lib.lib()
    rc = L.qcau_fp8_gemm(P[0], P[1], P[2], P[3], P[4], 4, 128, 100, 0, 0, None)
    _expect(rc, ValueError)
    assert b"multiple of 128" in L.qcau_last_error()


@no_device
def test_attention_widths_unsupported_raise_not_implemented():
    L = _lib.lib()
    rc = L.qcau_sparse_attn(P[0], P[1], None, P[2], P[3], 1, 1, 4, 8, 8, 8, 4, 2, 1.0, 0, None, 0,
                            0, 0, None)
    _expect(rc, NotImplementedError)


@no_device
def test_sparse_attn_rejects_empty_kv():
    L = _lib.lib()
    rc = L.qcau_sparse_attn(P[0], P[1], None, P[2], P[3], 1, 1, 4, 512, 512, 512, 0, 2, 1.0, 0,
                            None, 0, 0, 0, None)
    _expect(rc, ValueError)
    assert b"at least one latent row" in L.qcau_last_error()


def _plan_slots(rows, max_len, rule, pairs=74):
    """Partial slots of the balanced decode plan (128 heads): the most pieces
    any row's 128-token tiles are cut into by 74 equal pair ranges, or 0 when
    a pair would get fewer than 32 tiles, or fewer than 64 where the split
    count `rule` is 1 (the split count runs then)."""
    nt = (max_len + 127) // 128
    g = rows * nt
    pairs = max(1, min(pairs, g // 4))
    if g < 32 * pairs or (rule <= 1 and g < 64 * pairs):
        return 0
    return max(((i + 1) * nt * pairs - 1) // g - ((i * nt + 1) * pairs - 1) // g + 1
               for i in range(rows))


def test_decode_split_counts_measured_best():
    """The two-CTA kernel's split counts at the shapes they were measured on
    (128 heads, 512-wide values, B200), read back from the workspace the
    decode entry asks for (fp32 O and (max, sum) partials per slot): 128
    sequences x 32K in 4 splits, 64 x 32K and 128 x 4K unsplit (the faster
    choices over 8 and 4 splits), 16 x 32K in 4; decode rows also get the
    balanced plan's slots where it applies (the larger of the two counts)."""
    L = _lib.lib()

    def ws(b, splits):
        return b * splits * 128 * (512 + 2) * 4 if splits > 1 else 0

    for b, ctx, rule in ((128, 32768, 4), (64, 32768, 1), (128, 4096, 1), (16, 32768, 4)):
        assert L.qcau_decode_attn_workspace_size(b, 128, 512, ctx) == \
            ws(b, max(rule, _plan_slots(b, ctx, rule))), (b, ctx)
    assert _plan_slots(128, 32768, 4) == 2 and _plan_slots(128, 4096, 1) == 0


@no_device
def test_workspace_errors_before_launch():
    L = _lib.lib()
    need = L.qcau_decode_attn_workspace_size(128, 128, 512, 32768)
    assert need > 0
    rc = L.qcau_decode_attn_paged(P[0], P[1], P[2], P[3], None, P[4], 128, 128, 576, 512, 576, 64,
                                  512, 65536, 32768, 0.07, P[5], need - 1, None)
    _expect(rc, ValueError)
    assert b"workspace too small" in L.qcau_last_error()


@no_device
def test_forward_freqs_coverage_error():
    L = _lib.lib()
    rc = L.qcau_forward(P[0], P[1], P[2], 0, 1, None, P[3], P[4], P[5], P[6], P[7], 1, 4, 2, 512,
                        1024, 8, 8, 64, 3, 0, 1e-6, 0.04, P[0], 1 << 20, None)
    _expect(rc, ValueError)
    assert b"freqs_cis" in L.qcau_last_error()


@no_device
def test_mla_decode_rejects_bad_layout():
    L = _lib.lib()
    d = _lib.MlaDims(batch=4, n_heads=16, dc=1536, d_nope=64, d_rope=64, kv_lora=512, d_v=128,
                     dim=7168, page_size=64, max_pages=4, num_pages=16, max_seqlen=256,
                     npos=512, softmax_scale=0.07, w_scale_dtype=0, act_round_scale=0,
                     out_dtype=0)
    rc = L.qcau_mla_decode(d, *(P + P[:4]), P[4], 1 << 20, None)
    _expect(rc, ValueError)
