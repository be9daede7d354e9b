"""Host-side logic of the KV build and caches, and the golden wire format,
checked without a GPU:

  * window_slots places tokens where the reference's window ring does
    (Deepseek_origin/inference/model.py:517-533, restated below);
  * PagedKVCache hands out and takes back pages, and its block tables and
    lengths describe the rows it returned;
  * the golden-vector reader and writer round-trip every format, and read
    the reference's own case files into the committed fixtures;
  * the oracle's KV build matches the reference's own computation
    (tests/golden/kv_build.npz, made by make_golden.py from model.py and
    kernel_fallback.py).
"""
import os
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from qcau_b200 import golden_io
from qcau_b200.cache import PagedKVCache, window_slots

GOLDEN = Path(__file__).resolve().parent / "golden"


def _reference_ring(bsz, seqlen, start_pos, win, tokens):
    """model.py:517-533 on a [bsz, win] ring of token ids (-1 = empty)."""
    ring = np.full((bsz, win), -1, dtype=np.int64)
    kv = np.asarray(tokens)
    if start_pos == 0:
        if seqlen <= win:
            ring[:, :seqlen] = kv
        else:
            cutoff = seqlen % win
            last = kv[:, -win:]
            ring[:, cutoff:win], ring[:, :cutoff] = last[:, :win - cutoff], last[:, win - cutoff:]
    else:
        ring[:, start_pos % win] = kv[:, 0]
    return ring


@pytest.mark.parametrize("seqlen,start_pos,win", [(5, 0, 8), (8, 0, 8), (21, 0, 8), (1, 7, 8),
                                                  (1, 8, 8), (1, 131, 128), (300, 0, 128)])
def test_window_slots_match_reference_ring(seqlen, start_pos, win):
    bsz = 3
    ids = np.arange(bsz * seqlen).reshape(bsz, seqlen)
    ref = _reference_ring(bsz, seqlen, start_pos, win, ids)
    ring_rows = win + 5  # ring rows per sequence (the compressed part follows in the model)
    slots = window_slots(bsz, seqlen, start_pos, win, ring_rows, "cpu").numpy()
    got = np.full((bsz * ring_rows,), -1, dtype=np.int64)
    for tok, s in zip(ids.reshape(-1), slots):
        if s >= 0:
            got[s] = tok
    got = got.reshape(bsz, ring_rows)[:, :win]
    if start_pos > 0:  # decode writes one slot; the rest of the ring is older state
        mask = ref >= 0
        assert np.array_equal(got[mask], ref[mask])
    else:
        assert np.array_equal(got, ref)


def test_paged_cache_allocation_and_rows():
    c = PagedKVCache(num_pages=10, max_seqs=3, max_pages=4, width=64, page_size=4, device="cpu")
    rows = c.append([0, 1], [6, 3]).tolist()
    assert c.free_pages == 10 - 3
    t = c.block_table
    assert rows[:6] == [int(t[0, p // 4]) * 4 + p % 4 for p in range(6)]
    assert rows[6:] == [int(t[1, p // 4]) * 4 + p % 4 for p in range(3)]
    assert c.seqlens.tolist() == [6, 3, 0]
    assert c.positions([0, 1], [6, 3]).tolist() == list(range(6)) + list(range(3))
    more = c.append([1], [2]).tolist()
    assert more == [int(c.block_table[1, p // 4]) * 4 + p % 4 for p in range(3, 5)]
    assert c.free_pages == 10 - 4
    used = set(int(x) for x in c.block_table[0, :2]) | set(int(x) for x in c.block_table[1, :2])
    assert len(used) == 4  # distinct pages
    c.release(0)
    assert c.free_pages == 10 - 2 and c.seqlens.tolist() == [0, 5, 0]
    with pytest.raises(ValueError):
        c.append([2], [17])  # 5 pages > max_pages
    c.append([0, 2], [16, 12])  # 4 + 3 of the 8 free pages
    assert c.free_pages == 1
    with pytest.raises(MemoryError):
        c.append([1], [8])  # 13 tokens: 2 more pages, 1 free


@pytest.mark.parametrize("kind,values", [
    ("bf16", np.array([[0x3f80, 0xbf80, 0x7f80], [0x0001, 0x8000, 0xffff]], dtype=np.uint16)),
    ("fp8_e4m3", np.array([0x00, 0x7e, 0xfe, 0x38], dtype=np.uint8)),
    ("e8m0", np.array([[0x7f, 0x80], [0x01, 0xfe]], dtype=np.uint8)),
    ("fp32", np.array([1.5, -2.25e-30, 3.4028235e38], dtype=np.float32)),
    ("int", np.array([[0, -1], [131071, 7]], dtype=np.int64)),
])
def test_golden_io_round_trip(tmp_path, kind, values):
    golden_io.write_tensor(tmp_path, "t", values, kind)
    assert golden_io.tensor_kind(tmp_path, "t") == kind
    back = golden_io.read_tensor(tmp_path, "t")
    assert back.shape == values.shape
    if kind == "fp32":
        assert np.array_equal(back.view(np.uint32), values.view(np.uint32))
    else:
        assert np.array_equal(back, values)


def _reference_vectors():
    root = Path(os.environ.get("QCAU_REFERENCE_ROOT") or
                Path(__file__).resolve().parents[2] / "reference")
    return root / "QCAU/QCAU_inference/framework/test_vectors"


@pytest.mark.skipif(not _reference_vectors().exists(), reason="reference checkout not present")
def test_golden_io_reads_reference_cases():
    g = np.load(GOLDEN / "act_quant_goldens.npz")
    a = np.load(GOLDEN / "attn_goldens.npz")
    for name in list(g["cases"])[:6]:
        case = golden_io.read_case(_reference_vectors() / name)
        S = case["metadata"]["seq_len"]
        assert np.array_equal(case["c_q"].reshape(S, -1), g[f"{name}/c_q"])
        assert np.array_equal(case["linear_x_after_act_quant"].reshape(S, -1), g[f"{name}/x"])
        assert np.array_equal(case["linear_s_after_act_quant"].reshape(S, -1), g[f"{name}/s"])
        assert np.array_equal(case["kv_after_rope_quant_compress"], a[f"{name}/kv"])
        assert np.array_equal(case["topk_idxs"].astype(np.int32), a[f"{name}/idx"])


def test_oracle_kv_build_matches_reference_code():
    """The whole KV build is bit-exact with the reference's own code; the
    norm + RoPE stage alone may differ by an ulp where torch sums the squares
    in another order (the FP8 round trip absorbs it)."""
    g = np.load(GOLDEN / "kv_build.npz")
    rows = g["x"].shape[0]
    pos = np.arange(rows, dtype=np.int32)  # row r of the fixture's freqs is its position's
    full = O.kv_build(g["x"], g["weight"], 512, 1e-6, g["freqs"], pos, 64, 448, True)
    assert np.array_equal(full, g["kv"])
    nr = O.kv_build(g["x"], g["weight"], 512, 1e-6, g["freqs"], pos, 64, 0, True)
    diff = np.abs(O.bf16_to_f32(nr) - O.bf16_to_f32(g["after_norm_rope"]))
    ulp = np.spacing(np.abs(O.bf16_to_f32(g["after_norm_rope"]))) * 65536
    assert np.all(diff <= ulp) and int(np.sum(diff > 0)) <= nr.size // 1000
    # the FP8 stage alone, from the reference's own normalised rows
    q = O.kv_build(g["after_norm_rope"], None, 0, 1e-6, g["freqs"], pos, 0, 448, True)
    assert np.array_equal(q, g["kv"])
