"""CPU oracle for the index-list producers -- TEST INFRASTRUCTURE ONLY.

Only tests/ import this module, as the checker of the library's indexer
kernels.  numpy restatements (bf16 as uint16 bit patterns), each citing the
reference lines it follows (QCAU/QCAU_inference/inference/model.py unless
another file is named):

  hadamard_rotate   rotate_activation's own fallback, model.py:302-323
  fp4_quant         fp4_act_quant(x, 32, inplace=True), Deepseek_origin/
                    inference/kernel.py:128-200 (fast_round_scale :22-37)
  raw_scores        the bf16 einsum "bshd,btd->bsht", model.py:518
  index_scores      (relu(raw) * w).sum(heads) in bf16 tensors, model.py:519
  topk              index_score.topk(k) under the prefill mask, model.py:522-533
  window_topk_idxs  get_window_topk_idxs, model.py:326-357
  compress_topk_idxs get_compress_topk_idxs, model.py:359-376
  index_lists       their concatenation in Attention.forward, model.py:614-624

The Walsh-Hadamard transform is the third-party fast_hadamard_transform
(Dao-AILab, not vendored with the reference and not installed here); the
reference's model.py carries its own fp32 restatement, used whenever the
package is absent, and that is what hadamard_rotate follows.  Its parity is
pinned against that code (tests/golden/indexer.npz).  The CPU fallback of
fp4_act_quant (kernel_fallback.py:116-132) does not round to FP4 at all, so
fp4_quant follows the GPU kernel's source instead; that stage is pinned by
this restatement only.
"""
from __future__ import annotations

import numpy as np

from oracle import bf16_to_f32, f32_to_bf16


def hadamard_rotate(x_bf16: np.ndarray) -> np.ndarray:
    """model.py:302-323: fp32 butterflies in Sylvester order (span 1, 2, 4 ..:
    the first half of each 2*span block becomes left + right, the second
    left - right), times fp32(n^-1/2), rounded to bf16."""
    n = x_bf16.shape[-1]
    y = bf16_to_f32(x_bf16).reshape(-1, n).astype(np.float32)
    span = 1
    while span < n:
        y = y.reshape(-1, n // (2 * span), 2 * span)
        left, right = y[..., :span], y[..., span:]
        y = np.concatenate([left + right, left - right], axis=-1).reshape(-1, n)
        span *= 2
    y = y * np.float32(n ** -0.5)
    return f32_to_bf16(y.reshape(x_bf16.shape))


_E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def _e2m1_round(q: np.ndarray) -> np.ndarray:
    """Nearest FP4 e2m1 value of |q| <= 6, ties to the even code (the
    hardware's cvt.rn to e2m1 that the TileLang cast lowers to)."""
    a = np.abs(q)
    d = np.abs(a[..., None] - _E2M1)                     # distance to each code
    best = d.min(axis=-1, keepdims=True)
    cand = d == best                                     # one code, or two on a tie
    codes = np.arange(8)
    # among the nearest codes take the even one (a tie is always one odd, one even)
    pick = np.where(cand & (codes % 2 == 0), codes, 99).min(axis=-1)
    single = np.where(cand.sum(-1) == 1, np.argmax(cand, axis=-1), pick)
    return np.copysign(_E2M1[single], q).astype(np.float32)


def fp4_quant(x_bf16: np.ndarray, block: int = 32) -> np.ndarray:
    """kernel.py:128-200 with inplace=True: per 1 x block values,
    amax = max(|x|, 6 * 2^-126); s = 2^ceil(log2(fp32(amax * fp32(1/6))))
    by the exponent bits; y = bf16(e2m1(clamp(x / s, -6, 6)) * s)."""
    shp = x_bf16.shape
    x = bf16_to_f32(x_bf16).reshape(-1, block)
    amax = np.maximum(np.abs(x).max(axis=1), np.float32(6 * 2.0 ** -126)).astype(np.float32)
    r = (amax * np.float32(1.0 / 6.0)).astype(np.float32)
    bits = r.view(np.uint32)
    e = ((bits >> 23) & 0xFF).astype(np.int64) - 127 + ((bits & 0x7FFFFF) != 0)
    s = ((e + 127).astype(np.uint32) << 23).view(np.float32)
    q = np.clip(x / s[:, None], -6.0, 6.0).astype(np.float32)
    y = (_e2m1_round(q) * s[:, None]).astype(np.float32)
    return f32_to_bf16(y).reshape(shp)


def raw_scores(q_bf16: np.ndarray, kv_bf16: np.ndarray) -> np.ndarray:
    """model.py:518: raw[b, s, h, t] = bf16(q[b, s, h, :] . kv[b, t, :]), the
    dot product exact (float64 here) and rounded once; a GPU or CPU einsum
    rounds its fp32 partial sums, so it may differ by one bf16 ulp."""
    q = bf16_to_f32(q_bf16).astype(np.float64)
    k = bf16_to_f32(kv_bf16).astype(np.float64)
    r = np.einsum("bshd,btd->bsht", q, k, optimize=True)
    return f32_to_bf16(r.astype(np.float32))


def index_scores(raw_bf16: np.ndarray, w_bf16: np.ndarray) -> np.ndarray:
    """model.py:519 on bf16 tensors: each relu(raw) * w rounded to bf16, the
    products summed over the heads in order in fp32, the sum rounded to bf16.
    raw [..., H, T], w [..., H] -> [..., T] fp32 holding bf16 values."""
    raw = np.maximum(bf16_to_f32(raw_bf16), 0).astype(np.float32)
    w = bf16_to_f32(w_bf16).astype(np.float32)
    prod = bf16_to_f32(f32_to_bf16((raw * w[..., None]).astype(np.float32)))
    acc = np.zeros(prod.shape[:-2] + prod.shape[-1:], dtype=np.float32)
    for h in range(prod.shape[-2]):
        acc = (acc + prod[..., h, :]).astype(np.float32)
    return bf16_to_f32(f32_to_bf16(acc))


def topk(score: np.ndarray, k: int, offset: int = 0, seqlen: int | None = None,
         mask_ratio: int = 0) -> np.ndarray:
    """model.py:522-533 for rows score [R, T]: positions >= (row % seqlen + 1)
    // mask_ratio excluded when mask_ratio > 0 (the prefill), -inf never
    taken; the k largest by score descending then index ascending, + offset,
    -1 past the row's candidates."""
    R, T = score.shape
    out = np.full((R, k), -1, dtype=np.int32)
    idx = np.arange(T)
    for r in range(R):
        lim = T if mask_ratio <= 0 else min(T, (r % seqlen + 1) // mask_ratio)
        v = score[r, :lim]
        ok = np.isfinite(v) | (v > 0)                      # +inf counts, -inf does not
        cand = idx[:lim][ok]
        order = np.lexsort((cand, -v[ok].astype(np.float64)))
        sel = cand[order][:k]
        out[r, :len(sel)] = sel + offset
    return out


def window_topk_idxs(window: int, bsz: int, seqlen: int, start_pos: int) -> np.ndarray:
    """model.py:326-357 -> [bsz, seqlen, w] (seqlen 1 at decode)."""
    if start_pos >= window - 1:
        sp = start_pos % window
        m = np.concatenate([np.arange(sp + 1, window), np.arange(0, sp + 1)])[None]
    elif start_pos > 0:
        m = np.full((1, window), -1, dtype=np.int64)
        m[0, :start_pos + 1] = np.arange(start_pos + 1)
    else:
        base = np.arange(seqlen)[:, None]
        m = np.maximum(base - window + 1, 0) + np.arange(min(seqlen, window))
        m = np.where(m > base, -1, m)
    return np.broadcast_to(m, (bsz,) + m.shape).astype(np.int32)


def compress_topk_idxs(ratio: int, bsz: int, seqlen: int, start_pos: int, offset: int) -> np.ndarray:
    """model.py:359-376 -> [bsz, seqlen, w]."""
    if start_pos > 0:
        m = (np.arange((start_pos + 1) // ratio) + offset)[None]
    else:
        m = np.tile(np.arange(seqlen // ratio), (seqlen, 1))
        mask = m >= (np.arange(1, seqlen + 1)[:, None] // ratio)
        m = np.where(mask, -1, m + offset)
    return np.broadcast_to(m, (bsz,) + m.shape).astype(np.int32)


def index_lists(window: int, ratio: int, bsz: int, seqlen: int, start_pos: int, offset: int,
                selected: np.ndarray | None = None) -> np.ndarray:
    """model.py:614-624: the window list, then the indexer's list or the
    compressed positions (ratio 0: the window list alone)."""
    parts = [window_topk_idxs(window, bsz, seqlen, start_pos)]
    if selected is not None:
        parts.append(np.asarray(selected, dtype=np.int32))
    elif ratio:
        parts.append(compress_topk_idxs(ratio, bsz, seqlen, start_pos, offset))
    return np.concatenate(parts, axis=-1).astype(np.int32)
