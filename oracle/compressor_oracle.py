"""CPU oracle for the KV compressor -- TEST INFRASTRUCTURE ONLY.

Only tests/ import this module, as the checker of the library's compressor.
A numpy restatement (fp32) of Compressor.forward after its projections,
QCAU/QCAU_inference/inference/model.py:415-476 (Deepseek_origin/inference/
model.py:317-376 is the same code):

  prefill   the gated pooling of each complete group, with the overlapping
            window of the ratio-4 compressor (overlap_transform, :406-413),
            and the state left for decode (:422-429)
  decode    one token into the state, pooling at a group boundary and the
            state shift (:441-457)
  finish    the pooled rows' RMSNorm, RoPE and FP8 round trip (or Hadamard +
            FP4 for the indexer's compressor) (:459-470), by the C oracle's
            kv_build and indexer_oracle

The softmax uses numpy's float32 exp, not torch's, so a pooled value may
differ from the reference's by an ulp of fp32 and, rarely, its bf16 rounding
by one ulp; the tests allow that.
"""
from __future__ import annotations

import numpy as np

import indexer_oracle as IO
import oracle as O


def _pool(kvw: np.ndarray, scw: np.ndarray) -> np.ndarray:
    """Softmax over axis -2 (the window) of scw, weighted sum of kvw: fp32,
    max-subtracted, summed in window order."""
    m = scw.max(axis=-2, keepdims=True)
    e = np.exp((scw - m).astype(np.float32)).astype(np.float32)
    s = np.zeros(e.shape[:-2] + e.shape[-1:], dtype=np.float32)
    for j in range(e.shape[-2]):
        s = (s + e[..., j, :]).astype(np.float32)
    acc = np.zeros_like(s)
    for j in range(e.shape[-2]):
        acc = (acc + kvw[..., j, :] * (e[..., j, :] / s)).astype(np.float32)
    return acc


def new_state(bsz: int, ratio: int, d: int, overlap: bool):
    coff = 2 if overlap else 1
    kv = np.zeros((bsz, coff * ratio, coff * d), dtype=np.float32)
    sc = np.full_like(kv, -np.inf)
    return kv, sc


def prefill(kv, score, ape, ratio: int, overlap: bool, kv_state, score_state):
    """model.py:415-440 -> pooled [b, s // ratio, d] bf16 bits; the states are
    updated in place."""
    b, s, cw = kv.shape
    d = cw // 2 if overlap else cw
    rem = s % ratio
    cutoff = s - rem
    off = ratio if overlap else 0
    if overlap and cutoff >= ratio:
        kv_state[:b, :ratio] = kv[:, cutoff - ratio:cutoff]
        score_state[:b, :ratio] = score[:, cutoff - ratio:cutoff] + ape
    if rem > 0:
        kv_state[:b, off:off + rem] = kv[:, cutoff:]
        score_state[:b, off:off + rem] = score[:, cutoff:] + ape[:rem]
    n = cutoff // ratio
    k = kv[:, :cutoff].reshape(b, n, ratio, cw)
    sc = (score[:, :cutoff].reshape(b, n, ratio, cw) + ape).astype(np.float32)
    if overlap:
        kw = np.zeros((b, n, 2 * ratio, d), dtype=np.float32)
        sw = np.full((b, n, 2 * ratio, d), -np.inf, dtype=np.float32)
        kw[:, :, ratio:] = k[..., d:]
        sw[:, :, ratio:] = sc[..., d:]
        kw[:, 1:, :ratio] = k[:, :-1, :, :d]
        sw[:, 1:, :ratio] = sc[:, :-1, :, :d]
        k, sc = kw, sw
    return O.f32_to_bf16(_pool(k, sc))


def decode(kv, score, ape, ratio: int, overlap: bool, kv_state, score_state, start_pos: int):
    """model.py:441-457 for one token -> pooled [b, 1, d] bf16 bits, or None
    off a group boundary; the states are updated in place."""
    b, _, cw = kv.shape
    d = cw // 2 if overlap else cw
    p = start_pos % ratio
    sc = score[:, 0] + ape[p]
    slot = ratio + p if overlap else p
    kv_state[:b, slot] = kv[:, 0]
    score_state[:b, slot] = sc
    if (start_pos + 1) % ratio:
        return None
    if overlap:
        kw = np.concatenate([kv_state[:b, :ratio, :d], kv_state[:b, ratio:, d:]], axis=1)
        sw = np.concatenate([score_state[:b, :ratio, :d], score_state[:b, ratio:, d:]], axis=1)
        out = _pool(kw, sw)
        kv_state[:b, :ratio] = kv_state[:b, ratio:]
        score_state[:b, :ratio] = score_state[:b, ratio:]
    else:
        out = _pool(kv_state[:b], score_state[:b])
    return O.f32_to_bf16(out[:, None])


def finish(pooled_bf16, norm_weight, freqs, positions, rotate: bool, eps: float = 1e-6,
           rope_dim: int = 64):
    """model.py:459-470 on pooled rows [rows, d]: RMSNorm, RoPE at the given
    positions (freqs [npos, rope_dim / 2, 2]), then the FP8 round trip of the
    non-rope values (UE8M0, block 64) or the Hadamard rotation + FP4."""
    rows = np.ascontiguousarray(pooled_bf16.reshape(-1, pooled_bf16.shape[-1]))
    d = rows.shape[-1]
    quant = 0 if rotate else d - rope_dim
    y = O.kv_build(rows, np.ascontiguousarray(norm_weight, dtype=np.float32), d, eps,
                   np.ascontiguousarray(freqs, dtype=np.float32),
                   np.ascontiguousarray(positions, dtype=np.int32), rope_dim, quant, True)
    if rotate:
        y = IO.fp4_quant(IO.hadamard_rotate(y))
    return y
