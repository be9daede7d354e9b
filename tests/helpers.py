"""Shared helpers of the parity tests: bit-pattern conversions and the
tolerance checks used throughout.

Tolerances (stated once, used by every floating-point parity test):
  * attention / QCAU / decode-layer outputs: cosine >= 0.999 and
    max |diff| <= 2e-2 * RMS(reference)   (the bar stated for this path).
    With strict=False an element may also differ by one bf16 ulp of its
    reference value: for peaked attention an output element can be ~10x the
    RMS, and one bf16 rounding step of it (2^-8 relative) then exceeds
    2e-2 * RMS even though both sides are correctly rounded.  The number of
    elements that pass only through that allowance is recorded
    (ULP_ONLY_LOG) and returned; strict=True allows none;
  * GEMM-only outputs additionally: >= 99% of bf16 values within one ulp.
Integer / byte outputs (FP8 codes, E8M0 scales) must be bit-exact.
"""
from __future__ import annotations

import numpy as np
import torch

COS_MIN = 0.999
MAXABS_RMS = 2e-2


def t_bf16(u16: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).to(device)


def t_u8(u8: np.ndarray, dtype=torch.float8_e4m3fn, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u8, dtype=np.uint8)).view(dtype).to(device)


def n_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def n_u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def cosine(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb + 1e-300))


# (what, elements within 1 bf16 ulp but beyond 2e-2 * RMS, total elements) of
# every non-strict comparison that needed the allowance
ULP_ONLY_LOG: list = []


def assert_close_attn(got, ref, what="", strict=False):
    """The path's floating-point bar: cosine >= 0.999, max-abs <= 2e-2 * RMS.

    Returns (cosine, max |diff|, n_ulp_only): the elements that pass only by
    the one-ulp allowance (always 0 with strict=True)."""
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    c = cosine(got, ref)
    diff = np.abs(got - ref)
    m = float(diff.max()) if got.size else 0.0
    assert c >= COS_MIN, f"{what}: cosine {c}"
    bar = np.float32(MAXABS_RMS * max(rms, 1e-6))
    beyond = diff > bar
    if strict:
        bad = int(np.sum(beyond))
        assert bad == 0, (f"{what}: {bad} elements beyond 2e-2*rms; max|diff| {m}, "
                          f"rms {rms}, max|diff|/rms {m / max(rms, 1e-30):.4f}")
        return c, m, 0
    ulp = np.spacing(np.abs(ref).astype(np.float32)) * np.float32(65536.0)  # bf16 ulp
    bad = int(np.sum(beyond & (diff > ulp)))
    assert bad == 0, (f"{what}: {bad} elements beyond max(2e-2*rms, 1 bf16 ulp); "
                      f"max|diff| {m}, rms {rms}")
    n_ulp = int(np.sum(beyond))
    if n_ulp:
        ULP_ONLY_LOG.append((what, n_ulp, int(got.size)))
    return c, m, n_ulp
