"""CPU oracle for the QCAU path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker.  The product library (qcau_b200) never
imports it and has no CPU fallback.

It wraps two native programs built by oracle/Makefile:
  * _build/libqcau_oracle.so -- the C restatement in qcau_oracle.c (each
    function there cites the reference lines it follows);
  * _ref/qcau_ref            -- the reference's own qcau_c C++ port compiled
    from its sources, driven through raw binary files.

Arrays cross the boundary as numpy arrays of raw bit patterns: bf16 as
uint16, e4m3 / e8m0 as uint8.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libqcau_oracle.so"
REF_BIN = HERE / "_ref" / "qcau_ref"

_lib = None


def build() -> None:
    """Build the C oracle (and the qcau_c driver when its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        I = ctypes.c_int64
        F = ctypes.c_float
        i32 = ctypes.c_int
        _lib.orc_act_quant.argtypes = [P, I, I, i32, i32, P, P]
        _lib.orc_act_quant_inplace.argtypes = [P, I, I, i32, i32]
        _lib.orc_fp8_gemm.argtypes = [P, P, P, P, I, I, I, P]
        _lib.orc_head_rms_norm.argtypes = [P, I, I, P, I, F]
        _lib.orc_rope.argtypes = [P, I, I, I, I, P, I, I, I, i32]
        _lib.orc_sparse_attn.argtypes = [P, P, P, P, I, I, I, I, I, I, I, I, F, P]
        _lib.orc_paged_decode_attn.argtypes = [P, P, P, P, P, I, I, I, I, I, I, I, F, P, P]
        _lib.orc_mla_absorb.argtypes = [P, I, P, I, I, I, I, I, P, I]
        _lib.orc_mla_vup.argtypes = [P, P, I, I, I, I, I, P]
        _lib.orc_kv_build.argtypes = [P, I, I, P, I, F, P, P, I, I, i32]
        _lib.orc_grouped_proj.argtypes = [P, P, I, I, I, I, P]
        _lib.orc_f32_to_bf16_n.argtypes = [P, P, I]
        _lib.orc_f32_to_e4m3_n.argtypes = [P, P, I]
        _lib.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        _lib.orc_e4m3_to_f32.restype = ctypes.c_float
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- formats

def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_n(_p(x), _p(out), x.size)
    return out


_E4M3_LUT = None


def e4m3_to_f32(u8: np.ndarray) -> np.ndarray:
    global _E4M3_LUT
    if _E4M3_LUT is None:
        _E4M3_LUT = np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return _E4M3_LUT[np.asarray(u8, dtype=np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().orc_f32_to_e4m3_n(_p(x), _p(out), x.size)
    return out


def e8m0_to_f32(u8: np.ndarray) -> np.ndarray:
    e = np.asarray(u8, dtype=np.int32)
    return np.ldexp(np.float32(1.0), e - 127).astype(np.float32)


def f32_pow2_to_e8m0(s: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(s, dtype=np.float32).view(np.uint32)
    return ((bits >> 23) & 0xFF).astype(np.uint8)


# ---------------------------------------------------------------- kernels

def act_quant(x_bf16: np.ndarray, block: int = 128, round_scale: bool = False):
    """kernel.py:105-125 act_quant -> (e4m3 codes uint8, fp32 scales)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    n = x.shape[-1]
    m = x.size // n
    y = np.empty(x.shape, dtype=np.uint8)
    s = np.empty(x.shape[:-1] + (n // block,), dtype=np.float32)
    lib().orc_act_quant(_p(x), m, n, block, int(round_scale), _p(y), _p(s))
    return y, s


def act_quant_inplace(x_bf16: np.ndarray, block: int, round_scale: bool) -> np.ndarray:
    x = np.array(x_bf16, dtype=np.uint16, copy=True, order="C")
    n = x.shape[-1]
    lib().orc_act_quant_inplace(_p(x), x.size // n, n, block, int(round_scale))
    return x


def kv_build(x_bf16: np.ndarray, weight: np.ndarray | None, norm_dim: int, eps: float,
             freqs: np.ndarray, positions: np.ndarray, rope_dim: int, quant_dims: int,
             round_scale: bool) -> np.ndarray:
    """model.py:502-506 on rows [rows, d] bf16: RMSNorm, RoPE, FP8 round trip."""
    x = np.array(x_bf16, dtype=np.uint16, copy=True, order="C")
    d = x.shape[-1]
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    f = np.ascontiguousarray(freqs, dtype=np.float32)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    lib().orc_kv_build(_p(x), x.size // d, d, _p(w), norm_dim, float(eps), _p(f),
                       _p(pos), rope_dim, quant_dims, int(round_scale))
    return x


def grouped_proj(o_bf16: np.ndarray, w_bf16: np.ndarray) -> np.ndarray:
    """model.py:537-541 einsum bsgd,grd->bsgr: o [rows, G, gd], w [G, R, gd]
    -> [rows, G, R] bf16 (fp32 sums)."""
    o = np.ascontiguousarray(o_bf16, dtype=np.uint16)
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    G, R, gd = w.shape
    rows = o.size // (G * gd)
    h = np.empty((rows, G, R), dtype=np.uint16)
    lib().orc_grouped_proj(_p(o), _p(w), rows, G, gd, R, _p(h))
    return h


def fp8_gemm(a_u8, a_s, b_u8, b_s) -> np.ndarray:
    """kernel.py:257-273 fp8_gemm with two-level accumulation -> fp32 [M,N]."""
    a = np.ascontiguousarray(a_u8, dtype=np.uint8)
    b = np.ascontiguousarray(b_u8, dtype=np.uint8)
    k = a.shape[-1]
    m = a.size // k
    n = b.shape[0]
    sa = np.ascontiguousarray(a_s, dtype=np.float32)
    sb = np.ascontiguousarray(b_s, dtype=np.float32)
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_fp8_gemm(_p(a), _p(sa), _p(b), _p(sb), m, n, k, _p(c))
    return c.reshape(a.shape[:-1] + (n,))


def head_rms_norm(x_bf16: np.ndarray, eps: float, gamma_bf16: np.ndarray | None = None) -> np.ndarray:
    """model.py:498 / QCAU.py:16-27 per-head RMSNorm in bf16 arithmetic."""
    x = np.array(x_bf16, dtype=np.uint16, copy=True, order="C")
    d = x.shape[-1]
    h = x.shape[-2]
    g = None if gamma_bf16 is None else np.ascontiguousarray(gamma_bf16, dtype=np.uint16)
    lib().orc_head_rms_norm(_p(x), x.size // d, d, _p(g), h, float(eps))
    return x


def rope(x_bf16: np.ndarray, freqs: np.ndarray, rope_dim: int, pos0: int = 0,
         inverse: bool = False) -> np.ndarray:
    """model.py:231-243 RoPE on the last rope_dim values of [B,S,H,D] rows.

    freqs: [P, rope_dim/2, 2] fp32 (re, im); row (b,s,h) uses freqs[pos0+s].
    """
    x = np.array(x_bf16, dtype=np.uint16, copy=True, order="C")
    B, S, H, D = x.shape
    f = np.ascontiguousarray(freqs, dtype=np.float32)
    lib().orc_rope(_p(x), B * S * H, D, D, rope_dim, _p(f), H, S, pos0, int(inverse))
    return x


def sparse_attn(q_bf16, kv_bf16, sink, idx, scale: float, d_v: int | None = None) -> np.ndarray:
    """kernel.py:276-368 sparse_attn (bf16 P, sink, -1 masking) -> fp32 out.

    q [B,S,H,Dqk]; kv [B,N,Dkv]; idx [B,S,K] int32; V = kv[..., :d_v].
    """
    q = np.ascontiguousarray(q_bf16, dtype=np.uint16)
    kv = np.ascontiguousarray(kv_bf16, dtype=np.uint16)
    ix = np.ascontiguousarray(idx, dtype=np.int32)
    sk = None if sink is None else np.ascontiguousarray(sink, dtype=np.float32)
    B, S, H, Dqk = q.shape
    N, Dkv = kv.shape[1], kv.shape[2]
    dv = Dqk if d_v is None else d_v
    out = np.empty((B, S, H, dv), dtype=np.float32)
    lib().orc_sparse_attn(_p(q), _p(kv), _p(sk), _p(ix), B, S, H, Dqk, dv, Dkv, N,
                          ix.shape[-1], float(scale), _p(out))
    return out


def paged_decode_attn(q_bf16, cache_bf16, table, seqlens, sink, scale: float, d_v: int,
                      want_lse: bool = False):
    """Dense decode over a paged cache (one query token per sequence).

    q [B,H,Dqk]; cache [pages, page, Dkv]; table [B, max_pages]; seqlens [B].
    """
    q = np.ascontiguousarray(q_bf16, dtype=np.uint16)
    c = np.ascontiguousarray(cache_bf16, dtype=np.uint16)
    t = np.ascontiguousarray(table, dtype=np.int32)
    sl = np.ascontiguousarray(seqlens, dtype=np.int32)
    sk = None if sink is None else np.ascontiguousarray(sink, dtype=np.float32)
    B, H, Dqk = q.shape
    out = np.empty((B, H, d_v), dtype=np.float32)
    lse = np.empty((B, H), dtype=np.float32) if want_lse else None
    lib().orc_paged_decode_attn(_p(q), _p(c), _p(t), _p(sl), _p(sk), B, H, Dqk, d_v,
                                c.shape[-1], c.shape[1], t.shape[1], float(scale),
                                _p(out), _p(lse))
    return (out, lse) if want_lse else out


def mla_absorb(q_bf16, wkv_bf16, d_nope: int, d_v: int) -> np.ndarray:
    """Absorbed query: q[b,h,:d_nope] . W_UK[h] -> [B,H,kv_lora] bf16."""
    q = np.ascontiguousarray(q_bf16, dtype=np.uint16)
    w = np.ascontiguousarray(wkv_bf16, dtype=np.uint16)
    B, H, dq = q.shape
    kv_lora = w.shape[1]
    out = np.empty((B, H, kv_lora), dtype=np.uint16)
    lib().orc_mla_absorb(_p(q), dq, _p(w), B, H, d_nope, d_v, kv_lora, _p(out), kv_lora)
    return out


def mla_vup(o_lat_bf16, wkv_bf16, d_nope: int, d_v: int) -> np.ndarray:
    """o_v[b,h,:] = o_lat[b,h,:] . W_UV[h]^T -> [B,H,d_v] bf16."""
    o = np.ascontiguousarray(o_lat_bf16, dtype=np.uint16)
    w = np.ascontiguousarray(wkv_bf16, dtype=np.uint16)
    B, H, kv_lora = o.shape
    out = np.empty((B, H, d_v), dtype=np.uint16)
    lib().orc_mla_vup(_p(o), _p(w), B, H, d_nope, d_v, kv_lora, _p(out))
    return out


# ------------------------------------------------- the reference's own C++

def ref_available() -> bool:
    return REF_BIN.exists()


def ref_sparse_attention(q_bf16, kv_bf16, idx, sink) -> np.ndarray:
    """Run qcau_c sparse_attention (qcau.cpp:169-284) on one batch element.

    q [S,H,C] bf16, kv [N,C] bf16, idx [S,K] int32, sink [H] -> [S,H,C] bf16.
    The reference fixes the softmax scale to 1/sqrt(C).
    """
    S, H, C = q_bf16.shape
    N = kv_bf16.shape[0]
    K = idx.shape[-1]
    with tempfile.TemporaryDirectory() as d:
        np.ascontiguousarray(q_bf16, dtype=np.uint16).tofile(os.path.join(d, "q.bin"))
        np.ascontiguousarray(kv_bf16, dtype=np.uint16).tofile(os.path.join(d, "kv.bin"))
        np.ascontiguousarray(idx, dtype=np.int32).tofile(os.path.join(d, "idx.bin"))
        np.ascontiguousarray(sink, dtype=np.float32).tofile(os.path.join(d, "sink.bin"))
        subprocess.run([str(REF_BIN), "attn", d, str(S), str(H), str(C), str(N), str(K)],
                       check=True)
        return np.fromfile(os.path.join(d, "out.bin"), dtype=np.uint16).reshape(S, H, C)


def ref_quant_gemm(a_f32, sa, w_f32, sw) -> np.ndarray:
    """Run qcau_c quant_gemm (qcau.cpp:30-90): fp8 values held as bf16."""
    S, Dc = a_f32.shape
    N = w_f32.shape[0]
    with tempfile.TemporaryDirectory() as d:
        f32_to_bf16(a_f32).tofile(os.path.join(d, "a.bin"))
        np.ascontiguousarray(sa, dtype=np.float32).tofile(os.path.join(d, "sa.bin"))
        f32_to_bf16(w_f32).tofile(os.path.join(d, "w.bin"))
        np.ascontiguousarray(sw, dtype=np.float32).tofile(os.path.join(d, "sw.bin"))
        subprocess.run([str(REF_BIN), "qgemm", d, str(S), str(Dc), str(N)], check=True)
        return np.fromfile(os.path.join(d, "out.bin"), dtype=np.uint16).reshape(S, N)


def ref_bench_decode(threads: int, seqs: int, heads: int, width: int, ctx: int,
                     dc: int, nq: int, no: int, steps: int = 1, warmup: int = 0) -> dict:
    """Time qcau_c on `seqs` decode tokens (one per sequence) on `threads` cores:
    inputs generated first, then `warmup` untimed and `steps` timed steps."""
    out = subprocess.run([str(REF_BIN), "bench_decode", str(threads), str(seqs), str(heads),
                          str(width), str(ctx), str(dc), str(nq), str(no), str(steps),
                          str(warmup)],
                         check=True, capture_output=True, text=True)
    return json.loads(out.stdout.strip().splitlines()[-1])
