"""The reference's own call site, replayed through qcau_b200.kernel on the GPU.

tests/golden/attention_trace.npz holds every call that the reference's
Attention.forward (Deepseek_origin/inference/model.py:484-543; the module
that does `from kernel import ...`, model.py:12) made into its kernel module
during a prefill and two decode steps of a seeded V4-width layer, run on the
CPU with the reference's kernel_fallback as that module (make_golden.py,
attention_trace_fixture).  Each call kept its arguments exactly as the call
site passed them -- positional and keyword layout, dtypes, and views such as
the in-place act_quant(kv[..., :-64], 64, ...) on a strided slice -- and its
results.

Here every call is made again, in order, on qcau_b200.kernel -- the module a
user installs as sys.modules["kernel"] -- with the same arguments on the GPU:

  act_quant          bit-exact with the reference (codes, scales, and for the
                     in-place calls the whole tensor the view belongs to)
  fp8_gemm           the reference's fp32 GEMM within fp32 summation order:
                     >= 99 % of outputs identical, the rest one bf16 ulp
  sparse_attn        the path's bar (cosine >= 0.999, max-abs <= 2e-2 * RMS;
                     elements passing only by the one-ulp allowance are
                     reported); kernel_fallback's sparse_attn keeps P in fp32
                     where the reference's GPU kernel rounds it to bf16
  fp4_act_quant      bit-exact with the oracle's restatement of the GPU
                     kernel (kernel_fallback's version does not round to FP4)
"""
import json
import os
from pathlib import Path

import numpy as np
import pytest
import torch

import indexer_oracle as IO
from helpers import assert_close_attn, cosine, f32, n_bf16

GOLDEN = Path(__file__).resolve().parent / "golden"

_DT = {"bf16": torch.bfloat16, "fp32": torch.float32, "e4m3": torch.float8_e4m3fn,
       "e8m0": torch.float8_e8m0fnu, "int32": torch.int32, "int64": torch.int64}


def _load():
    g = np.load(GOLDEN / "attention_trace.npz")
    return g, json.loads(str(g["calls"]))


def _tensor(g, spec, device):
    a = g[spec["t"]]
    dt = _DT[spec["dtype"]]
    if dt == torch.bfloat16:
        base = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    elif dt in (torch.float8_e4m3fn, torch.float8_e8m0fnu):
        base = torch.from_numpy(a.copy()).view(dt)
    else:
        base = torch.from_numpy(a.copy())
    base = base.reshape(spec["base_size"]).to(device)
    if spec["size"] == spec["base_size"] and spec["offset"] == 0 and base.is_contiguous() \
            and list(base.stride()) == spec["stride"]:
        return base, base
    return torch.as_strided(base, spec["size"], spec["stride"], spec["offset"]), base


def _value(g, spec, device):
    if "t" in spec:
        return _tensor(g, spec, device)[0]
    if "dtype_arg" in spec:
        return _DT[spec["dtype_arg"]]
    if "seq" in spec:
        return tuple(_value(g, s, device) for s in spec["seq"])
    return spec["v"]


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu):
        return t.view(torch.uint8).numpy()
    return t.numpy()


def _ref_bits(g, spec):
    return _bits(_tensor(g, spec, "cpu")[0])


def test_trace_covers_the_call_site():
    _, calls = _load()
    fns = {c["fn"] for c in calls}
    assert {"act_quant", "fp8_gemm", "sparse_attn", "fp4_act_quant"} <= fns
    steps = {c["step"] for c in calls}
    assert steps == {0, 1, 2}
    # the in-place KV round trip on a strided view is among them
    assert any(c["fn"] == "act_quant" and "out_base_after" in c for c in calls)


def test_every_call_binds_to_the_library_signatures():
    import inspect

    from qcau_b200 import kernel

    _, calls = _load()
    for c in calls:
        sig = inspect.signature(getattr(kernel, c["fn"]))
        sig.bind(*[None] * len(c["args"]), **{k: None for k in c["kwargs"]})


@pytest.mark.gpu
def test_replay_reference_attention_calls_through_qcau_kernel():
    from qcau_b200 import _lib, kernel

    g, calls = _load()
    prev = torch.get_default_dtype()
    seen = {}
    try:
        for i, c in enumerate(calls):
            what = f"call {i} {c['fn']} (step {c['step']})"
            torch.set_default_dtype(_DT[c["default_dtype"]])
            args = [_value(g, a, "cuda") for a in c["args"]]
            kwargs = {k: _value(g, v, "cuda") for k, v in c["kwargs"].items()}
            fp4_in = n_bf16(args[0]) if c["fn"] == "fp4_act_quant" else None
            out = getattr(kernel, c["fn"])(*args, **kwargs)
            torch.cuda.synchronize()
            seen[c["fn"]] = seen.get(c["fn"], 0) + 1
            if c["fn"] == "act_quant":
                if "seq" in c["out"]:
                    y, s = out
                    ry, rs = (_ref_bits(g, sp) for sp in c["out"]["seq"])
                    assert np.array_equal(_bits(y), ry), what
                    assert np.array_equal(_bits(s), rs), what
                else:
                    assert np.array_equal(_bits(out), _ref_bits(g, c["out"])), what
                    if "out_base_after" in c:
                        base = out._base if out._base is not None else out
                        assert np.array_equal(_bits(base), _ref_bits(g, c["out_base_after"])), what
            elif c["fn"] == "fp8_gemm":
                got = f32(_bits(out)) if out.dtype == torch.bfloat16 else _bits(out)
                ref = _ref_bits(g, c["out"])
                ref = f32(ref) if out.dtype == torch.bfloat16 else ref
                assert out.dtype == _DT[c["out"]["dtype"]], what
                assert np.mean(got == ref) >= 0.99, what
                ulp = np.spacing(np.abs(ref).astype(np.float32)) * 65536
                assert np.all(np.abs(got - ref) <= ulp), what
                assert cosine(got, ref) > 0.99999, what
            elif c["fn"] == "sparse_attn":
                assert_close_attn(f32(_bits(out)), f32(_ref_bits(g, c["out"])), what)
            elif c["fn"] == "fp4_act_quant":
                assert np.array_equal(_bits(out), IO.fp4_quant(fp4_in)), what
            else:
                pytest.fail(f"unexpected call {c['fn']}")
    finally:
        torch.set_default_dtype(prev)
    assert _lib.device_error() == 0
    assert seen["sparse_attn"] == 3 and seen["fp8_gemm"] >= 10


def _reference_model_file() -> Path:
    root = Path(os.environ.get("QCAU_REFERENCE_ROOT") or
                Path(__file__).resolve().parents[2] / "reference")
    return root / "Deepseek_origin/inference/model.py"


@pytest.mark.skipif(not _reference_model_file().exists(), reason="reference checkout not present")
def test_reference_model_imports_with_qcau_kernel_module():
    """model.py:12 (`from kernel import act_quant, fp4_act_quant, fp8_gemm,
    fp4_gemm, sparse_attn, hc_split_sinkhorn`) resolves every name on
    qcau_b200.kernel, and the model's kernel calls are then the library's."""
    import importlib.util
    import sys

    from qcau_b200 import kernel

    saved = sys.modules.get("kernel")
    sys.modules["kernel"] = kernel
    try:
        spec = importlib.util.spec_from_file_location("ref_model_qcau_swap", _reference_model_file())
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        if saved is None:
            sys.modules.pop("kernel", None)
        else:
            sys.modules["kernel"] = saved
    for name in ("act_quant", "fp4_act_quant", "fp8_gemm", "fp4_gemm", "sparse_attn",
                 "hc_split_sinkhorn"):
        assert getattr(mod, name) is getattr(kernel, name), name
