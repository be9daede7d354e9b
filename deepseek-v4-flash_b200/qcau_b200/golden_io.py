"""The reference's golden-vector wire format (QCAU/QCAU_inference/framework/
README.md:76-115), read and written exactly.

A case directory holds one file per tensor plus `<name>.shape.txt` (the
dimensions, whitespace separated) and `metadata.json`:

    <name>.bf16_hex.txt      one bf16 bit pattern a line, 4 hex digits
    <name>.fp8_e4m3_hex.txt  one e4m3 byte a line, 2 hex digits
    <name>.e8m0_hex.txt      one E8M0 scale byte a line, 2 hex digits
    <name>.fp32.txt          decimal text, one value a line
    <name>.int.txt           decimal integers

Values are flat row-major.  bf16 / fp8 / e8m0 tensors come back as their raw
bit patterns (uint16 / uint8 numpy arrays) so nothing is rounded on the way;
as_torch() views them as the matching torch dtypes.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Dict

import numpy as np

_SUFFIX = {
    "bf16": (".bf16_hex.txt", np.uint16, 4),
    "fp8_e4m3": (".fp8_e4m3_hex.txt", np.uint8, 2),
    "e8m0": (".e8m0_hex.txt", np.uint8, 2),
    "fp32": (".fp32.txt", np.float32, None),
    "int": (".int.txt", np.int64, None),
}


def read_shape(case: Path, name: str) -> tuple:
    return tuple(int(x) for x in (Path(case) / f"{name}.shape.txt").read_text().split())


def tensor_kind(case: Path, name: str) -> str:
    """Which of the formats a tensor of the case is stored in."""
    for kind, (suffix, _, _) in _SUFFIX.items():
        if (Path(case) / f"{name}{suffix}").exists():
            return kind
    raise FileNotFoundError(f"{name} not found in {case}")


def read_tensor(case: Path, name: str) -> np.ndarray:
    """The tensor `name` of a case directory, shaped; hex formats as raw bits."""
    case = Path(case)
    kind = tensor_kind(case, name)
    suffix, dtype, digits = _SUFFIX[kind]
    text = (case / f"{name}{suffix}").read_text().split()
    if digits is not None:
        flat = np.fromiter((int(t, 16) for t in text), dtype=np.int64, count=len(text))
        if flat.size and (flat.min() < 0 or flat.max() >= 1 << (4 * digits)):
            raise ValueError(f"{name}: value outside {digits} hex digits")
        flat = flat.astype(dtype)
    elif kind == "int":
        flat = np.asarray(text, dtype=np.int64)
    else:
        flat = np.asarray(text, dtype=np.float64).astype(np.float32)
    shape_file = case / f"{name}.shape.txt"
    return flat.reshape(read_shape(case, name)) if shape_file.exists() else flat


def write_tensor(case: Path, name: str, values: np.ndarray, kind: str) -> None:
    """Write `values` in the reference's format (kind: bf16, fp8_e4m3, e8m0,
    fp32, int); hex kinds take raw bit patterns."""
    case = Path(case)
    case.mkdir(parents=True, exist_ok=True)
    suffix, dtype, digits = _SUFFIX[kind]
    v = np.asarray(values)
    if digits is not None:
        flat = v.astype(np.int64).ravel()
        lines = [format(int(x), f"0{digits}x") for x in flat]
    elif kind == "int":
        lines = [str(int(x)) for x in v.ravel()]
    else:
        lines = [repr(float(np.float32(x))) for x in v.ravel()]
    (case / f"{name}{suffix}").write_text("\n".join(lines) + "\n")
    (case / f"{name}.shape.txt").write_text(" ".join(str(s) for s in v.shape) + "\n")


def read_case(case: Path) -> Dict[str, object]:
    """Every tensor of a case (by name) plus "metadata"."""
    case = Path(case)
    out: Dict[str, object] = {"metadata": json.loads((case / "metadata.json").read_text())}
    names = set()
    for kind, (suffix, _, _) in _SUFFIX.items():
        for f in case.glob(f"*{suffix}"):
            names.add(f.name[: -len(suffix)])
    for n in sorted(names):
        out[n] = read_tensor(case, n)
    return out


def as_torch(bits: np.ndarray, kind: str, device="cpu"):
    """Raw bit patterns as a torch tensor of the format's dtype."""
    import torch

    if kind == "bf16":
        return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(
            torch.bfloat16).to(device)
    if kind == "fp8_e4m3":
        return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint8)).view(
            torch.float8_e4m3fn).to(device)
    if kind == "e8m0":
        return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint8)).view(
            torch.float8_e8m0fnu).to(device)
    return torch.from_numpy(np.asarray(bits)).to(device)
