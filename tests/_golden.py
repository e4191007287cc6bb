"""Loaders for the golden vectors in tests/golden (made by make_golden.py)."""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


@dataclass
class Case:
    name: str
    op: str
    args: list  # numpy arrays or ints
    out: np.ndarray | None
    raises: str | None
    message: str | None


def load_cases() -> list[Case]:
    z = np.load(GOLDEN / "ref_cases.npz")
    meta = json.loads(bytes(z["__meta__"]).decode())
    cases = []
    for name in sorted(meta):
        entry = meta[name]
        args = [z[a["tensor"]] if "tensor" in a else a["int"] for a in entry["args"]]
        out = z[f"{name}__out"] if entry["raises"] is None else None
        cases.append(Case(name, entry["op"], args, out, entry["raises"], entry.get("message")))
    return cases


@dataclass
class LganCase:
    name: str
    op: str
    args: list  # numpy arrays or ints
    outs: list[np.ndarray]
    raises: str | None
    message: str | None


def load_lgan_cases() -> list[LganCase]:
    z = np.load(GOLDEN / "ref_lgan.npz")
    meta = json.loads(bytes(z["__meta__"]).decode())
    cases = []
    for name in sorted(meta):
        entry = meta[name]
        args = [z[a["tensor"]] if "tensor" in a else a["int"] for a in entry["args"]]
        outs = [z[f"{name}__out{k}"] for k in range(entry.get("outputs") or 0)]
        cases.append(LganCase(name, entry["op"], args, outs, entry["raises"], entry.get("message")))
    return cases


@dataclass
class PackCase:
    name: str
    op: str
    args: list  # lists of numpy arrays, lists of ints, or ints
    outs: list[np.ndarray]
    raises: str | None
    message: str | None


def load_pack_cases() -> list[PackCase]:
    z = np.load(GOLDEN / "ref_pack.npz")
    meta = json.loads(bytes(z["__meta__"]).decode())
    cases = []
    for name in sorted(meta):
        entry = meta[name]
        args = []
        for a in entry["args"]:
            if "tensors" in a:
                args.append([z[k] for k in a["tensors"]])
            elif "ints" in a:
                args.append(list(a["ints"]))
            else:
                args.append(a["int"])
        outs = [z[f"{name}__out{k}"] for k in range(3)] if entry["raises"] is None else []
        cases.append(PackCase(name, entry["op"], args, outs, entry["raises"], entry.get("message")))
    return cases


def load_cfg1() -> tuple[dict, dict[str, np.ndarray]]:
    z = np.load(GOLDEN / "ref_cfg1.npz")
    meta = json.loads(bytes(z["__meta__"]).decode())
    arrays = {k: z[k] for k in z.files if not k.startswith("__")}
    return meta, arrays


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def close(a: np.ndarray, b: np.ndarray, rtol: float, atol: float) -> bool:
    """allclose with NaN == NaN and matching infinities (torch.allclose equal_nan=True)."""

    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if a.shape != b.shape:
        return False
    return bool(np.allclose(a, b, rtol=rtol, atol=atol, equal_nan=True))
