"""Loader for the golden vectors in tests/golden (made by make_golden.py)."""

from __future__ import annotations

import json
import os

import numpy as np

from oracle.fd_oracle import bf16_bits_to_f32

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _to_f32(arr: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(arr)
    return np.asarray(arr, dtype=np.float32)


def load_golden() -> list[dict]:
    """Cases as dicts: op, dtype, params, inputs/outputs (name -> (float32 array, dtype))."""
    with open(os.path.join(HERE, "manifest.json")) as f:
        manifest = json.load(f)
    z = np.load(os.path.join(HERE, "golden.npz"))
    cases = []
    for c in manifest["cases"]:
        case = {"id": c["id"], "op": c["op"], "dtype": c["dtype"], "params": c["params"]}
        for kind in ("inputs", "outputs"):
            case[kind] = {
                name: (_to_f32(z[f"{c['id']}/{name}"], meta["dtype"]), meta["dtype"])
                for name, meta in c[kind].items()
            }
        cases.append(case)
    return cases


def torch_dtype(name: str):
    import torch

    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[name]


def to_torch(arr_dtype, device="cuda"):
    """(float32 array, dtype name) -> torch tensor of that dtype (values exact)."""
    import torch

    arr, dtype = arr_dtype
    return torch.from_numpy(np.ascontiguousarray(arr)).to(device=device, dtype=torch_dtype(dtype))
