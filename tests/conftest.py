"""Shared pytest set-up: the `gpu` marker, import paths and golden fixtures."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_npz(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as data:
        return {key: data[key] for key in data.files}


def load_json(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


def to_tensor(raw: np.ndarray, dtype: str) -> torch.Tensor:
    """Inverse of make_golden._raw: uint16 bits back to bf16/fp16."""
    if dtype == "bfloat16":
        return torch.from_numpy(raw.view(np.int16).copy()).view(torch.bfloat16)
    if dtype == "float16":
        return torch.from_numpy(raw.copy()).view(torch.float16)
    return torch.from_numpy(raw.copy())


def ffn_case(name: str) -> dict:
    data = load_npz("ffn_cases.npz")
    dtype = str(data[f"{name}/dtype"])
    out = {"dtype": dtype}
    for key in ("gate", "up", "down", "x", "y", "activation", "masked_dense", "dense_activation"):
        out[key] = to_tensor(data[f"{name}/{key}"], dtype)
    out["ids"] = torch.from_numpy(data[f"{name}/ids"].copy())
    return out


FFN_CASES = ["reftest_f32", "phase5b_f16", "small_f32", "small_bf16", "pad_bf16", "wide_bf16", "f16_b3"]

# rel-L2 tolerances of y against the reference (16-bit weights / fp32 weights).
TOL = {"bfloat16": 1e-2, "float16": 1e-2, "float32": 1e-5}


@pytest.fixture(scope="session")
def golden_ffn():
    return {name: ffn_case(name) for name in FFN_CASES}
