"""Shared test setup: import paths, the ``gpu`` marker and golden-fixture loading."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "mixture-of-convolutions_b200")
for path in (ROOT, PKG_ROOT):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


class Golden:
    def __init__(self) -> None:
        self.arrays = dict(np.load(os.path.join(GOLDEN_DIR, "moc_golden.npz")))
        with open(os.path.join(GOLDEN_DIR, "moc_golden_meta.json")) as f:
            self.meta = json.load(f)

    def t(self, key: str) -> torch.Tensor:
        return torch.from_numpy(self.arrays[key].copy())


_GOLDEN = None


@pytest.fixture(scope="session")
def golden() -> Golden:
    global _GOLDEN
    if _GOLDEN is None:
        _GOLDEN = Golden()
    return _GOLDEN


DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / max |ref|: error relative to the tensor's scale."""
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    scale = ref.abs().max().item()
    return (got - ref).abs().max().item() / (scale if scale > 0 else 1.0)
