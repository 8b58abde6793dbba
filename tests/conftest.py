"""Shared pytest setup: import paths, the `gpu` marker, golden fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "continuous-time-attention_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden" / "golden.pt"


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items) -> None:
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="requires a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN, weights_only=False)


def contracted(dtype: torch.dtype) -> bool:
    """Whether a forward of this dtype runs the contracted update by default
    (16-bit tensors; fp32 is always exact)."""
    return dtype in (torch.bfloat16, torch.float16)


def assert_close(a: torch.Tensor, b: torch.Tensor, *, fp32_tol: float = 1e-5, half_tol: float = 2e-2) -> None:
    """Parity bar: max-abs error <= fp32_tol * max|ref| in fp32, <= half_tol in bf16/fp16."""
    half = a.dtype in (torch.bfloat16, torch.float16) or b.dtype in (torch.bfloat16, torch.float16)
    a = a.detach().float().cpu()
    b = b.detach().float().cpu()
    assert a.shape == b.shape, (a.shape, b.shape)
    if a.numel() == 0:
        return
    err = (a - b).abs().max().item()
    scale = max(b.abs().max().item(), 1e-30)
    tol = half_tol if half else fp32_tol * scale
    assert err <= tol, f"max abs err {err:.3e} > tol {tol:.3e}"
