"""Shared pytest setup.

* ``-m gpu`` tests need a CUDA device (a B200); everything else runs on CPU.
* The product package lives in ``causal-conv1d-mojo_b200/`` (not a valid
  module name), so that directory is put on ``sys.path``; the repo root is
  put there for the test-only ``oracle`` package.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
PROJECT = REPO / "causal-conv1d-mojo_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PROJECT), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}

# Parity tolerances (elementwise |a-b| <= atol + rtol*|b|), per dtype: the
# bar of the build's north star -- 1e-5 in fp32, 1e-2 in bf16/fp16.
TOL = {
    torch.float32: dict(rtol=1e-5, atol=1e-5),
    torch.bfloat16: dict(rtol=1e-2, atol=1e-2),
    torch.float16: dict(rtol=1e-2, atol=1e-2),
}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


class Golden:
    """Cases and arrays written by tests/golden/make_golden.py."""

    def __init__(self):
        self.manifest = json.loads((GOLDEN / "cases.json").read_text())
        self._npz = {}

    def cases(self, group):
        return self.manifest["groups"][group]

    def arrays(self, group):
        if group not in self._npz:
            self._npz[group] = np.load(GOLDEN / f"golden_{group}.npz")
        return self._npz[group]

    def inputs(self, group, case):
        dt = DTYPES[case["dtype"]]
        z = self.arrays(group)
        pre = f"{case['name']}/in/"
        out = {}
        for key in z.files:
            if key.startswith(pre):
                a = torch.from_numpy(z[key].copy())
                out[key[len(pre):]] = a if a.dtype == torch.int32 else a.to(dt)
        return out

    def expected(self, group, case):
        z = self.arrays(group)
        pre = f"{case['name']}/exp/"
        return {k[len(pre):]: torch.from_numpy(z[k].copy()) for k in z.files if k.startswith(pre)}


_GOLDEN = Golden()


@pytest.fixture(scope="session")
def golden():
    return _GOLDEN


def golden_cases(group):
    return _GOLDEN.cases(group)


def assert_close(actual, expected, dtype, what="", rtol=None, atol=None):
    tol = dict(TOL[dtype])
    if rtol is not None:
        tol["rtol"] = rtol
    if atol is not None:
        tol["atol"] = atol
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} vs {tuple(e.shape)}"
    assert torch.isfinite(a).all(), f"{what}: non-finite values"
    if not torch.allclose(a, e, **tol):
        diff = (a - e).abs()
        i = int(diff.argmax())
        raise AssertionError(
            f"{what}: max |diff| {diff.max().item():.3e} at flat index {i} "
            f"(got {a.flatten()[i].item():.6g}, want {e.flatten()[i].item():.6g}, tol {tol})"
        )


def assert_bitwise(actual, expected, what=""):
    a = actual.detach().cpu()
    e = expected.detach().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} vs {tuple(e.shape)}"
    if a.dtype != e.dtype:
        e = e.to(a.dtype)
    if not torch.equal(a, e):
        n = (a != e).sum().item()
        raise AssertionError(f"{what}: {n} elements differ (bit-exact expected)")
