"""Shared test plumbing.

Markers: `gpu` tests need a CUDA device and go through libmlb.so's C ABI;
everything else runs on the CPU (oracle pinning, the C-ABI surface, host
logic, gloo multi-process checks).
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG = os.path.join(ROOT, "mini-lla_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity bound for the floating-point operators whose reduction order or exp
# differs from the reference CPU path (RMSNorm output, SiLU/SwiGLU, softmax).
REL_TOL = 1e-5


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def ensure_built():
    """Builds libmlb.so and the oracle in-tree when they are missing (the
    GPU box has the same toolchain)."""
    if not os.path.exists(os.path.join(PKG, "libmlb.so")):
        subprocess.run(["make", "-s", "-C", PKG, "-j8"], check=True)
    if not os.path.exists(os.path.join(ORACLE_DIR, "liboracle.so")):
        subprocess.run(["make", "-s", "-C", ORACLE_DIR, "all"], check=True)


ensure_built()


def golden(name: str):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def assert_bitexact(got, want, what=""):
    """Bit-for-bit equality; NaNs compare equal to any NaN (the payload of a
    NaN differs between an x86 multiply and a GPU multiply)."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    want = np.ascontiguousarray(want, dtype=np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn), f"{what}: NaN positions differ"
    gb = got.view(np.uint32)[~gn]
    wb = want.view(np.uint32)[~wn]
    bad = np.nonzero(gb != wb)[0]
    assert bad.size == 0, (
        f"{what}: {bad.size} of {gb.size} values differ; first at flat "
        f"{bad[0]}: got {got[~gn][bad[0]]!r} want {want[~wn][bad[0]]!r}")


def max_rel(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    same = (got == want) | (np.isnan(got) & np.isnan(want))
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = np.where(same, 0.0, np.abs(got - want) / np.abs(want))
    rel = np.where(np.isnan(rel), np.inf, rel)
    return float(rel.max()) if rel.size else 0.0


def assert_rel(got, want, tol=REL_TOL, what=""):
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    r = max_rel(got, want)
    assert r <= tol, f"{what}: max relative error {r:.3e} > {tol:.0e}"


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        pytest.skip("reference CPU library (oracle/_ref) not built here")
    return Reference()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mlb
    mlb.load()
    return torch.device("cuda:0")
