"""Shared pytest setup: the `gpu` marker, import paths, and lazily built native libraries.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's golden vectors, the host logic of the
C ABI (legality, names, tables) and that the library exports every declared symbol. GPU tests
(`-m gpu`) are the parity tests proper and call the CUDA kernels through the C ABI.
"""
import json
import os
import pathlib
import subprocess
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "h100-dsmem-collectives_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


def _build_native():
    lib = PKG / "lib" / "libdsmem_b200.so"
    if not lib.exists():
        subprocess.run(["make", "-s", "-C", str(PKG), "-j8"], check=True)
    orc = ROOT / "oracle" / "_build" / "liboracle.so"
    if not orc.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)


@pytest.fixture(scope="session")
def dsmem():
    _build_native()
    import dsmem_b200

    dsmem_b200.lib()
    return dsmem_b200


@pytest.fixture(scope="session")
def orc():
    _build_native()
    from oracle import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def reference_root():
    """The reference checkout where it is mounted: $REF, else BASELINE.json's reference_path; None if absent.
    Only CPU tests that build or read the reference's own sources use it (never a GPU test)."""
    ref = os.environ.get("REF")
    if not ref:
        try:
            ref = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            ref = None
    return pathlib.Path(ref) if ref and pathlib.Path(ref).is_dir() else None
