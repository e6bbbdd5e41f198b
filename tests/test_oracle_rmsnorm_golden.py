"""The RMSNorm oracle (orc_rmsnorm, a restatement of clusterfusion_rmsnorm.py:62-66 in double) pinned to the
reference itself, on the CPU, through tests/golden/rmsnorm_golden.npz (made by tests/golden/make_rmsnorm_golden.py):
  * y_expr: the reference wrapper's own fp32 torch expression (the `y32` of its check(), evaluated from the
    reference source on the CPU) -- the oracle agrees to fp32 rounding;
  * y_kernel_fp16 (when present): the reference's own RMSNormKernel (kernels/rmsnorm__llama__clusterfusion.cu,
    fp16, cluster 2) run on a B200 -- the oracle agrees within the wrapper's own tolerance, max abs 1e-2
    (clusterfusion_rmsnorm.py:28), here to fp16 rounding.
The inputs are regenerated from the oracle's seeded draws and checked against the fixture's SHA-256.
"""
import hashlib
import importlib.util
import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def golden(orc):
    spec = importlib.util.spec_from_file_location("make_rmsnorm_golden", GOLDEN / "make_rmsnorm_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    d = dict(np.load(GOLDEN / "rmsnorm_golden.npz"))
    x, w = mod.inputs()
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(d["x_sha256"])
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(d["w_sha256"])
    return d, x, w


def test_oracle_matches_reference_expression(orc, golden):
    d, x, w = golden
    rows = d["kept_rows"]
    y, _ = orc.rmsnorm(0, x, w, float(d["eps"]))
    err = np.abs(y[rows] - d["y_expr"].astype(np.float64)) / (1.0 + np.abs(y[rows]))
    assert err.max() <= 2e-6, f"oracle vs the reference's fp32 expression: max rel {err.max():.3e}"
    # the check is sensitive: a wrong eps or a dropped weight is far outside it
    y_eps, _ = orc.rmsnorm(0, x, w, 1e-2)
    assert (np.abs(y_eps[rows] - d["y_expr"]) / (1.0 + np.abs(y_eps[rows]))).max() > 1e-4
    y_now, _ = orc.rmsnorm(0, x, np.ones_like(w), float(d["eps"]))
    assert (np.abs(y_now[rows] - d["y_expr"]) / (1.0 + np.abs(y_now[rows]))).max() > 1e-3


def test_oracle_matches_reference_kernel(orc, golden):
    d, x, w = golden
    if "y_kernel_fp16" not in d:
        pytest.skip("fixture has no reference-kernel output (make_rmsnorm_golden.py kernel not run yet)")
    rows = d["kept_rows"]
    yk = d["y_kernel_fp16"].view(np.float16).astype(np.float64)
    y, _ = orc.rmsnorm(0, x, w, float(d["eps"]))
    err = np.abs(yk - y[rows])
    assert err.max() <= 1e-2, f"reference kernel vs oracle: max abs {err.max():.3e} (tolerance 1e-2)"
    # fp16 rounding of the output (2^-11 relative) plus the kernel's fp32 arithmetic
    assert (err / (1.0 + np.abs(y[rows]))).max() <= 2e-3
