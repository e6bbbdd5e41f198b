"""Seeded inputs of the row-wise reduction-reuse workloads (kernels/*__reduction_reuse__credit.cu), shared by
tests/golden/make_rowwise_golden.py (which records the reference kernels' outputs on them) and the tests.

numpy's PCG64 stream is stable across numpy versions, so a case's inputs are reproduced from its seed; the
fixture stores their SHA-256 to detect a change of generator anyway.
"""
from __future__ import annotations

import hashlib

import numpy as np

WORKLOADS = ("rowwise_quant", "lars_momentum", "layernorm_backward", "pearson_backward", "softmax_logits_backward",
             "weighted_var_backward")

# (rows, cols, cluster size P of the reference launch): full slices, ragged columns (cols % 4 != 0, and
# slices that end past the row), the reference shape's slice width (512 at 4096 / 8)
GOLDEN_SHAPES = ((16, 512, 8), (6, 1003, 4), (5, 130, 2), (2, 4096, 8))


def inputs(workload, rows, cols, seed):
    """Dict of float32 arrays (and per-column / per-row vectors) for one case."""
    g = np.random.default_rng(seed)

    def nrm(*shape, scale=1.0, mean=0.0):
        return (mean + scale * g.standard_normal(shape)).astype(np.float32)

    if workload == "rowwise_quant":
        x = nrm(rows, cols)
        x[0] = 0.0                     # all-zero row: scale 0, q 0
        if rows > 1:
            x[1, cols // 3] = 40.0     # one outlier sets the row's scale
        return {"x": x}
    if workload == "lars_momentum":
        return {"w": nrm(rows, cols), "g": nrm(rows, cols, scale=0.1), "m": nrm(rows, cols, scale=0.05)}
    if workload == "layernorm_backward":
        return {"x": nrm(rows, cols, mean=0.5), "dy": nrm(rows, cols), "gamma": nrm(cols, scale=0.1, mean=1.0)}
    if workload == "pearson_backward":
        x = nrm(rows, cols)
        return {"x": x, "y": (0.6 * x + nrm(rows, cols, scale=0.8)).astype(np.float32), "grad": nrm(rows)}
    if workload == "softmax_logits_backward":
        return {"z": nrm(rows, cols, scale=2.0), "dy": nrm(rows, cols)}
    if workload == "weighted_var_backward":
        return {"x": nrm(rows, cols), "w": g.random((rows, cols), dtype=np.float32), "dy": nrm(rows, cols)}
    raise KeyError(workload)


def digest(arrays):
    h = hashlib.sha256()
    for k in sorted(arrays):
        h.update(k.encode())
        h.update(np.ascontiguousarray(arrays[k]).tobytes())
    return h.hexdigest()


def case_seed(workload, shape_index):
    return 1000 * (WORKLOADS.index(workload) + 1) + shape_index


def oracle_outputs(O, workload, a):
    """The oracle's outputs of one case, as a tuple (float64 or the exact integer type)."""
    if workload == "rowwise_quant":
        return O.rowwise_quant(a["x"])
    if workload == "lars_momentum":
        d = O.LARS_DEFAULTS
        return O.lars_momentum(a["w"], a["g"], a["m"], d["mu"], d["wd"], d["lr"], d["eta"], d["eps"])
    if workload == "layernorm_backward":
        return (O.layernorm_backward(a["x"], a["dy"], a["gamma"], O.LN_BWD_EPS),)
    if workload == "pearson_backward":
        return O.pearson_backward(a["x"], a["y"], a["grad"], O.PEARSON_EPS)
    if workload == "softmax_logits_backward":
        return (O.softmax_logits_backward(a["z"], a["dy"]),)
    if workload == "weighted_var_backward":
        return (O.weighted_var_backward(a["x"], a["w"], a["dy"], O.WVAR_EPS),)
    raise KeyError(workload)


def close(out, ref, rel):
    """max |out - ref| <= rel * max(|ref|) (+ a tiny absolute floor); returns (ok, err, scale)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = float(np.max(np.abs(ref))) if ref.size else 0.0
    err = float(np.max(np.abs(out - ref))) if ref.size else 0.0
    return err <= rel * scale + 1e-30, err, scale
