"""CPU tests of the row-wise reduction-reuse oracle and host logic (no GPU).

The oracle (oracle/dsmem_oracle.c, orc_rowwise_* and friends) restates the clustered kernels of
kernels/*__reduction_reuse__credit.cu. It is pinned here against the reference kernels' own outputs
(tests/golden/rowwise_golden.npz, recorded on a B200 by tests/golden/make_rowwise_golden.py): the int8
quantisation bit-exactly, fp32 outputs within 5e-5 of their largest magnitude (the reference accumulates in
fp32, the oracle in double).
"""
import ctypes
import os
import pathlib

import numpy as np
import pytest

import rowwise_cases as RC

GOLDEN = pathlib.Path(os.environ.get("ROWWISE_GOLDEN", pathlib.Path(__file__).resolve().parent / "golden" / "rowwise_golden.npz"))
REL_REF = 5e-5
N_OUT = {"rowwise_quant": 2, "lars_momentum": 2, "pearson_backward": 2}


@pytest.mark.skipif(not GOLDEN.exists(), reason="rowwise golden fixture not generated")
@pytest.mark.parametrize("workload", RC.WORKLOADS)
def test_oracle_matches_reference_kernels(orc, workload):
    g = np.load(GOLDEN)
    for si, (rows, cols, p) in enumerate(RC.GOLDEN_SHAPES):
        key = f"{workload}__{si}"
        a = RC.inputs(workload, rows, cols, RC.case_seed(workload, si))
        assert str(g[key + "__sha256"]) == RC.digest(a)
        ref = [g[f"{key}__out{j}"] for j in range(N_OUT.get(workload, 1))]
        got = RC.oracle_outputs(orc, workload, a)
        if workload == "rowwise_quant":
            assert np.array_equal(got[0], ref[0]), f"{key}: int8 outputs differ"
            assert np.array_equal(got[1].view(np.uint32), ref[1].view(np.uint32)), f"{key}: scales differ"
            continue
        for j, (o, r) in enumerate(zip(got, ref)):
            ok, err, scale = RC.close(o, r, REL_REF)
            assert ok, f"{key} output {j}: max err {err:.3e} vs scale {scale:.3e}"


def test_quantize_element_formula(orc):
    """quantize_to_i8 (rowwise_quant :100-105): round half to even, clamp at +-127, NaN to -127 (fmaxf)."""
    q = orc.lib().orc_quantize_i8
    assert q(2.5, 1.0) == 2 and q(3.5, 1.0) == 4 and q(-2.5, 1.0) == -2
    assert q(1000.0, 1.0) == 127 and q(-1000.0, 1.0) == -127
    assert q(float("nan"), 1.0) == -127
    assert q(5.0, 0.0) == 0


def test_merged_statistics_equal_reference_stages(orc):
    """The kernels merge per-slice records (count/weight, mean, centred sums) instead of the reference's
    stage-by-stage sums; in exact arithmetic both give the same row statistics. Checked here in double on
    random slices: LayerNorm-backward's {mean, var, sum dyg*xhat}, the weighted variance's eps-shifted mean,
    variance and sum dy*(x - mean)."""
    g = np.random.default_rng(5)
    cols, eps = 1003, 1e-6
    x, dy, gm = g.standard_normal(cols), g.standard_normal(cols), 1 + 0.1 * g.standard_normal(cols)
    w = g.random(cols)
    cuts = [0, 251, 502, 753, cols]

    def merge_ln(a, b):
        n = a[0] + b[0]
        m = (a[0] * a[1] + b[0] * b[1]) / n if n else 0.0
        da, db = a[1] - m, b[1] - m
        return (n, m, a[2] + b[2] + a[0] * da * da + b[0] * db * db, a[3] + b[3], a[4] + b[4] + da * a[3] + db * b[3])

    recs = []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        xs, dyg = x[lo:hi], dy[lo:hi] * gm[lo:hi]
        m = xs.mean()
        recs.append((hi - lo, m, ((xs - m) ** 2).sum(), dyg.sum(), (dyg * (xs - m)).sum()))
    t = recs[0]
    for r in recs[1:]:
        t = merge_ln(t, r)
    mean, var = x.mean(), (x * x).mean() - x.mean() ** 2
    inv_std = 1 / np.sqrt(var + eps)
    assert abs(t[1] - mean) < 1e-12 and abs(t[2] / cols - var) < 1e-12
    assert abs(t[4] * inv_std - (dy * gm * (x - mean) * inv_std).sum()) < 1e-9

    recs = []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        xs, ws, ds = x[lo:hi], w[lo:hi], dy[lo:hi]
        W = ws.sum()
        m = (ws * xs).sum() / W
        recs.append((W, m, (ws * (xs - m) ** 2).sum(), ds.sum(), (ds * (xs - m)).sum()))
    t = recs[0]
    for r in recs[1:]:
        t = merge_ln(t, r)   # the same update with weights in place of counts
    inv_sum_w = 1 / (w.sum() + eps)
    mean_ref = (w * x).sum() * inv_sum_w
    d = t[1] - t[1] * t[0] * inv_sum_w
    assert abs(t[1] * t[0] * inv_sum_w - mean_ref) < 1e-12
    assert abs((t[2] + t[0] * d * d) * inv_sum_w - (w * (x - mean_ref) ** 2).sum() * inv_sum_w) < 1e-12
    assert abs((t[4] + d * t[3]) - (dy * (x - mean_ref)).sum()) < 1e-9


def test_softmax_record_merge(orc):
    """(max, sum exp(z - max), sum exp(z - max) dy) records merge to the row's own values."""
    g = np.random.default_rng(6)
    z, dy = 3 * g.standard_normal(700), g.standard_normal(700)
    recs = []
    for lo, hi in ((0, 100), (100, 350), (350, 700)):
        m = z[lo:hi].max()
        e = np.exp(z[lo:hi] - m)
        recs.append((m, e.sum(), (e * dy[lo:hi]).sum()))
    M = max(r[0] for r in recs)
    S = sum(r[1] * np.exp(r[0] - M) for r in recs)
    Dd = sum(r[2] * np.exp(r[0] - M) for r in recs)
    p = np.exp(z - z.max()) / np.exp(z - z.max()).sum()
    assert abs(Dd / S - (p * dy).sum()) < 1e-12


def test_capi_rowwise_argument_checks(dsmem):
    """Host-side checks of the row-wise C ABI, which return before any device call."""
    lib = dsmem.lib()
    fake = ctypes.c_void_p(0x10000)
    null = ctypes.c_void_p(None)
    s = dsmem.Status
    # one row slice of the three LARS inputs at 65536 columns over 2 CTAs is 384 KiB > 227 KiB
    assert lib.dsmem_lars_momentum_launch(fake, fake, fake, fake, fake, 4096, 65536, 0.9, 0.01, 1e-3, 0.02, 1e-6, 2,
                                          null) == s.SMEM_LIMIT
    assert lib.dsmem_rowwise_quant_launch(fake, fake, fake, 16, 4096, 3, null) == s.INVALID_ARGUMENT
    assert lib.dsmem_rowwise_quant_launch(null, fake, fake, 16, 4096, 8, null) == s.INVALID_ARGUMENT
    assert lib.dsmem_softmax_logits_backward_launch(fake, fake, fake, 16, 0, 8, null) == s.INVALID_ARGUMENT
    assert lib.dsmem_weighted_var_backward_launch(fake, fake, fake, fake, 0, 4096, 1e-6, 8, null) == s.OK

