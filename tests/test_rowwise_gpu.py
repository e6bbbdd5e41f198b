"""GPU parity of the row-wise reduction-reuse kernels (ext_rowwise.cu) against the CPU oracle and against the
reference's own clustered kernels (kernels/*__reduction_reuse__credit.cu run on a B200, tests/golden/).

Tolerances: the int8 quantisation and its scales are bit-exact (the row maximum is order-free and the element
formula is the reference's fp32 arithmetic). fp32 outputs: max |got - ref| <= 1e-4 * max |ref| over the case,
against the oracle (double statistics) and against the reference kernels (fp32 with their own summation order);
the kernels merge per-CTA records (one exchange per row) where the reference runs 1-3 AllReduce stages, so
the last bits differ by design.
"""
import os
import pathlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402
import rowwise_cases as RC  # noqa: E402

REL = 1e-4
GOLDEN = pathlib.Path(os.environ.get("ROWWISE_GOLDEN", pathlib.Path(__file__).resolve().parent / "golden" / "rowwise_golden.npz"))


def ours(torch, workload, a, n):
    """Run our kernel on host arrays `a`; returns the outputs as numpy arrays."""
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in a.items()}
    if workload == "rowwise_quant":
        outs = D.rowwise_quant(t["x"], cluster_size=n)
    elif workload == "lars_momentum":
        outs = D.lars_momentum(t["w"], t["g"], t["m"], cluster_size=n)
    elif workload == "layernorm_backward":
        outs = (D.layernorm_backward(t["x"], t["dy"], t["gamma"], cluster_size=n),)
    elif workload == "pearson_backward":
        outs = D.pearson_backward(t["x"], t["y"], t["grad"], cluster_size=n)
    elif workload == "softmax_logits_backward":
        outs = (D.softmax_logits_backward(t["z"], t["dy"], cluster_size=n),)
    else:
        outs = (D.weighted_var_backward(t["x"], t["w"], t["dy"], cluster_size=n),)
    torch.cuda.synchronize()
    D.rowwise_check()
    return [o.cpu().numpy() for o in outs]


def assert_match(workload, got, ref, what):
    if workload == "rowwise_quant":
        q, sc = got
        rq, rsc = ref
        assert np.array_equal(sc.view(np.uint32), np.asarray(rsc, np.float32).view(np.uint32)), f"{what}: scales"
        bad = np.argwhere(q != rq)
        assert bad.size == 0, f"{what}: {len(bad)} int8 mismatches, first at {bad[:3].tolist()}"
        return
    for j, (g, r) in enumerate(zip(got, ref)):
        assert np.isfinite(g).all(), f"{what}: output {j} not finite"
        ok, err, scale = RC.close(g, r, REL)
        assert ok, f"{what}: output {j} max err {err:.3e} > {REL} x {scale:.3e}"


@pytest.mark.parametrize("workload", RC.WORKLOADS)
@pytest.mark.parametrize("n,rows,cols", [(8, 37, 4096), (1, 9, 512), (2, 11, 2048), (4, 13, 1003), (16, 10, 8192),
                                         (8, 7, 5), (8, 70, 200), (2, 3, 130)])
def test_matches_oracle(cuda, orc, workload, n, rows, cols):
    a = RC.inputs(workload, rows, cols, 77 + rows)
    assert_match(workload, ours(cuda, workload, a, n), RC.oracle_outputs(orc, workload, a),
                 f"{workload} {rows}x{cols} N={n}")


@pytest.mark.skipif(not GOLDEN.exists(), reason="rowwise golden fixture not generated")
@pytest.mark.parametrize("workload", RC.WORKLOADS)
def test_matches_reference_kernels(cuda, orc, workload):
    g = np.load(GOLDEN)
    for si, (rows, cols, p) in enumerate(RC.GOLDEN_SHAPES):
        key = f"{workload}__{si}"
        assert tuple(g[key + "__shape"]) == (rows, cols, p)
        a = RC.inputs(workload, rows, cols, RC.case_seed(workload, si))
        assert str(g[key + "__sha256"]) == RC.digest(a), "input generator changed since the fixture was made"
        ref = [g[f"{key}__out{j}"] for j in range(2 if workload in ("rowwise_quant", "lars_momentum",
                                                                     "pearson_backward") else 1)]
        for n in sorted({p, 8}):
            assert_match(workload, ours(cuda, workload, a, n), ref, f"{workload} {rows}x{cols} N={n} vs reference")


def _big_inputs(torch, workload, rows, cols, seed):
    """Full-size inputs generated on the device (seeded), as torch tensors."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    nrm = lambda *s, scale=1.0, mean=0.0: mean + scale * torch.randn(*s, device="cuda", generator=gen)  # noqa: E731
    if workload == "rowwise_quant":
        return {"x": nrm(rows, cols)}
    if workload == "lars_momentum":
        return {"w": nrm(rows, cols), "g": nrm(rows, cols, scale=0.1), "m": nrm(rows, cols, scale=0.05)}
    if workload == "layernorm_backward":
        return {"x": nrm(rows, cols, mean=0.5), "dy": nrm(rows, cols), "gamma": nrm(cols, scale=0.1, mean=1.0)}
    if workload == "pearson_backward":
        x = nrm(rows, cols)
        return {"x": x, "y": 0.6 * x + nrm(rows, cols, scale=0.8), "grad": nrm(rows)}
    if workload == "softmax_logits_backward":
        return {"z": nrm(rows, cols, scale=2.0), "dy": nrm(rows, cols)}
    return {"x": nrm(rows, cols), "w": torch.rand(rows, cols, device="cuda", generator=gen), "dy": nrm(rows, cols)}


@pytest.mark.parametrize("workload", RC.WORKLOADS)
@pytest.mark.parametrize("cols", [4096, 16384, 65536])
def test_reference_shapes_sampled_rows(cuda, orc, workload, cols):
    """The reference's shapes (4096 rows x {4k, 16k, 64k} cols, cluster 8): every output row is computed on the
    device; 48 rows spread over the tensor (first, last, and between) are checked against the oracle."""
    torch = cuda
    rows = 4096
    t = _big_inputs(torch, workload, rows, cols, 5 + cols)
    if workload == "rowwise_quant":
        outs = D.rowwise_quant(t["x"])
    elif workload == "lars_momentum":
        outs = D.lars_momentum(t["w"], t["g"], t["m"])
    elif workload == "layernorm_backward":
        outs = (D.layernorm_backward(t["x"], t["dy"], t["gamma"]),)
    elif workload == "pearson_backward":
        outs = D.pearson_backward(t["x"], t["y"], t["grad"])
    elif workload == "softmax_logits_backward":
        outs = (D.softmax_logits_backward(t["z"], t["dy"]),)
    else:
        outs = (D.weighted_var_backward(t["x"], t["w"], t["dy"]),)
    torch.cuda.synchronize()
    D.rowwise_check()
    sel = np.unique(np.concatenate([[0, rows - 1], np.linspace(1, rows - 2, 46).astype(np.int64)]))
    idx = torch.from_numpy(sel).cuda()
    a = {k: (v[idx] if v.dim() == 2 or k == "grad" else v).cpu().numpy() for k, v in t.items()}
    got = [(o[idx] if o.dim() == 2 or workload == "rowwise_quant" else o).cpu().numpy() for o in outs]
    assert_match(workload, got, RC.oracle_outputs(orc, workload, a), f"{workload} {rows}x{cols} N=8 sampled")
    del t, outs
    torch.cuda.empty_cache()


def test_quant_all_zero_and_outlier_rows(cuda, orc):
    a = RC.inputs("rowwise_quant", 4, 4096, 3)
    q, sc = ours(cuda, "rowwise_quant", a, 8)
    assert sc[0] == 0.0 and not q[0].any()
    assert q[1].max() == 127 and sc[1] == np.float32(np.float32(40.0) / np.float32(127.0))


def test_launch_order_of_shapes(cuda, orc):
    """One kernel launched with a larger, then a smaller, then the larger shared-memory size again (the
    dynamic shared-memory opt-in of a kernel only grows)."""
    for cols in (16384, 512, 16384):
        a = RC.inputs("softmax_logits_backward", 6, cols, cols)
        assert_match("softmax_logits_backward", ours(cuda, "softmax_logits_backward", a, 8),
                     RC.oracle_outputs(orc, "softmax_logits_backward", a), f"softmax 6x{cols}")


@pytest.mark.parametrize("n", [2, 8])
def test_edge_rows(cuda, orc, n):
    """Rows whose slices are degenerate on some CTAs: constant rows (zero variance), zero weights over whole
    slices (a zero-weight record in the merge), logits of -inf over whole slices (a -inf maximum in the merge)."""
    rows, cols = 6, 4096
    g = np.random.default_rng(40 + n)
    a = RC.inputs("layernorm_backward", rows, cols, 9)
    a["x"][0] = 0.5
    a["x"][1, : cols // 2] = -1.25
    assert_match("layernorm_backward", ours(cuda, "layernorm_backward", a, n),
                 RC.oracle_outputs(orc, "layernorm_backward", a), f"LN edge rows N={n}")
    a = RC.inputs("pearson_backward", rows, cols, 10)
    a["x"][0] = 0.5
    a["y"][1] = -2.0
    assert_match("pearson_backward", ours(cuda, "pearson_backward", a, n),
                 RC.oracle_outputs(orc, "pearson_backward", a), f"Pearson edge rows N={n}")
    a = RC.inputs("weighted_var_backward", rows, cols, 11)
    a["w"][0, : cols // 2] = 0.0
    a["w"][1] = 0.0
    a["x"][2] = 0.75
    assert_match("weighted_var_backward", ours(cuda, "weighted_var_backward", a, n),
                 RC.oracle_outputs(orc, "weighted_var_backward", a), f"wvar edge rows N={n}")
    a = RC.inputs("softmax_logits_backward", rows, cols, 12)
    a["z"][0, : cols // 2] = -np.inf
    a["z"][1, cols // 4:] = -np.inf
    a["z"][2] = 3.0
    assert_match("softmax_logits_backward", ours(cuda, "softmax_logits_backward", a, n),
                 RC.oracle_outputs(orc, "softmax_logits_backward", a), f"softmax edge rows N={n}")
    a = RC.inputs("lars_momentum", rows, cols, 13)
    a["w"][0] = 0.0
    a["g"][1] = 0.0
    a["m"][1] = 0.0
    assert_match("lars_momentum", ours(cuda, "lars_momentum", a, n),
                 RC.oracle_outputs(orc, "lars_momentum", a), f"LARS edge rows N={n}")
    del g
