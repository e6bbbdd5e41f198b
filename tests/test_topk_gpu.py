"""GPU parity of the exact top-k kernel (ext_topk.cu) against the CPU oracle.

The reference's criterion (hpc-ops tests/test_topk.py `_validate`, quoted by roofline/workloads/
hpcops_topk_cluster8.yaml): per row, k unique in-range indices whose selected values, sorted, equal torch.topk's
(exact; under ties any choice among equal values is valid). The oracle (orc_topk_values) gives the k largest values
in torch.topk's order; equality is exact, with NaN equal to NaN and -0.0 equal to +0.0.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402


def check_rows(orc, x, idx, k, what):
    rows, n = x.shape
    ref = orc.topk_values(x, k)
    for r in range(rows):
        ir = idx[r].astype(np.int64)
        assert ir.min() >= 0 and ir.max() < n, f"{what} row {r}: index out of range"
        assert np.unique(ir).size == k, f"{what} row {r}: repeated indices"
        got = np.sort(x[r, ir])[::-1]
        exp = np.sort(ref[r])[::-1]
        assert np.array_equal(got, exp, equal_nan=True), f"{what} row {r}: selected values differ"


def run(torch, orc, x, k, n_cta, what):
    tx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = torch.full((x.shape[0], k), -1, dtype=torch.int32, device="cuda")
    D.topk(tx, k=k, cluster_size=n_cta, out=out)
    torch.cuda.synchronize()
    D.topk_check()
    check_rows(orc, x, out.cpu().numpy(), k, what)


@pytest.mark.parametrize("m,n", [(8, 32768), (16, 65536), (8, 244650)])
def test_reference_shapes(cuda, orc, m, n):
    """roofline/workloads/hpcops_topk_cluster8.yaml shapes (randn rows, k = 2048, cluster 8)."""
    x = np.random.default_rng(m * n).standard_normal((m, n)).astype(np.float32)
    run(cuda, orc, x, 2048, 8, f"{m}x{n}")


@pytest.mark.parametrize("n_cta", [2, 4, 16])
def test_cluster_sizes(cuda, orc, n_cta):
    x = np.random.default_rng(n_cta).standard_normal((8, 32768)).astype(np.float32)
    run(cuda, orc, x, 2048, n_cta, f"8x32768 N={n_cta}")


@pytest.mark.parametrize("m,n,k", [(3, 1000, 100), (5, 4097, 7), (4, 300, 300), (6, 513, 1), (2, 5, 3),
                                   (300, 4096, 64), (9, 30001, 2048)])
def test_shapes_and_k(cuda, orc, m, n, k):
    x = (3 * np.random.default_rng(n + k).standard_normal((m, n))).astype(np.float32)
    run(cuda, orc, x, k, 8, f"{m}x{n} k={k}")


def test_ties(cuda, orc):
    """Heavy ties (ten distinct values), an all-equal row, signed zeros and infinities: the refinement rounds
    run to the last bit and the exact ties are shared among the ranks."""
    g = np.random.default_rng(11)
    m, n = 6, 20000
    x = g.integers(0, 10, (m, n)).astype(np.float32)
    x[1] = 1.5
    x[2] = np.where(g.random(n) < 0.5, -0.0, 0.0).astype(np.float32)
    x[3, ::7] = np.inf
    x[3, 1::7] = -np.inf
    x[4] = -np.abs(x[4]) - 1e-3 * np.arange(n, dtype=np.float32)
    x[5] = g.standard_normal(n).astype(np.float16).astype(np.float32)   # values on the fp16 grid
    for k in (1, 2048, 19999):
        for n_cta in (2, 8):
            run(cuda, orc, x, k, n_cta, f"ties k={k} N={n_cta}")


def test_nan_ranks_above_inf(cuda, orc):
    """NaN ranks above +inf (torch's order) and all NaNs of a sign tie exactly: the cut inside a group of NaN
    ties (k smaller than the NaN count) shares them like any other exact ties."""
    g = np.random.default_rng(12)
    x = g.standard_normal((3, 20000)).astype(np.float16).astype(np.float32)
    x[:, ::997] = np.nan
    x[1, 5] = np.inf
    x[2, ::991] = -np.nan
    for k in (1, 2, 21, 2048):
        for n_cta in (2, 8):
            run(cuda, orc, x, k, n_cta, f"nan k={k} N={n_cta}")


def test_close_values_need_all_fine_rounds(cuda, orc):
    """Values within one fp16 step and one fp32 ulp apart: the coarse bin holds every element."""
    base = np.float32(1.0)
    x = (base + np.arange(50000, dtype=np.float32) * np.float32(2.0 ** -23)).reshape(1, -1)
    x = np.random.default_rng(3).permutation(x.ravel()).reshape(1, -1).astype(np.float32)
    for k in (1, 777, 49999):
        run(cuda, orc, x, k, 8, f"close k={k}")


def test_rejects_bad_arguments(cuda):
    import torch

    x = torch.zeros(4, 100, device="cuda")
    with pytest.raises(D.DsmemError):
        D.topk(x, k=101)
    with pytest.raises(D.DsmemError):
        D.topk(x, k=10, cluster_size=3)
