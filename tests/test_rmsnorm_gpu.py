"""GPU parity of the cluster-fused RMSNorm against the CPU oracle (clusterfusion_rmsnorm.py:65 in double).

Tolerance: |got - ref| <= rtol * (1 + |ref|) with rtol 1e-2 for bf16 outputs (the bf16 bound of the
north-star; the reference wrapper used max abs 1e-2 for fp16, clusterfusion_rmsnorm.py:28) and 1e-5 for f32.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402

RTOL = {D.Dtype.BF16: 1e-2, D.Dtype.F32: 1e-5}


def to_torch(torch, host, dt):
    if dt == D.Dtype.BF16:
        return torch.from_numpy(host.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(host.copy()).cuda()


def to_np(t, dt):
    import torch

    t = t.cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if dt == D.Dtype.BF16 else t.numpy()


def run(torch, orc, dt, rows, hidden, n, residual=False, seed=0):
    odt = 1 if dt == D.Dtype.BF16 else 0
    x = orc.normal(odt, rows * hidden, seed, 0.0, 1.0).reshape(rows, hidden)
    w = orc.normal(odt, hidden, seed + 1, 1.0, 0.02)
    res = orc.normal(odt, rows * hidden, seed + 2, 0.0, 1.0).reshape(rows, hidden) if residual else None
    tx, tw = to_torch(torch, x, dt), to_torch(torch, w, dt)
    tr = to_torch(torch, res, dt) if residual else None
    ty = torch.full_like(tx, float("nan"))
    tp = torch.full_like(tx, float("nan")) if residual else None
    D.rmsnorm(tx, tw, 1e-6, cluster_size=n, out=ty, residual=tr, pre_norm=tp)
    torch.cuda.synchronize()
    D.rmsnorm_check()
    if residual:
        # the kernel rounds h = x + res to the element type before normalising (as hpc-ops' packed add)
        if dt == D.Dtype.BF16:
            hx = orc.bf16_to_f32(x).astype(np.float64) + orc.bf16_to_f32(res).astype(np.float64)
            h = orc.f32_to_bf16(hx.astype(np.float32))
        else:
            h = (x.astype(np.float32) + res.astype(np.float32)).astype(np.float32)
        bad, ma, _ = orc.check(odt, to_np(tp, dt).ravel(), (orc.bf16_to_f32(h) if dt == D.Dtype.BF16 else h)
                               .astype(np.float64).ravel(), 0)
        assert bad == 0, f"pre-norm output differs ({bad} elements, max abs {ma})"
        ref, _ = orc.rmsnorm(odt, h.reshape(rows, hidden), w, 1e-6)
    else:
        ref, _ = orc.rmsnorm(odt, x, w, 1e-6)
    bad, ma, mr = orc.check(odt, to_np(ty, dt).ravel(), ref.ravel(), 1, RTOL[dt])
    assert bad == 0, f"{bad} elements beyond tolerance (max abs {ma}, max rel {mr})"


@pytest.mark.parametrize("n", (1, 2, 4, 8, 16))
@pytest.mark.parametrize("dt", (D.Dtype.BF16, D.Dtype.F32))
def test_rmsnorm_small(cuda, orc, n, dt):
    for rows in (1, 7, 8, 37, 300):
        for hidden in (n * 8 * (2 if dt == D.Dtype.BF16 else 1) * k for k in (1, 4, 16)):
            if hidden // n * (2 if dt == D.Dtype.BF16 else 4) > 2048:
                continue
            run(cuda, orc, dt, rows, hidden, n, seed=rows + hidden)


def test_rmsnorm_config3(cuda, orc):
    """bf16 4096 x 4096, w ~ N(1, 0.02), eps 1e-6, cluster 8."""
    run(cuda, orc, D.Dtype.BF16, 4096, 4096, 8, seed=0)


@pytest.mark.parametrize("n", (2, 8))
def test_rmsnorm_residual(cuda, orc, n):
    for dt in (D.Dtype.BF16, D.Dtype.F32):
        run(cuda, orc, dt, 129, 2048 if dt == D.Dtype.BF16 else 1024, n, residual=True, seed=3)


@pytest.mark.parametrize("n,hidden,rows", ((2, 1024, 16 * 1000 + 5), (8, 4096, 8192 + 3), (16, 4096, 5000)))
def test_rmsnorm_many_groups_per_cluster(cuda, orc, n, hidden, rows):
    """Many 16-row groups per cluster (interleaved over the clusters, the last one partial), launched
    three times in a row; a skipped group would keep the NaN the output starts with."""
    for seed in (11, 12, 13):
        run(cuda, orc, D.Dtype.BF16, rows, hidden, n, seed=seed)


def test_rmsnorm_many_groups_residual(cuda, orc):
    run(cuda, orc, D.Dtype.BF16, 9001, 2048, 8, residual=True, seed=13)
    run(cuda, orc, D.Dtype.F32, 9001, 1024, 4, residual=True, seed=14)


def test_rmsnorm_tp_shape(cuda, orc):
    """The hidden size of BASELINE config 5 (8192, bf16) at cluster 8 (2 KiB per CTA row slice)."""
    run(cuda, orc, D.Dtype.BF16, 64, 8192, 8, seed=5)


def test_rmsnorm_rejects_bad_shapes(cuda):
    torch = cuda
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(100, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(D.DsmemError) as e:
        D.rmsnorm(x, w, cluster_size=8)
    assert e.value.status == D.Status.ILLEGAL_CONFIG


def test_rmsnorm_launch_order_of_shapes(cuda, orc):
    """One kernel (2 units per lane) with a larger, a smaller and again the larger shared-memory size: the
    kernel's dynamic shared-memory opt-in only grows, so the third launch still fits."""
    for hidden in (4096, 3072, 4096):
        run(cuda, orc, D.Dtype.BF16, 40, hidden, 8, seed=hidden)


@pytest.mark.parametrize("dt,n", ((D.Dtype.BF16, 8), (D.Dtype.BF16, 16), (D.Dtype.F32, 16)))
def test_rmsnorm_reference_golden(cuda, orc, dt, n):
    """The kernel on the pinned fixture's inputs (64 x 8192, exact in fp16 and bf16) against the reference's own
    outputs: its wrapper's fp32 expression, and (when recorded) its RMSNormKernel's fp16 output on a B200. Cluster
    sizes whose row slice fits the kernel's 2 KiB per CTA."""
    import importlib.util
    import pathlib

    torch = cuda
    golden = pathlib.Path(__file__).resolve().parent / "golden"
    spec = importlib.util.spec_from_file_location("make_rmsnorm_golden", golden / "make_rmsnorm_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    d = dict(np.load(golden / "rmsnorm_golden.npz"))
    x, w = mod.inputs()
    if dt == D.Dtype.BF16:
        tx, tw = torch.from_numpy(x).to(torch.bfloat16).cuda(), torch.from_numpy(w).to(torch.bfloat16).cuda()
    else:
        tx, tw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    ty = torch.full_like(tx, float("nan"))
    D.rmsnorm(tx, tw, float(d["eps"]), cluster_size=n, out=ty)
    torch.cuda.synchronize()
    D.rmsnorm_check()
    got = ty.float().cpu().numpy()[d["kept_rows"]].astype(np.float64)
    refs = {"reference fp32 expression": d["y_expr"].astype(np.float64)}
    if "y_kernel_fp16" in d:
        refs["reference RMSNormKernel (fp16)"] = d["y_kernel_fp16"].view(np.float16).astype(np.float64)
    for name, ref in refs.items():
        err = (np.abs(got - ref) / (1.0 + np.abs(ref))).max()
        # bf16 output rounding (2^-9 relative) for bf16; fp32 rounding, plus the fp16 reference's own
        # rounding (2^-11) when comparing with the kernel
        tol = RTOL[dt] if dt == D.Dtype.BF16 else (1e-5 if "expression" in name else 2e-3)
        assert err <= tol, f"{name}: max rel {err:.3e} > {tol}"
