"""Generate tests/golden/rmsnorm_golden.npz, pinning the RMSNorm oracle to the reference twice.

Step `expr` (where the reference checkout is mounted, CPU only): the reference's RMSNorm wrapper checks its kernels
against an fp32 torch expression, `y32` in check() of roofline/harness/workloads/clusterfusion_rmsnorm.py:62-66.
This step reads that function's source, takes the expression assigned to y32 and the module's EPS, and evaluates
them with torch on the CPU -- the reference's own code, without importing the module (which needs a GPU and
flashinfer). Outputs are kept for every eighth row; the inputs are regenerated from the oracle's seeded draws. Inputs: 64 x 8192 rows (the compiled shape of the reference kernel), x ~ N(0, 1) and w ~ N(1, 0.02)
(the oracle's seeded draws) rounded to grids that are exact in both fp16 (the reference's dtype) and bf16: x = k / 32 with |k| <= 128, w = 1 +
k / 128 with |k| <= 8.

Step `kernel` (on a GPU box, after `make -C oracle ref-rmsnorm`): runs the reference's own RMSNormKernel
(kernels/rmsnorm__llama__clusterfusion.cu, included unmodified by oracle/ref_rmsnorm.cu: fp16, cluster of 2 per
row, one remote atomicAdd) on the same inputs and adds its fp16 output to the fixture.

    python tests/golden/make_rmsnorm_golden.py expr            # needs $REF or BASELINE.json's reference_path
    python tests/golden/make_rmsnorm_golden.py kernel [out]    # needs a GPU and oracle/_ref/librmsnorm_ref.so

The fixture is committed; tests never need the reference or its library at run time.
"""
import ast
import ctypes
import hashlib
import json
import os
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "rmsnorm_golden.npz"
ROWS, HIDDEN = 64, 8192
KEEP = slice(0, ROWS, 8)   # outputs are stored for every eighth row (8 rows), to keep the fixture small


def reference_root():
    ref = os.environ.get("REF") or json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
    if not ref or not pathlib.Path(ref).is_dir():
        raise SystemExit("set REF to the reference checkout")
    return pathlib.Path(ref)


def inputs():
    """x ~ N(0, 1) and w ~ N(1, 0.02) from the oracle's seeded draws (mt19937_64, Box-Muller), on grids exact in
    fp16 and bf16. The tests regenerate them with this function and check the SHA-256 stored in the fixture."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as orc

    x = orc.normal(0, ROWS * HIDDEN, 20261202, 0.0, 1.0).astype(np.float64).reshape(ROWS, HIDDEN)
    w = orc.normal(0, HIDDEN, 20261203, 1.0, 0.02).astype(np.float64)
    x = np.clip(np.rint(x * 32), -128, 128) / 32
    w = 1 + np.clip(np.rint((w - 1) * 128), -8, 8) / 128
    return x.astype(np.float32), w.astype(np.float32)


def step_expr():
    import torch

    src_path = reference_root() / "roofline" / "harness" / "workloads" / "clusterfusion_rmsnorm.py"
    tree = ast.parse(src_path.read_text())
    eps = next(ast.literal_eval(n.value) for n in tree.body
               if isinstance(n, ast.Assign) and any(getattr(t, "id", None) == "EPS" for t in n.targets))
    check = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "check")
    expr = next(n.value for n in ast.walk(check)
                if isinstance(n, ast.Assign) and any(getattr(t, "id", None) == "y32" for t in n.targets))
    code = compile(ast.Expression(expr), str(src_path), "eval")
    x, w = inputs()
    xh, wh = torch.from_numpy(x).to(torch.float16), torch.from_numpy(w).to(torch.float16)
    assert np.array_equal(xh.float().numpy(), x) and np.array_equal(wh.float().numpy(), w), "inputs not exact in fp16"
    assert not (x.view(np.uint32) & 0xFFFF).any() and not (w.view(np.uint32) & 0xFFFF).any(), "not exact in bf16"
    # the names the expression uses in check(): xf = x.float(), w (fp16), EPS, torch
    y32 = eval(code, {"torch": torch, "EPS": eps}, {"xf": xh.float(), "w": wh}).numpy()
    np.savez_compressed(OUT, eps=np.float64(eps), y_expr=y32[KEEP].astype(np.float32),
                        kept_rows=np.arange(ROWS)[KEEP],
                        expr=np.array(ast.unparse(expr)),
                        x_sha256=np.array(hashlib.sha256(x.tobytes()).hexdigest()),
                        w_sha256=np.array(hashlib.sha256(w.tobytes()).hexdigest()))
    print("wrote", OUT, "expression:", ast.unparse(expr), "EPS =", eps)


def step_kernel(out):
    import torch

    d = dict(np.load(OUT))
    xs, ws = inputs()
    assert hashlib.sha256(xs.tobytes()).hexdigest() == str(d["x_sha256"]), "regenerated x differs from the fixture's"
    L = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "librmsnorm_ref.so"))
    r, h, cs = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    L.ref_rmsnorm_shape(ctypes.byref(r), ctypes.byref(h), ctypes.byref(cs))
    assert (r.value, h.value) == (ROWS, HIDDEN), (r.value, h.value)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(xs).to(torch.float16).to(dev)
    w = torch.from_numpy(ws).to(torch.float16).to(dev)
    y = torch.full_like(x, float("nan"))
    L.ref_rmsnorm_launch.argtypes = [ctypes.c_void_p] * 3
    rc = L.ref_rmsnorm_launch(x.data_ptr(), w.data_ptr(), y.data_ptr())
    assert rc == 0, f"reference kernel launch failed ({rc})"
    d["y_kernel_fp16"] = y.cpu().numpy().view(np.uint16)[KEEP]
    d["kernel_cluster_size"] = np.int64(cs.value)
    np.savez_compressed(out, **d)
    print("wrote", out, "cluster", cs.value)


if __name__ == "__main__":
    if len(sys.argv) >= 2 and sys.argv[1] == "expr":
        step_expr()
    elif len(sys.argv) >= 2 and sys.argv[1] == "kernel":
        step_kernel(sys.argv[2] if len(sys.argv) > 2 else OUT)
    else:
        raise SystemExit(__doc__)
