"""Generate tests/golden/rowwise_golden.npz from the reference's OWN clustered row-wise kernels.

The six kernels of kernels/*__reduction_reuse__credit.cu are included unmodified by oracle/ref_rowwise.cu and
built for the B200 by `make -C oracle ref-rowwise` (here, where the reference is mounted); this script runs them
on cuda:0 -- so it runs on a GPU box -- as the reference launches them (one cluster of P CTAs per row,
256 threads, slice = ceil(cols / P)) on the seeded inputs of tests/rowwise_cases.py, and stores for every
(workload, shape) the SHA-256 of the inputs and the reference's outputs.

    make -C oracle ref-rowwise && python tests/golden/make_rowwise_golden.py [out.npz]

The fixture is committed; tests never need the reference or its library at run time.
"""
import ctypes
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "tests"))

import rowwise_cases as RC  # noqa: E402

LIB = ROOT / "oracle" / "_ref" / "librowwise_ref.so"
LN_EPS, PEARSON_EPS = 1e-5, 1e-5   # the eps the reference harness passes (the kernels' kEps, :29)


def run_case(L, torch, workload, a, rows, cols, p):
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(v).to(dev) for k, v in a.items()}
    f32 = lambda: torch.empty((rows, cols), dtype=torch.float32, device=dev)  # noqa: E731
    vp = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    if workload == "rowwise_quant":
        q = torch.empty((rows, cols), dtype=torch.int8, device=dev)
        sc = torch.empty(rows, dtype=torch.float32, device=dev)
        rc = L.ref_rowwise_quant(vp(t["x"]), vp(q), vp(sc), rows, cols, p)
        outs = (q, sc)
    elif workload == "lars_momentum":
        wo, mo = f32(), f32()
        rc = L.ref_lars_momentum(vp(t["w"]), vp(t["g"]), vp(t["m"]), vp(wo), vp(mo), rows, cols, p)
        outs = (wo, mo)
    elif workload == "layernorm_backward":
        dx = f32()
        rc = L.ref_layernorm_backward(vp(t["x"]), vp(t["dy"]), vp(t["gamma"]), vp(dx), rows, cols,
                                      ctypes.c_float(LN_EPS), p)
        outs = (dx,)
    elif workload == "pearson_backward":
        dx, dy = f32(), f32()
        rc = L.ref_pearson_backward(vp(t["x"]), vp(t["y"]), vp(t["grad"]), vp(dx), vp(dy), rows, cols,
                                    ctypes.c_float(PEARSON_EPS), p)
        outs = (dx, dy)
    elif workload == "softmax_logits_backward":
        dx = f32()
        rc = L.ref_softmax_logits_backward(vp(t["z"]), vp(t["dy"]), vp(dx), rows, cols, p)
        outs = (dx,)
    else:
        dx = f32()
        rc = L.ref_weighted_var_backward(vp(t["x"]), vp(t["w"]), vp(t["dy"]), vp(dx), rows, cols, p)
        outs = (dx,)
    if rc != 0:
        raise RuntimeError(f"{workload} {rows}x{cols} P={p}: launcher returned {rc}")
    return [o.cpu().numpy() for o in outs]


def main(out_path):
    import torch

    L = ctypes.CDLL(str(LIB))
    arrays = {}
    for workload in RC.WORKLOADS:
        for si, (rows, cols, p) in enumerate(RC.GOLDEN_SHAPES):
            a = RC.inputs(workload, rows, cols, RC.case_seed(workload, si))
            outs = run_case(L, torch, workload, a, rows, cols, p)
            key = f"{workload}__{si}"
            arrays[key + "__shape"] = np.array([rows, cols, p], np.int64)
            arrays[key + "__sha256"] = np.array(RC.digest(a))
            for j, o in enumerate(outs):
                arrays[f"{key}__out{j}"] = o
            print(key, rows, cols, p, [o.dtype.name for o in outs])
    np.savez_compressed(out_path, **arrays)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "rowwise_golden.npz"))
