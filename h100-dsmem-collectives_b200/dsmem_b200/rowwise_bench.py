"""Timing of the row-wise reduction-reuse kernels at the reference's shapes (python -m dsmem_b200.rowwise_bench).

Shapes and bytes follow the reference's roofline workloads (roofline/workloads/credit_<name>.yaml): 4096 rows
(LayerNorm backward: 2048) x {4096, 16384, 65536} fp32 columns; min_hbm_bytes = every array once. Inputs are seeded synthetic N(0, 1)
(weights U(0, 1)), generated on the device. Launches rotate over as many input/output sets as keep 256 MiB or
more between two uses of a set (the reference flushes a 256 MB L2 buffer before every launch), and the `reps`
launches are captured once in a CUDA graph and replayed, so the per-launch time is the device time of
back-to-back launches.
"""
from __future__ import annotations

import argparse
import json
import statistics

import dsmem_b200 as D

COLS = (4096, 16384, 65536)
ROWS = {"layernorm_backward": 2048}   # credit_layernorm_backward.yaml:9-11; the others 4096
# bytes per launch (roofline/workloads/credit_<name>.yaml, min_hbm_bytes)
MIN_HBM_BYTES = {
    "rowwise_quant": lambda r, c: r * c * 5 + r * 4,
    "lars_momentum": lambda r, c: r * c * 20,
    "layernorm_backward": lambda r, c: r * c * 12 + c * 4,
    "pearson_backward": lambda r, c: r * c * 16 + r * 4,
    "softmax_logits_backward": lambda r, c: r * c * 12,
    "weighted_var_backward": lambda r, c: r * c * 16,
}
WORKLOADS = tuple(MIN_HBM_BYTES)
# H100 NVL medians of the reference's clustered kernels at the best P per shape (roofline/results/points.csv,
# cluster_smem rows, nsys kernel time), for context
H100_US = {
    "rowwise_quant": {4096: 45.7, 16384: 120.8, 65536: 513.5},
    "lars_momentum": {4096: 99.7, 16384: 413.8, 65536: 2126.3},
    "layernorm_backward": {4096: 44.5, 16384: 146.9, 65536: 645.0},
    "pearson_backward": {4096: 99.7, 16384: 333.2, 65536: 1466.9},
    "softmax_logits_backward": {4096: 95.9, 16384: 330.8, 65536: 1501.7},
    "weighted_var_backward": {4096: 115.8, 16384: 485.4, 65536: 2399.5},
}


def make_set(torch, workload, rows, cols, gen):
    nrm = lambda *s: torch.randn(*s, device="cuda", generator=gen)  # noqa: E731
    if workload == "rowwise_quant":
        ins = {"x": nrm(rows, cols)}
        outs = {"q": torch.empty(rows, cols, dtype=torch.int8, device="cuda"),
                "s": torch.empty(rows, device="cuda")}
    elif workload == "lars_momentum":
        ins = {"w": nrm(rows, cols), "g": nrm(rows, cols), "m": nrm(rows, cols)}
        outs = {"wo": torch.empty(rows, cols, device="cuda"), "mo": torch.empty(rows, cols, device="cuda")}
    elif workload == "layernorm_backward":
        ins = {"x": nrm(rows, cols), "dy": nrm(rows, cols), "gamma": 1 + 0.1 * nrm(cols)}
        outs = {"dx": torch.empty(rows, cols, device="cuda")}
    elif workload == "pearson_backward":
        ins = {"x": nrm(rows, cols), "y": nrm(rows, cols), "grad": nrm(rows)}
        outs = {"dx": torch.empty(rows, cols, device="cuda"), "dy": torch.empty(rows, cols, device="cuda")}
    elif workload == "softmax_logits_backward":
        ins = {"z": nrm(rows, cols), "dy": nrm(rows, cols)}
        outs = {"dx": torch.empty(rows, cols, device="cuda")}
    else:
        ins = {"x": nrm(rows, cols), "w": torch.rand(rows, cols, device="cuda", generator=gen), "dy": nrm(rows, cols)}
        outs = {"dx": torch.empty(rows, cols, device="cuda")}
    return ins, outs


def launch(workload, ins, outs, n):
    if workload == "rowwise_quant":
        D.rowwise_quant(ins["x"], cluster_size=n, q=outs["q"], scales=outs["s"])
    elif workload == "lars_momentum":
        D.lars_momentum(ins["w"], ins["g"], ins["m"], cluster_size=n, weight_out=outs["wo"], momentum_out=outs["mo"])
    elif workload == "layernorm_backward":
        D.layernorm_backward(ins["x"], ins["dy"], ins["gamma"], cluster_size=n, dx=outs["dx"])
    elif workload == "pearson_backward":
        D.pearson_backward(ins["x"], ins["y"], ins["grad"], cluster_size=n, dx=outs["dx"], dy=outs["dy"])
    elif workload == "softmax_logits_backward":
        D.softmax_logits_backward(ins["z"], ins["dy"], cluster_size=n, dx=outs["dx"])
    else:
        D.weighted_var_backward(ins["x"], ins["w"], ins["dy"], cluster_size=n, dx=outs["dx"])


def rows_of(workload):
    return ROWS.get(workload, 4096)


def measure(torch, workload, cols, n, hbm_peak, rows=None, reps=20, trials=5, sets=None):
    """Median per-launch device time (CUDA graph replay of `reps` launches over rotating sets) and GB/s."""
    rows = rows_of(workload) if rows is None else rows
    nbytes = MIN_HBM_BYTES[workload](rows, cols)
    if sets is None:
        sets = max(1, -(-(256 << 20) // nbytes) + 1)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(cols + n)
    data = [make_set(torch, workload, rows, cols, gen) for _ in range(sets)]
    for i in range(3):
        launch(workload, *data[i % sets], n)
    torch.cuda.synchronize()
    D.rowwise_check()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(reps):
            launch(workload, *data[i % sets], n)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(trials):
        torch.cuda._sleep(200_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / reps)
    D.rowwise_check()
    del graph, data
    ms = statistics.median(times)
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": workload, "rows": rows, "cols": cols, "cluster_size": n, "us": round(ms * 1e3, 2),
            "hbm_GBps": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 4), "min_hbm_bytes": nbytes,
            "input_sets": sets, "h100_us": H100_US[workload][cols]}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workloads", default=",".join(WORKLOADS))
    ap.add_argument("--cols", default=",".join(map(str, COLS)))
    ap.add_argument("--clusters", default="2,4,8")
    ap.add_argument("--hbm-peak", type=float, default=6447.8)
    args = ap.parse_args(argv)
    import torch

    torch.cuda.set_device(0)
    for w in args.workloads.split(","):
        for c in map(int, args.cols.split(",")):
            for n in map(int, args.clusters.split(",")):
                try:
                    r = measure(torch, w, c, n, args.hbm_peak)
                except D.DsmemError as e:
                    r = {"workload": w, "cols": c, "cluster_size": n, "skip": str(e)}
                print(json.dumps(r), flush=True)
                torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
