"""Timing of the exact top-k kernel at the reference's shapes (python -m dsmem_b200.topk_bench).

Shapes of roofline/workloads/hpcops_topk_cluster8.yaml (k = 2048; randn rows, seeded, generated on the device):
m8_n32k, m16_n64k, m8_n240k. The `reps` launches are captured once in a CUDA graph and replayed; the per-launch
time is the median over trials of replay time / reps (the logits stay in the L2 across launches, as in the
reference's own measurement loop, which calls hpc.topk back to back). H100 column: the reference's
topk_filtered_cluster8_exact_kernel on H100 NVL, median nsys kernel time (roofline/results/points.csv).
"""
from __future__ import annotations

import argparse
import json
import statistics

import dsmem_b200 as D

SHAPES = {"m8_n32k": (8, 32768), "m16_n64k": (16, 65536), "m8_n240k": (8, 244650)}
H100_US = {"m8_n32k": 12.8, "m16_n64k": 19.616, "m8_n240k": 26.624}


def measure(torch, name, n_cta, k=2048, reps=50, trials=5):
    m, n = SHAPES[name]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(m * n)
    x = torch.randn(m, n, device="cuda", generator=gen)
    out = torch.empty(m, k, dtype=torch.int32, device="cuda")
    for _ in range(3):
        D.topk(x, k=k, cluster_size=n_cta, out=out)
    torch.cuda.synchronize()
    D.topk_check()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for _ in range(reps):
            D.topk(x, k=k, cluster_size=n_cta, out=out)
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
    D.topk_check()
    del graph
    us = statistics.median(times) * 1e3
    return {"shape": name, "m": m, "n": n, "k": k, "cluster_size": n_cta, "us": round(us, 2),
            "rows_per_s": round(m / (us * 1e-6), 1), "min_hbm_bytes": m * n * 4 + m * k * 4,
            "h100_us": H100_US[name], "vs_h100": round(H100_US[name] / us, 3)}


def profile_launches(torch, plan=(("m16_n64k", 4), ("m8_n240k", 8)), warm=3):
    """The launch sequence an ncu capture selects from: `warm` launches of each (shape, cluster) of `plan` in turn,
    then one more of each (so `-s warm*len(plan) -c len(plan)` captures one warm launch per shape)."""
    data = {}
    for name, c in plan:
        m, n = SHAPES[name]
        gen = torch.Generator(device="cuda")
        gen.manual_seed(m * n)
        data[name] = (torch.randn(m, n, device="cuda", generator=gen),
                      torch.empty(m, 2048, dtype=torch.int32, device="cuda"), c)
    for name in [nm for nm, _ in plan for _ in range(warm)] + [nm for nm, _ in plan]:
        x, out, c = data[name]
        D.topk(x, k=2048, cluster_size=c, out=out)
    torch.cuda.synchronize()
    D.topk_check()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--clusters", default="4,8,16")
    ap.add_argument("--profile-launches", action="store_true",
                    help="no timing: 3 launches each of m16_n64k (cluster 4) and m8_n240k (cluster 8), then one more of "
                         "each, for an ncu capture with -s 6 -c 2")
    args = ap.parse_args(argv)
    import torch

    torch.cuda.set_device(0)
    if args.profile_launches:
        profile_launches(torch)
        return
    for s in args.shapes.split(","):
        for c in map(int, args.clusters.split(",")):
            try:
                r = measure(torch, s, c)
            except D.DsmemError as e:
                r = {"shape": s, "cluster_size": c, "skip": str(e)}
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
