"""Catalogue sweep on one B200 and the measured AUTO table.

    python -m dsmem_b200.sweep [--out-table autotune_b200.tsv] [--out-json sweep.json] [--dtype f32]
                               [--ops allreduce,...] [--regime both|single] [--merge old_table.tsv]

For every op x algorithm x cluster size N in {2, 4, 8, 16} x bytes per CTA P in {256 B .. 128 KiB, 192 KiB}
(the reference sweep's grid, driver.py:156-163) that is legal, two figures:
  single   one cluster per launch, as the reference harness runs it (collectives/harness/main.cu): the
           in-kernel span max(stamp[1]) - min(stamp[0]) over the N CTAs (%globaltimer), median of
           `--reps` launches; algbw = P / span, busbw = algbw * the op's bus factor (perf_report.py:99-100:
           AllReduce 2(N-1)/N, the others (N-1)/N);
  batch    a grid-filled batch of independent problems (enough for four full waves of resident clusters and
           at least `--batch-mib` MiB of input, default 256: pipelined drivers need many problems per resident
           cluster to reach their steady state), CUDA events over `--batch-reps` launches; algbw = problems * N *
           P / time (the whole batch's per-CTA payloads, as bench.py's value).
The AUTO table (one line per (op, N, P, dtype, regime) with the fastest algorithm) is the input of
dsmem_autotune_table_load; regime `single` picks by span, `batch` by batch throughput. `--regime single` measures
the single figure only (every algorithm, a few seconds per op), and `--merge` then replaces only the table's
single lines of the swept (op, dtype): the way to enter latency variants without re-running the batch regime.
"""
from __future__ import annotations

import argparse
import json
import statistics

from . import (CATALOGUE, CLUSTER_SIZES, EXTENSIONS, STAMPS_PER_RANK, Alg, Dtype, DsmemError, Op, Status, check,
               collective, in_elems_per_rank, max_active_clusters, msg_elems, out_elems_per_rank, query)

PAYLOADS = [256 << k for k in range(10)] + [196608]
BUS = {Op.ALLREDUCE: lambda n: 2 * (n - 1) / n, Op.ALLGATHER: lambda n: (n - 1) / n,
       Op.REDUCESCATTER: lambda n: (n - 1) / n, Op.ALLTOALL: lambda n: (n - 1) / n,
       Op.BROADCAST: lambda n: 1.0, Op.REDUCE: lambda n: 1.0,   # nccl-tests: broadcast / reduce busbw = algbw
       Op.GATHER: lambda n: (n - 1) / n, Op.SCATTER: lambda n: (n - 1) / n}
OP_NAMES = {Op.ALLREDUCE: "allreduce", Op.ALLGATHER: "allgather", Op.REDUCESCATTER: "reducescatter",
            Op.ALLTOALL: "alltoall", Op.BROADCAST: "broadcast", Op.REDUCE: "reduce", Op.GATHER: "gather",
            Op.SCATTER: "scatter"}
DT_NAMES = {Dtype.F32: "f32", Dtype.BF16: "bf16", Dtype.I32: "i32"}
ALG_NAMES = {a: (a.name.lower() if a != Alg.MESH_2D else "2d_mesh") for a in Alg}   # dsmem_alg_name()
# (op, alg) with a pipelined or streamed driver: they also run payloads whose one-piece buffers exceed shared memory
PIPELINED = {(Op.ALLREDUCE, Alg.TWO_SHOT_PUSH), (Op.ALLREDUCE, Alg.RS_PUSH_GLOBAL_AG),
             (Op.REDUCESCATTER, Alg.DIRECT_PUSH), (Op.ALLTOALL, Alg.DIRECT_PUSH),
             (Op.ALLGATHER, Alg.DIRECT_REPLICATED_PUSH)}


def measure(torch, op, alg, n, p, dt, reps, batch_reps, buf_in, buf_out, stamps, batch_bytes=256 << 20,
            batch=True):
    m = msg_elems(op, n, p, dt)
    per_in = n * in_elems_per_rank(op, n, m)
    per_out = n * out_elems_per_rank(op, n, m)
    tdt = {Dtype.F32: torch.float32, Dtype.BF16: torch.bfloat16, Dtype.I32: torch.int32}[dt]
    esz = {Dtype.F32: 4, Dtype.BF16: 2, Dtype.I32: 4}[dt]
    inp = buf_in[: per_in * esz].view(tdt)
    out = buf_out[: per_out * esz].view(tdt)
    # single: `reps` launches, each with its own stamp slice, read back once
    st = stamps[: reps * n * STAMPS_PER_RANK].view(reps, n * STAMPS_PER_RANK)
    for r in range(reps):
        collective(op, alg, inp, out, n, p, num_clusters=1, stamps=st[r])
    check()
    s = st.view(reps, n, STAMPS_PER_RANK).cpu()
    spans = (s[:, :, 1].max(dim=1).values - s[:, :, 0].min(dim=1).values).tolist()
    span_ns = statistics.median(spans[min(5, reps // 4):])
    algbw_single = p / span_ns
    single = {"span_ns": round(span_ns, 1), "algbw_GBps": round(algbw_single, 3),
              "busbw_GBps": round(algbw_single * BUS[op](n), 3)}
    if not batch:
        return single
    # batch: four waves of resident clusters, at least batch_bytes of input, within the buffers
    try:
        res = max_active_clusters(op, alg, dt, n, p)
    except DsmemError:   # a payload only the pipelined driver runs: size the batch by bytes alone
        res = 1
    problems = max(4 * res, batch_bytes // (per_in * esz))
    problems = min(problems, buf_in.numel() // (per_in * esz), buf_out.numel() // (per_out * esz))
    inp = buf_in[: problems * per_in * esz].view(tdt)
    out = buf_out[: problems * per_out * esz].view(tdt)
    for _ in range(2):
        collective(op, alg, inp, out, n, p, num_clusters=problems)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(batch_reps):
        collective(op, alg, inp, out, n, p, num_clusters=problems)
    e1.record()
    torch.cuda.synchronize()
    check()
    ms = e0.elapsed_time(e1) / batch_reps
    return {**single, "batch_problems": problems, "batch_ms": round(ms, 4),
            "batch_algbw_GBps": round(problems * n * p / (ms * 1e-3) / 1e9, 1)}


def run(dtypes=(Dtype.F32,), reps=60, batch_reps=5, sizes=CLUSTER_SIZES, payloads=PAYLOADS, ops=tuple(Op),
        batch_bytes=256 << 20, batch=True):
    import torch

    torch.cuda.set_device(0)
    buf_in = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    buf_out = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    buf_in.random_(0, 64)   # small positive bytes: finite floats, no overflow in int sums
    stamps = torch.zeros(reps * 16 * STAMPS_PER_RANK, dtype=torch.int64, device="cuda")
    algs = [k for k in list(CATALOGUE) + list(EXTENSIONS) if k[0] in ops]
    results = []
    for dt in dtypes:
        for (op, alg) in algs:
            for n in sizes:
                for p in payloads:
                    qs = query(op, alg, dt, n, p)[0]
                    if qs != Status.OK and not (qs == Status.SMEM_LIMIT and (op, alg) in PIPELINED):
                        continue
                    try:
                        r = measure(torch, op, alg, n, p, dt, reps, batch_reps, buf_in, buf_out, stamps, batch_bytes,
                                    batch=batch)
                    except DsmemError as e:
                        r = {"error": str(e)}
                    r.update({"op": OP_NAMES[op], "alg": ALG_NAMES[alg], "n": n, "bytes": p, "dtype": DT_NAMES[dt]})
                    results.append(r)
    return results


def merge(old_text, new_text, results, regimes=("single", "batch")):
    """The lines of `old_text` whose (op, dtype, regime) the sweep `results` did not cover, then `new_text`'s."""
    covered = {(r["op"], r["dtype"]) for r in results}
    keep = [ln for ln in old_text.splitlines()
            if ln.strip() and not ln.startswith("#")
            and ((ln.split()[0], ln.split()[3]) not in covered or ln.split()[5] not in regimes)]
    new = [ln for ln in new_text.splitlines() if ln.strip() and not ln.startswith("#")]
    head = "# op cluster_size bytes_per_cta dtype alg regime  (measured on B200 by dsmem_b200.sweep)"
    key = lambda ln: (ln.split()[0], int(ln.split()[1]), int(ln.split()[2]), ln.split()[3], ln.split()[5])
    return "\n".join([head] + sorted(keep + new, key=key)) + "\n"


def table(results):
    """Fastest algorithm per (op, N, P, dtype, regime)."""
    best = {}
    for r in results:
        if "error" in r:
            continue
        for regime, key, better in (("single", "span_ns", lambda a, b: a < b),
                                    ("batch", "batch_algbw_GBps", lambda a, b: a > b)):
            if key not in r:
                continue
            k = (r["op"], r["n"], r["bytes"], r["dtype"], regime)
            if k not in best or better(r[key], best[k][key]):
                best[k] = r
    lines = ["# op cluster_size bytes_per_cta dtype alg regime  (measured on B200 by dsmem_b200.sweep)"]
    for (op, n, p, dt, regime), r in sorted(best.items()):
        lines.append(f"{op} {n} {p} {dt} {r['alg']} {regime}")
    return "\n".join(lines) + "\n"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out-table", default="autotune_b200.tsv")
    ap.add_argument("--out-json", default="sweep_b200.json")
    ap.add_argument("--dtype", default="f32", choices=["f32", "bf16", "i32", "all"])
    ap.add_argument("--reps", type=int, default=60)
    ap.add_argument("--ops", default="all", help="comma list of allreduce,allgather,reducescatter,alltoall,broadcast,reduce,gather,scatter")
    ap.add_argument("--merge", default=None, help="existing table: keep its lines for the (op, dtype) not swept")
    ap.add_argument("--batch-mib", type=int, default=256, help="input MiB of each batch-regime launch (at least)")
    ap.add_argument("--regime", default="both", choices=["both", "single"],
                    help="single: one cluster per launch only (no batch launches; --merge keeps the batch lines)")
    args = ap.parse_args(argv)
    dts = {"f32": (Dtype.F32,), "bf16": (Dtype.BF16,), "i32": (Dtype.I32,),
           "all": (Dtype.F32, Dtype.BF16, Dtype.I32)}[args.dtype]
    by_name = {v: k for k, v in OP_NAMES.items()}
    ops = tuple(Op) if args.ops == "all" else tuple(by_name[o] for o in args.ops.split(","))
    batch = args.regime == "both"
    res = run(dts, reps=args.reps, ops=ops, batch_bytes=args.batch_mib << 20, batch=batch)
    with open(args.out_json, "w") as f:
        json.dump(res, f)
    text = table(res)
    if args.merge:
        with open(args.merge) as f:
            text = merge(f.read(), text, res, ("single", "batch") if batch else ("single",))
    with open(args.out_table, "w") as f:
        f.write(text)
    print(f"{len(res)} configurations; table -> {args.out_table}; results -> {args.out_json}", flush=True)


if __name__ == "__main__":
    main()
