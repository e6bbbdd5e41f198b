"""SM-to-SM (DSMEM) traffic of the catalogue: a closed-form model per algorithm, and ncu evidence against it.

The model gives the cluster-wide payload one problem moves between the shared memories of different CTAs
(bulk pushes, st.async, remote stores, remote loads and remote atomics; local copies and mbarrier signals are
not payload), from each algorithm's rounds, partners and message sizes -- the same quantities the reference's
per-file table lists (collectives/README.md:19-49) and its harness replays (collectives/harness/
traffic_model.py). With M elements per rank block and B bytes per element (the payload convention of
msg_elems), "sent once to every peer" is (N-1) M B per CTA.

    python -m dsmem_b200.traffic run --out cases.json [--problems 64]
        launches, once each, the kernel AUTO picks for batches of every (op, N) at 16 and 64 KiB per CTA, then the
        consumer kernels (RMSNorm, top-k, the TP kernel emulated on one GPU); meant to run under
        ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum,
              l1tex__m_l1tex2xbar_write_bytes_mem_dshared.sum,l1tex__m_xbar2l1tex_read_bytes_mem_dshared.sum
    python -m dsmem_b200.traffic run --ops reduce,gather,scatter --every-alg --out cases.json
        the same for the named ops only, every legal algorithm (no consumers)
    python -m dsmem_b200.traffic summarize --cases cases.json --ncu launches.csv [--peaks peaks.json]
        pairs the captured launches with the cases (in order) and prints the markdown table of profiles/.
"""
from __future__ import annotations

import argparse
import csv
import json
import math

from . import Alg, Dtype, Op, autotune_pick, msg_elems

ELEM = {Dtype.F32: 4, Dtype.BF16: 2, Dtype.I32: 4}


def _log2(n):
    return int(round(math.log2(n)))


def dsmem_bytes(op, alg, n, p, dtype):
    """Cluster-wide SM-to-SM payload bytes of one problem (all N CTAs), or None if the algorithm is unknown."""
    op, alg, dtype = Op(op), Alg(alg), Dtype(dtype)
    m = msg_elems(op, n, p, dtype)
    blk = m * ELEM[dtype]           # one rank block, bytes
    lg = _log2(n)
    everyone = n * (n - 1) * blk    # every CTA sends its block to every peer
    if op == Op.ALLREDUCE:
        acc = 4 * m if dtype == Dtype.BF16 else blk   # remote atomics accumulate bf16 in fp32
        return {Alg.RING: 2 * (n - 1) * blk, Alg.RING_CREDIT: 2 * (n - 1) * blk,
                Alg.RECURSIVE_DOUBLING: n * lg * blk, Alg.RECURSIVE_DOUBLING_CREDIT: n * lg * blk,
                Alg.SHIFT_ACCUMULATE_BULK: n * (n - 2) * blk, Alg.SHIFT_ACCUMULATE_BULK_CREDIT: n * (n - 2) * blk,
                Alg.SHIFT_ACCUMULATE_ATOMIC: n * max(1, n - 2) * acc,
                Alg.DIRECT_REPLICATED_PUSH: everyone, Alg.ONE_SHOT_PULL: everyone,
                Alg.ATOMIC_ALL_PUSH: n * (n - 1) * acc,
                Alg.PULL_REDUCE_SCATTER_PUSH_ALLGATHER: 2 * (n - 1) * blk,
                Alg.RABENSEIFNER: 2 * (n - 1) * blk, Alg.RABENSEIFNER_CREDIT: 2 * (n - 1) * blk,
                Alg.TWO_SHOT_PUSH: 2 * (n - 1) * blk,
                Alg.REDUCE_BCAST_BINOMIAL: 2 * (n - 1) * blk, Alg.BINOMIAL_CREDIT: 2 * (n - 1) * blk, Alg.RS_PUSH_GLOBAL_AG: (n - 1) * blk,
                Alg.MESH_2D: _mesh2d(n, blk)}.get(alg)
    if op == Op.ALLGATHER:
        if alg in (Alg.GATHER_BCAST_BINOMIAL, Alg.BINOMIAL_CREDIT):
            return (n // 2) * lg * blk + (n - 1) * n * blk
        return everyone if alg in (Alg.RECURSIVE_DOUBLING, Alg.RECURSIVE_DOUBLING_CREDIT, Alg.DIRECT_SHIFT,
                                   Alg.DIRECT_REPLICATED_PUSH, Alg.RING, Alg.RING_CREDIT, Alg.BRUCK,
                                   Alg.BRUCK_CREDIT, Alg.DIRECT_PULL) else None
    if op == Op.REDUCESCATTER:
        return everyone if alg in (Alg.RING, Alg.RING_CREDIT, Alg.RECURSIVE_HALVING, Alg.RECURSIVE_HALVING_CREDIT,
                                   Alg.DIRECT_PUSH, Alg.DIRECT_PULL) else None
    if op == Op.ALLTOALL:
        if alg in (Alg.BRUCK, Alg.BRUCK_CREDIT):
            return n * (n // 2) * lg * blk
        return everyone if alg in (Alg.PAIRWISE_EXCHANGE, Alg.DIRECT_PUSH, Alg.PAIRWISE_XOR, Alg.PAIRWISE_XOR_CREDIT,
                                   Alg.SHIFT, Alg.DIRECT_PULL) else None
    if op == Op.BROADCAST:
        return (n - 1) * blk if alg in (Alg.DIRECT_PUSH, Alg.DIRECT_PULL, Alg.BINOMIAL) else None
    if op in (Op.REDUCE, Op.GATHER, Op.SCATTER):
        if alg in (Alg.DIRECT_PUSH, Alg.DIRECT_PULL) or (op == Op.REDUCE and alg == Alg.BINOMIAL):
            return (n - 1) * blk   # every non-root block crosses once (a reduce tree sends one partial per rank)
        if alg == Alg.BINOMIAL:
            return (n // 2) * lg * blk   # each round moves N/2 blocks (gather up, or scatter down, the tree)
        return None
    return None


def _mesh2d(n, blk):
    """R x C grid (allreduce__2d_mesh__generic.cu's Grid2D): row reduce-scatter push, column AllReduce push,
    row all-gather push, chunk M / C: per CTA (2 (C-1) + (R-1)) chunks."""
    r = 4 if n >= 16 else (2 if n >= 4 else 1)
    c = n // r
    return n * (2 * (c - 1) + (r - 1)) * (blk // c)


CAPTURE_OPS = (Op.ALLREDUCE, Op.ALLGATHER, Op.REDUCESCATTER, Op.ALLTOALL, Op.BROADCAST)
CAPTURE_SIZES = (2, 4, 8, 16)
CAPTURE_PAYLOADS = (16384, 65536)


def cases(ops=None, every_alg=False):
    """The captured configurations, in launch order: the AUTO batch pick of each (op, N, P) of CAPTURE_OPS, the
    two-shot beside it, and the consumers; with `ops`, the collectives of those ops only (no consumers), and with
    `every_alg`, every registered algorithm legal at that (N, P) instead of AUTO's pick."""
    from . import CATALOGUE, EXTENSIONS, Status, query

    out = []
    for op in (ops or CAPTURE_OPS):
        for n in CAPTURE_SIZES:
            for p in CAPTURE_PAYLOADS:
                if every_alg:
                    algs = [a for (o, a) in list(CATALOGUE) + list(EXTENSIONS)
                            if o == op and query(op, a, Dtype.F32, n, p)[0] == Status.OK]
                else:
                    algs = [autotune_pick(op, Dtype.F32, n, p, num_clusters=64)]
                for alg in algs:
                    if alg != Alg.AUTO:
                        out.append({"kind": "collective", "op": op.name, "alg": alg.name, "n": n, "p": p,
                                    "dtype": "F32"})
    if ops:
        return out
    for n in (8, 16):   # the DSMEM-bound two-shot beside the HBM-bound pick, for the SM-to-SM fraction
        c = {"kind": "collective", "op": "ALLREDUCE", "alg": "TWO_SHOT_PUSH", "n": n, "p": 65536, "dtype": "F32"}
        if c not in out:
            out.append(c)
    out.append({"kind": "rmsnorm", "rows": 4096, "hidden": 4096, "n": 8})
    out.append({"kind": "topk", "rows": 16, "cols": 65536, "k": 2048, "n": 4})
    out.append({"kind": "tp_emulate", "tp": 8, "rows": 1024, "hidden": 8192, "n": 8})
    return out


def run(problems=64, out=None, ops=None, every_alg=False):
    """Launch every case once (a synchronisation between cases), recording the list."""
    import torch

    from . import collective, in_elems_per_rank, out_elems_per_rank, rmsnorm, tp_emulate, topk

    torch.cuda.set_device(0)
    todo = cases(ops, every_alg)
    for c in todo:
        if c["kind"] == "collective":
            op, alg, n, p = Op[c["op"]], Alg[c["alg"]], c["n"], c["p"]
            m = msg_elems(op, n, p, Dtype.F32)
            x = torch.rand(problems * n * in_elems_per_rank(op, n, m), device="cuda")
            y = torch.empty(problems * n * out_elems_per_rank(op, n, m), device="cuda")
            torch.cuda.synchronize()
            collective(op, alg, x, y, n, p)
            c.update(problems=problems, model_bytes_per_problem=dsmem_bytes(op, alg, n, p, Dtype.F32),
                     dram_algorithmic=(x.numel() + y.numel()) * 4)
        elif c["kind"] == "rmsnorm":
            x = torch.randn(c["rows"], c["hidden"], device="cuda").to(torch.bfloat16)
            w = torch.ones(c["hidden"], device="cuda", dtype=torch.bfloat16)
            torch.cuda.synchronize()
            rmsnorm(x, w, 1e-6, cluster_size=c["n"])
            # payload: each CTA st.asyncs one fp32 partial per row to every CTA of the cluster, itself included
            # (16-byte st.async, four rows at a time; the counter counts whole 32-byte sectors: 2x the payload)
            c.update(model_bytes=c["rows"] * c["n"] * c["n"] * 4, dram_algorithmic=2 * x.numel() * 2)
        elif c["kind"] == "topk":
            x = torch.randn(c["rows"], c["cols"], device="cuda")
            torch.cuda.synchronize()
            topk(x, k=c["k"], cluster_size=c["n"])
            c.update(model_bytes=None, dram_algorithmic=x.numel() * 4 + c["rows"] * c["k"] * 4)
        else:
            xs = [torch.randn(c["rows"], c["hidden"], device="cuda").to(torch.bfloat16) for _ in range(c["tp"])]
            ys = [torch.empty_like(xs[0]) for _ in range(c["tp"])]
            w = torch.ones(c["hidden"], device="cuda", dtype=torch.bfloat16)
            torch.cuda.synchronize()
            tp_emulate(xs, ys, w, 1e-6, cluster_size=c["n"])
            # payload as the RMSNorm's, in 8-byte st.async (two rows at a time: 4x in 32-byte sectors)
            c.update(model_bytes=c["rows"] * c["n"] * c["n"] * 4,
                     dram_algorithmic=(c["tp"] + c["tp"]) * xs[0].numel() * 2)
        torch.cuda.synchronize()
    if out:
        with open(out, "w") as f:
            json.dump(todo, f)
    return todo


def _ncu_rows(path):
    """{launch index: {metric: value in base units}} of an ncu --csv metrics log, user kernels only."""
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "nsecond": 1, "usecond": 1e3, "msecond": 1e6,
             "second": 1e9}
    lines = [ln for ln in open(path) if not ln.startswith("==")]
    launches = {}
    for r in csv.DictReader(lines):
        name = r.get("Kernel Name", "")
        if not (name.startswith("void dsb::") or "dsmem" in name or "rmsnorm" in name or "topk" in name
                or "tp_allreduce" in name or "rowwise" in name or "batch_kernel" in name or "_kernel<" in name):
            continue
        key = int(r["ID"])
        v = float(r["Metric Value"].replace(",", ""))
        d = launches.setdefault(key, {"kernel": name})
        d[r["Metric Name"]] = v * scale.get(r["Metric Unit"], 1)
    return [launches[k] for k in sorted(launches)]


def summarize(cases_path, ncu_path, peaks=None):
    todo = json.load(open(cases_path))
    got = _ncu_rows(ncu_path)
    if len(got) != len(todo):
        raise SystemExit(f"{len(got)} captured launches for {len(todo)} cases")
    peaks = peaks or {}
    hbm = peaks.get("hbm_gbs")
    rows = ["| case | kernel | time us | DSMEM sent (counter) | model | counter/model | DSMEM GB/s | DRAM bytes / algorithmic | HBM GB/s |",
            "|---|---|---:|---:|---:|---:|---:|---:|---:|"]
    for c, g in zip(todo, got):
        t_ns = g.get("gpu__time_duration.sum", float("nan"))
        sent = g.get("l1tex__m_l1tex2xbar_write_bytes_mem_dshared.sum", float("nan"))
        dram = g.get("dram__bytes_read.sum", 0.0) + g.get("dram__bytes_write.sum", 0.0)
        if c["kind"] == "collective":
            label = f"{c['op'].lower()} N={c['n']} {c['p'] // 1024} KiB x{c['problems']}: {c['alg'].lower()}"
            model = c["model_bytes_per_problem"] * c["problems"] if c["model_bytes_per_problem"] else None
        else:
            label = f"{c['kind']} " + " ".join(f"{k}={c[k]}" for k in ("rows", "hidden", "cols", "k", "tp", "n") if k in c)
            model = c.get("model_bytes")
        ratio = f"{sent / model:.3f}" if model else "-"
        kname = g["kernel"].split("(")[0].replace("void ", "")[:70]
        rows.append(f"| {label} | `{kname}` | {t_ns / 1e3:.1f} | {sent / 1e6:.3f} MB | "
                    f"{(model or 0) / 1e6:.3f} MB | {ratio} | {sent / t_ns:.0f} | "
                    f"{dram / c['dram_algorithmic']:.3f} | {dram / t_ns:.0f}{f' ({dram / t_ns / hbm:.2f})' if hbm else ''} |")
    return "\n".join(rows)


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--out", default="traffic_cases.json")
    r.add_argument("--problems", type=int, default=64)
    r.add_argument("--ops", default=None, help="comma list of op names (e.g. reduce,gather,scatter): those ops only")
    r.add_argument("--every-alg", action="store_true", help="every legal algorithm, not only AUTO's batch pick")
    s = sub.add_parser("summarize")
    s.add_argument("--cases", required=True)
    s.add_argument("--ncu", required=True)
    s.add_argument("--peaks", default=None)
    a = ap.parse_args(argv)
    if a.cmd == "run":
        ops = tuple(Op[o.upper()] for o in a.ops.split(",")) if a.ops else None
        todo = run(a.problems, a.out, ops, a.every_alg)
        print(f"{len(todo)} cases launched -> {a.out}")
    else:
        peaks = json.load(open(a.peaks)) if a.peaks else None
        print(summarize(a.cases, a.ncu, peaks))


if __name__ == "__main__":
    main()
