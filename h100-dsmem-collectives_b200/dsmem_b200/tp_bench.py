"""Timing of the tensor-parallel AllReduce + RMSNorm on the GPUs of one node.

    torchrun --nnodes 1 --nproc-per-node 2 --master-addr 127.0.0.1 -m dsmem_b200.tp_bench

(run from the package directory, or with it on PYTHONPATH). Per rank: bf16 x [T x 8192] ~ N(0,1) with
seed + rank; the residual ~ N(0,1) and w ~ N(1, 0.02) from one seed shared by every rank (a TP layer's
normalisation weight and residual stream are replicated); eps 1e-6, cluster 8, T in {1, 64, 1024, 8192}. For each T:
  fused          dsmem_tp_allreduce_rmsnorm with x already in the context's x region and y left in its y
                 region (the zero-copy use: a producer writes x there, a consumer reads y there), the form the
                 context's default one-shot limit picks;
  fused_api      the same call from ordinary tensors (the two-shot copies x in and y out on the stream; the
                 one-shot reads and writes them in place);
  fused_twoshot  `fused` with the two-shot form forced (limit 0);
  fused_oneshot  `fused` with the one-shot form forced (where the tensor fits one LL slot);
  nccl           the composition: ncclAllReduce (bf16 sum) then the cluster RMSNorm
                 (dsmem_tp_allreduce_rmsnorm_nccl).
Each figure is the median over rounds of the mean over `reps` calls captured in one CUDA graph (so the
host's launch overhead is not timed), CUDA events on the replay stream, max over ranks. NVLink roofline of a
bandwidth-optimal AllReduce without in-switch reduction: each direction of a rank's links carries 2 (TP-1)/TP
of the tensor (the (TP-1)/TP its peers read or receive in the reduce-scatter, and the (TP-1)/TP it sends in the
all-gather), so the bound is 2 (TP-1)/TP * T*H*2 bytes / 770 GB/s (measured peer-copy bandwidth per direction on
this pool); frac = that time / measured time (= busbw / 770).
"""
from __future__ import annotations

import json
import statistics

NVLINK_GBS = 770.0
HIDDEN = 8192
TOKENS = (1, 64, 1024, 8192)


def _device_errors(ctx, dev_index):
    """(any error, text) of this rank's TP error words and RMSNorm error bits, read and cleared; no raise."""
    import ctypes

    from . import Status, lib

    st, bits, detail = ctx.status()
    rbits = ctypes.c_uint(0)
    rst = lib().dsmem_rmsnorm_check(int(dev_index), ctypes.byref(rbits))
    bad = st != Status.OK or rst != 0 or bool(rbits.value & 1)
    return bad, f"tp {st.name} (bits {bits:#x}, detail {detail:#x}), rmsnorm bits {rbits.value:#x}"


def run(tokens=TOKENS, hidden=HIDDEN, cluster=8, reps=20, rounds=5, warmup=5, on_tokens=None):
    """Times every case of every token count; returns the table. Every rank takes the same collective steps:
    device errors (a cross-GPU wait that gave up) are agreed on by an all-reduce after each token count, and
    all ranks stop together, with the table's row saying so, instead of one rank raising alone.
    on_tokens(ctx, tokens, hidden, cluster, x, w): called on every rank after each token count's timing (a
    result check, for instance); its return value goes into the row as "check"."""
    import torch
    import torch.distributed as dist

    from . import tp as T

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)      # x: each rank's own
    shared = torch.Generator(device=dev)
    shared.manual_seed(4321)          # w and the residual: the same on every rank (drawn in the same order)
    tmax = max(tokens)
    ctx = T.TPContext(T.tp_bytes(tmax, hidden))
    comm = T.NcclComm()
    w = (1 + 0.02 * torch.randn(hidden, device=dev, generator=shared)).to(torch.bfloat16)
    out = {}
    try:
        for t in tokens:
            x = torch.randn(t, hidden, device=dev, generator=gen).to(torch.bfloat16)
            res = torch.randn(t, hidden, device=dev, generator=shared).to(torch.bfloat16)
            y = torch.empty_like(x)
            xb, yb = ctx.buffers(t, hidden)
            xb.copy_(x)
            sum_buf = torch.empty_like(x)
            zero_copy = lambda: _zero_copy(ctx, w, res, t, hidden, cluster)   # noqa: E731
            cases = {   # name: (one-shot limit, call)
                "fused": (T.ONESHOT_DEFAULT, zero_copy),
                "fused_api": (T.ONESHOT_DEFAULT,
                              lambda: ctx.allreduce_rmsnorm(x, w, 1e-6, residual=res, out=y, cluster_size=cluster)),
                "fused_twoshot": (0, zero_copy),
                "nccl": (T.ONESHOT_DEFAULT,
                         lambda: comm.allreduce_rmsnorm(x, w, sum_buf, y, 1e-6, residual=res, cluster_size=cluster)),
            }
            if world > 1 and ctx.oneshot_fits(t, hidden):
                cases["fused_oneshot"] = (2 ** 62, zero_copy)
            row = {}
            for name, (limit, fn) in cases.items():
                ctx.set_oneshot_limit(limit)
                stream = torch.cuda.Stream()
                with torch.cuda.stream(stream):
                    for _ in range(warmup):
                        fn()
                torch.cuda.synchronize()
                dist.barrier()
                # `reps` calls captured in one CUDA graph, so host launch overhead stays out of the figure
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for _ in range(reps):
                        fn()
                torch.cuda.synchronize()
                dist.barrier()
                vals = []
                for _ in range(rounds):
                    with torch.cuda.stream(stream):
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                        graph.replay()
                        e1.record()
                    torch.cuda.synchronize()
                    vals.append(e0.elapsed_time(e1) * 1e3 / reps)
                del graph
                us = torch.tensor([statistics.median(vals)], device=dev)
                dist.all_reduce(us, op=dist.ReduceOp.MAX)
                us = us.item()
                size = t * hidden * 2
                bound_us = 2 * (world - 1) / world * size / (NVLINK_GBS * 1e9) * 1e6
                row[name] = {"us": round(us, 2), "algbw_GBps": round(size / (us * 1e-6) / 1e9, 1),
                             "busbw_GBps": round(size / (us * 1e-6) / 1e9 * 2 * (world - 1) / world, 1),
                             "nvlink_frac": round(bound_us / us, 4) if world > 1 else None}
                if name == "fused":
                    row[name]["form"] = "one-shot" if world > 1 and ctx.oneshot_picked(t, hidden) else "two-shot"
            ctx.set_oneshot_limit(T.ONESHOT_DEFAULT)
            if on_tokens is not None:
                row["check"] = on_tokens(ctx, t, hidden, cluster, x, w)
            bad, text = _device_errors(ctx, dev.index)
            flag = torch.tensor([1 if bad else 0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
            out[str(t)] = row
            if flag.item():
                row["error"] = f"device error words set on a rank (this rank: {text}); later token counts not run"
                break
            dist.barrier()
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        ctx.close()
    return {"tp": world, "hidden": hidden, "cluster_size": cluster, "dtype": "bf16", "nvlink_peak_GBps": NVLINK_GBS,
            "tokens": out}


def _zero_copy(ctx, w, res, t, hidden, cluster):
    """The fused call with x already in the x region and y left in the y region."""
    import ctypes

    import torch

    from . import Dtype, _ok, lib

    _ok(lib().dsmem_tp_allreduce_rmsnorm(ctx._ctx, int(Dtype.BF16), None, res.data_ptr(), w.data_ptr(), 1e-6, t,
                                         hidden, int(cluster), None,
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream or None)),
        "dsmem_tp_allreduce_rmsnorm")


def main():
    import datetime
    import os

    import torch
    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        res = run()
        if dist.get_rank() == 0:
            print(json.dumps(res), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
