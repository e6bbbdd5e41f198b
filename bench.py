#!/usr/bin/env python
"""Benchmark of the cluster AllReduce hot path on B200 (one JSON line on rank 0).

Workload (the catalogue sweep, at its AllReduce / cluster-8 point, with the
bytes per CTA of the north-star target; configs[0]'s 16 KiB ring / recursive-doubling numbers are added
under "single_cluster"): a grid-filled batch of independent cluster-8 AllReduce(sum) problems, f32,
P = 64 KiB per CTA, inputs U(-1,1) (seeded). One step = one launch of the persistent batch kernel over
the whole batch (inputs 2 GiB per GPU, far larger than the 126 MB L2, so no flush is needed).
    value        aggregate algbw = (problems x N x P) / step time, whole job (sum over GPUs), GB/s
    e2e          the same metric through the public API on host buffers (dsmem_collective_host): every step
                 copies its input from pinned host memory and its output back, in chunks whose copies in and
                 out overlap; the copies are inside the timed region
    roofline     HBM: algorithmic bytes per launch = problems x N x 2P (read in, write out); `dsmem`: the
                 algorithm's SM-to-SM bytes against the live-measured push ceiling
    cpu_baseline the reference's own reference() (collectives/harness/main.cu, compiled from the reference
                 sources into oracle/_ref/) on all host cores for ~10 s (the C oracle port, 1 thread, if that
                 binary is absent)
    check        a strided sample of the timed batch's own output against the CPU oracle
Extras (rank 0): configs[0]'s single-cluster latencies and its algorithms in a grid-filled batch (f32 and int32),
configs[2]'s RMSNorm, configs[3]'s decoder layer,
ceilings, and at N = 1 the row-wise and top-k consumers, each with a CPU baseline and its core count; at N > 1
every rank also runs configs[4]'s tensor-parallel AllReduce + RMSNorm across the N GPUs, whose result at 64 and
1,024 tokens (one-shot and two-shot forms) is checked against the CPU oracle (tokens.<T>.check).
--impl reference runs the reference's own CPU path (collectives/harness/main.cu reference(), compiled
from the reference sources into oracle/_ref/) on all host cores, same metric and config.
Multi-GPU: one process per GPU (torchrun), each GPU its own batch (weak scaling, no inter-GPU traffic).
"""
import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG = ROOT / "h100-dsmem-collectives_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "cluster AllReduce algbw GB/s & µs vs bytes/CTA; fused RMSNorm rows/s"
CLUSTER_N = 8
PAYLOAD = 65536           # bytes per CTA (f32: M = 16384)
BATCH_BYTES = 2 << 30     # input bytes per GPU per step
HBM_FALLBACK_GBS = 6650.0
# kernels the library launches for a batch (more than one cluster problem) with its pipelined drivers on
KERNEL_NAMES = {"TWO_SHOT_PUSH": "two_shot_pipelined_kernel<AR_TwoShotPipelined<{n},float,Sum>>",
                "RS_PUSH_GLOBAL_AG": "rs_global_ag_stream_kernel<AR_RsGlobalAgStream<{n},float,Sum>>"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--payload", type=int, default=PAYLOAD)
    ap.add_argument("--alg", default="auto")
    ap.add_argument("--no-extras", action="store_true", help="skip the single-cluster latency table")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", HBM_FALLBACK_GBS)), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return HBM_FALLBACK_GBS, "fallback 6.65 TB/s"


def profile_traffic(kernel_key):
    """Per-launch DRAM bytes of the headline kernel from the committed ncu summary, or None."""
    f = ROOT / "profiles" / "ncu_traffic.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_key and not line.startswith("#"):
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv is not None:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus and world > 1:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE {world}")
    return rank, world, local


# --------------------------------------------------------------------------------------------- reference
def run_reference(args, rank, world):
    if rank != 0:
        return
    cfg = {"workload": f"allreduce cluster{CLUSTER_N} {args.payload // 1024}KiB/CTA f32, host reference()",
           "cluster_size": CLUSTER_N, "bytes_per_cta": args.payload, "dtype": "f32"}
    m = args.payload // 4
    exe = ROOT / "oracle" / "_ref" / f"ref_op0_N{CLUSTER_N}_M{m}_float"
    threads = os.cpu_count() or 1
    samples = []
    kind = "reference"
    if exe.exists():
        for i in range(args.warmup + args.steps):
            out = subprocess.run([str(exe), "bench", "0.25" if i < args.warmup else "1.0", str(threads)],
                                 check=True, capture_output=True, text=True).stdout
            d = json.loads(out)
            if i >= args.warmup:
                samples.append(d["problems"] * CLUSTER_N * args.payload / d["seconds"] / 1e9)
        sample_desc = f"reference() of collectives/harness/main.cu on {threads} threads, 1 s per step"
    else:
        kind = "port"
        threads = 1
        samples = [oracle_rate(args.payload, seconds=1.0) for _ in range(args.steps)]
        sample_desc = "oracle port (C), 1 thread, 1 s per step (oracle/_ref not built)"
    v = statistics.median(samples)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (pattern B inputs)",
            "config": cfg,
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                             "sample": sample_desc},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reference_rate(payload, seconds, threads):
    """GB/s of per-CTA payload of the reference's own reference() (oracle/_ref binary) on `threads` host
    threads for ~`seconds`; None if the binary was not built."""
    exe = ROOT / "oracle" / "_ref" / f"ref_op0_N{CLUSTER_N}_M{payload // 4}_float"
    if not exe.exists():
        return None
    out = subprocess.run([str(exe), "bench", str(seconds), str(threads)], check=True, capture_output=True,
                         text=True).stdout
    d = json.loads(out)
    return d["problems"] * CLUSTER_N * payload / d["seconds"] / 1e9


def oracle_rate(payload, seconds):
    """CPU oracle (C, single thread) on a bounded sample: GB/s of per-CTA payload."""
    from oracle import oracle as orc

    n, m, clusters = CLUSTER_N, payload // 4, 16
    host = orc.uniform_real(orc.F32, clusters * n * m, 1, -1.0, 1.0)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        orc.reference(orc.ALLREDUCE, orc.F32, n, m, clusters, host)
        done += clusters
    el = time.perf_counter() - t0
    return done * n * payload / el / 1e9


# --------------------------------------------------------------------------------------------- ours
def single_cluster_latency(torch, D, reps=200):
    """one cluster per launch, N = 8, 16 KiB/CTA f32; in-kernel %globaltimer span
    (max exit - min entry, main.cu:344-349), median over reps, next to the reference's H100 numbers."""
    n, p = 8, 16384
    m = p // 4
    res = {}
    ref_h100 = {"ring": 9024, "recursive_doubling": 4864, "two_shot_push": 1440}
    auto = D.autotune_pick(D.Op.ALLREDUCE, D.Dtype.F32, n, p, 1)
    algs = [("ring", D.Alg.RING), ("recursive_doubling", D.Alg.RECURSIVE_DOUBLING),
            ("two_shot_push", D.Alg.TWO_SHOT_PUSH), ("one_shot_pull", D.Alg.ONE_SHOT_PULL),
            ("ring_credit", D.Alg.RING_CREDIT), ("recursive_doubling_credit", D.Alg.RECURSIVE_DOUBLING_CREDIT),
            ("rs_push_global_ag", D.Alg.RS_PUSH_GLOBAL_AG)]
    if all(a != auto for _, a in algs):
        algs.append((auto.name.lower(), auto))
    for name, alg in algs:
        tin = torch.rand(n * m, device="cuda") * 2 - 1
        tout = torch.empty_like(tin)
        stamps = torch.zeros(n * 32, dtype=torch.int64, device="cuda")
        lat = []
        for i in range(reps + 20):
            D.collective(D.Op.ALLREDUCE, alg, tin, tout, n, p, stamps=stamps)
            if i >= 20:
                st = stamps.view(n, 32)
                lat.append((st[:, 1].max() - st[:, 0].min()).item())
        D.check()
        med = statistics.median(lat)
        res[name] = {"latency_ns_median": med, "algbw_GBps": round(p / med, 3),
                     "busbw_GBps": round(p / med * 2 * (n - 1) / n, 3),
                     "h100_reference_ns": ref_h100.get(name)}
    res["auto_pick"] = auto.name.lower()
    res["timing"] = f"in-kernel span (max exit - min entry stamp), median of {reps} single-cluster launches"
    return res


def config0_batch(torch, D, hbm_peak, reps=5):
    """configs[0]'s algorithms in a grid-filled batch: the ring and recursive-doubling AllReduce and their
    mbarrier-credit forms, N = 8, 4,096 elements (16 KiB) per CTA, f32 U(-1,1) and int32 U[-1000, 1000], 8,192
    problems (1 GiB of input per launch, larger than the L2). CUDA events over `reps` launches after three
    warm-ups; a strided sample of each batch's output against the oracle (int32 bit-exact, f32 within
    1e-5 (1 + |ref|) ceil(log2 N)). Any failure is reported in the entry instead of ending the run."""
    from oracle import oracle as orc

    n, m = 8, 4096
    p = m * 4
    problems = (1 << 30) // (n * p)
    algs = (("ring", D.Alg.RING), ("recursive_doubling", D.Alg.RECURSIVE_DOUBLING),
            ("ring_credit", D.Alg.RING_CREDIT), ("recursive_doubling_credit", D.Alg.RECURSIVE_DOUBLING_CREDIT))
    res = {"problems": problems, "bytes_per_cta": p, "cluster_size": n,
           "timing": f"CUDA events over {reps} launches of the whole batch, after 3 warm-ups"}
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    for dname, odt in (("f32", orc.F32), ("i32", orc.I32)):
        try:
            if odt == orc.F32:
                tin = torch.rand(problems * n * m, device="cuda", generator=g) * 2 - 1
            else:
                tin = torch.randint(-1000, 1001, (problems * n * m,), dtype=torch.int32, device="cuda", generator=g)
            tout = torch.empty_like(tin)
            for name, alg in algs:
                for _ in range(3):
                    D.collective(D.Op.ALLREDUCE, alg, tin, tout, n, p)
                D.check()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    D.collective(D.Op.ALLREDUCE, alg, tin, tout, n, p)
                e1.record()
                torch.cuda.synchronize()
                D.check()
                ms = e0.elapsed_time(e1) / reps
                bad = 0
                for q in sorted({int(i * (problems - 1) / 7) for i in range(8)}):
                    a, b = q * n * m, (q + 1) * n * m
                    ref = orc.reference(orc.ALLREDUCE, odt, n, m, 1, tin[a:b].cpu().numpy())
                    got = tout[a:b].cpu().numpy()
                    bad += (orc.check(odt, got, ref, 0)[0] if odt == orc.I32
                            else orc.check(odt, got, ref, 1, 1e-5 * math.ceil(math.log2(n)))[0])
                res[f"{name}_{dname}"] = {
                    "ms": round(ms, 4), "algbw_GBps": round(problems * n * p / (ms * 1e-3) / 1e9, 1),
                    "hbm_frac": round(2 * problems * n * p / (ms * 1e-3) / 1e9 / hbm_peak, 4),
                    "check": {"problems_checked": 8, "bad_elements": int(bad), "ok": bad == 0}}
            del tin, tout
        except Exception as err:  # noqa: BLE001 -- reported in the line; the headline stands
            res[f"error_{dname}"] = f"{type(err).__name__}: {err}"
    torch.cuda.empty_cache()
    return res


def rmsnorm_config3(torch, D, hbm_peak, reps=50):
    """bf16 [4096 x 4096] ~ N(0,1), w ~ N(1, 0.02), eps 1e-6, cluster 8 per row.
    The 64 MiB of traffic fits the 126 MB L2, so every launch must start from cold rows (the reference's
    flush_l2: true, roofline/workloads/clusterfusion_rmsnorm.yaml:42): launches rotate over four (x, y)
    pairs, 256 MiB in all. The `reps` launches are captured once in a CUDA graph and replayed: a ~15 us
    kernel launched one call at a time from Python is bound by the host's launch rate, not by the GPU."""
    T, H, n = 4096, 4096, 8
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    # four (x, y) pairs, 256 MiB in all, used in rotation: each launch reads rows that left the L2 two
    # launches ago, so no flush kernel is needed and launches run back to back on the stream
    xs = [torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4)]
    ys = [torch.empty_like(xs[0]) for _ in range(4)]
    w = (1 + 0.02 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
    for i in range(8):
        D.rmsnorm(xs[i % 4], w, 1e-6, cluster_size=n, out=ys[i % 4])
    torch.cuda.synchronize()

    def timed(run):
        times = []
        for _ in range(5):
            torch.cuda._sleep(200_000)   # the host enqueues while the stream is busy
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / reps)
        return statistics.median(times)

    def stream_loop():
        for i in range(reps):
            D.rmsnorm(xs[i % 4], w, 1e-6, cluster_size=n, out=ys[i % 4])

    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        stream_loop()
    graph.replay()
    torch.cuda.synchronize()
    ms = timed(graph.replay)
    ms_stream = timed(stream_loop)
    D.rmsnorm_check()
    del graph
    algo = 2 * T * H * 2 + 2 * H   # read x, write y, read w (clusterfusion_rmsnorm.yaml:14 at bf16)
    gbs = algo / (ms * 1e-3) / 1e9
    return {"workload": "rmsnorm bf16 4096x4096 cluster8, cold L2 (4 rotating buffer pairs, 256 MiB)",
            "kernel_us_median": round(ms * 1e3, 3), "timing": f"CUDA graph of {reps} back-to-back launches",
            "stream_launch_us_median": round(ms_stream * 1e3, 3),
            "rows_per_s": round(T / (ms * 1e-3), 1), "hbm_GBps": round(gbs, 1),
            "hbm_frac": round(gbs / hbm_peak, 4), "algorithmic_bytes": algo, "reps": reps,
            "h100_reference_us": {"clusterfusion_cluster2_fp16_64x8192": 3.78}}


def dsmem_ceiling(D, n):
    """Measured SM-to-SM bandwidth at cluster size n (1/slope, GB/s): ring and all-peers push, in the
    reference's one-CTA-per-SM shape and with four CTAs per SM; the peak is the best of them."""
    out = {}
    for cps in (1, 4):
        for mode, name in ((1, "push_ring"), (2, "push_all_peers")):
            gbs, _ = D.dsmem_bandwidth_peak(mode, n, ctas_per_sm=cps)
            out[f"{name}_{cps}cta_GBps"] = round(gbs, 1)
    out["peak_GBps"] = max(out.values())
    return out


# Row-wise reduction-reuse workloads (kernels/*__reduction_reuse__credit.cu) at the middle reference shape
# (16384 columns), each at the cluster size measured fastest there; the full table is
# `python -m dsmem_b200.rowwise_bench`.
ROWWISE_BENCH = {"rowwise_quant": 2, "lars_momentum": 4, "layernorm_backward": 2, "pearson_backward": 2,
                 "softmax_logits_backward": 4, "weighted_var_backward": 4}
# Exact top-2048 (hpc-ops topk_filtered_cluster8) at the reference's three shapes, cluster size per shape.
TOPK_BENCH = {"m8_n32k": 8, "m16_n64k": 4, "m8_n240k": 8}


def rowwise_extras(torch, hbm_peak):
    from dsmem_b200 import rowwise_bench as RB

    out = {}
    for w, n in ROWWISE_BENCH.items():
        r = RB.measure(torch, w, 16384, n, hbm_peak)
        out[w] = {k: r[k] for k in ("rows", "cols", "cluster_size", "us", "hbm_GBps", "hbm_frac", "h100_us")}
        torch.cuda.empty_cache()
    return out


def topk_extras(torch):
    from dsmem_b200 import topk_bench as TB

    out = {}
    for s, n in TOPK_BENCH.items():
        r = TB.measure(torch, s, n)
        out[s] = {k: r[k] for k in ("m", "n", "k", "cluster_size", "us", "h100_us", "vs_h100")}
    return out


# SM-to-SM shots per problem: the two-shot pushes 2 (N-1)/N * P per CTA, the reduce-scatter with the all-gather
# through the outputs (N-1)/N * P
DSMEM_SHOTS = {"TWO_SHOT_PUSH": 2, "RS_PUSH_GLOBAL_AG": 1}


def check_sample(torch, tin, tout, n, m, problems, samples=16):
    """A strided sample of the timed batch's problems against the CPU oracle (the restatement of the reference's
    reference() and check(), main.cu:129-173): |got - ref| <= 1e-5 (1 + |ref|) ceil(log2 N)."""
    from oracle import oracle as orc

    picks = sorted(set(int(i * (problems - 1) / max(1, samples - 1)) for i in range(samples)))
    bad, worst = 0, 0.0
    for q in picks:
        a, b = q * n * m, (q + 1) * n * m
        host = tin[a:b].cpu().numpy()
        ref = orc.reference(orc.ALLREDUCE, orc.F32, n, m, 1, host)
        nb, _, mr = orc.check(orc.F32, tout[a:b].cpu().numpy(), ref, 1, 1e-5 * math.ceil(math.log2(n)))
        bad += nb
        worst = max(worst, mr)
    return {"problems_checked": len(picks), "of": problems, "bad_elements": bad, "max_rel_err": worst,
            "tolerance": f"1e-5*(1+|ref|)*ceil(log2 N) (main.cu:165)", "ok": bad == 0}


def headline_cpu_baseline(p):
    """The reference's own reference() on all host threads for ~10 s (the reference arm's measurement, on the
    same box in the same run); the C oracle port on one thread if the reference binary was not built."""
    threads = os.cpu_count() or 1
    v = reference_rate(p, 10.0, threads)
    if v is not None:
        return {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                "sample": f"reference() of collectives/harness/main.cu (oracle/_ref build), one cluster problem of "
                          f"the same shape per thread, {threads} threads, ~10 s"}
    v = oracle_rate(p, seconds=10.0)
    return {"value": round(v, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "oracle reference() restatement (C), 1 thread, 16 cluster problems of the same shape, 10 s"}


def _timed(fn, seconds):
    """(calls, elapsed s) of fn() repeated for at least `seconds`."""
    done, t0 = 0, time.perf_counter()
    while True:
        fn()
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            return done, el


def cpu_extras(extras, p):
    """CPU baselines beside the extras (rank 0, N = 1): the reference's own reference() where it exists, else the
    oracle's restatement, single-threaded, on a bounded sample of each workload, scaled to its unit."""
    import numpy as np

    from oracle import oracle as orc

    if "single_cluster" in extras:
        exe = ROOT / "oracle" / "_ref" / f"ref_op0_N{CLUSTER_N}_M4096_float"
        if exe.exists():
            d = json.loads(subprocess.run([str(exe), "bench", "2.0", "1"], check=True, capture_output=True,
                                          text=True).stdout)
            extras["single_cluster"]["cpu_baseline"] = {
                "value": round(d["seconds"] / d["problems"] * 1e9, 1), "unit": "ns per problem", "cores": 1,
                "kind": "reference", "sample": "reference() of main.cu, N = 8, 16 KiB per CTA, 1 thread, ~2 s"}
    if "config0_batch" in extras:
        threads = os.cpu_count() or 1
        v = reference_rate(16384, 3.0, threads)
        if v is not None:
            extras["config0_batch"]["cpu_baseline"] = {
                "value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                "sample": f"reference() of main.cu (oracle/_ref build), N = 8, 16 KiB per CTA, f32, one problem per "
                          f"thread, {threads} threads, ~3 s"}
    if "rmsnorm" in extras:
        x = orc.normal(1, 512 * 4096, 0, 0.0, 1.0).reshape(512, 4096)
        w = orc.normal(1, 4096, 1, 1.0, 0.02)
        calls, el = _timed(lambda: orc.rmsnorm(1, x, w, 1e-6), 2.0)
        extras["rmsnorm"]["cpu_baseline"] = {
            "value": round(calls * 512 / el, 1), "unit": "rows/s", "cores": 1, "kind": "port",
            "sample": "oracle RMSNorm (clusterfusion_rmsnorm.py:65 in double), 512 of the 4096 bf16 rows, ~2 s"}
    if "decoder" in extras:
        from dsmem_b200 import decoder_bench as DB

        h, f, S = DB.HID, DB.FFN, DB.S
        block = orc.f32_to_bf16(np.random.default_rng(0).standard_normal(1 << 20).astype(np.float32) * 0.02)
        fill = lambda *shape: np.resize(block, int(np.prod(shape))).reshape(shape)   # noqa: E731
        inv = 10000.0 ** (-np.arange(0, 128, 2) / 128)
        cs = np.concatenate([np.cos(S * inv)] * 2).astype(np.float32)
        sn = np.concatenate([np.sin(S * inv)] * 2).astype(np.float32)
        args = (fill(1, h), fill(1, h), fill(h), fill(3 * h, h), fill(h, h), fill(h), fill(2 * f, h), fill(h, f),
                fill(1, S + 1, DB.HEADS, 128), fill(1, S + 1, DB.HEADS, 128), cs, sn, S, 1e-5, DB.HEADS)
        calls, el = _timed(lambda: orc.decoder_layer(*args), 1.0)
        extras["decoder"]["cpu_baseline"] = {
            "value": round(calls / el, 2), "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": "oracle decoder layer (reference_fp32 of clusterfusion_llama2_7b_decoder.py:160-180 with the "
                      "FFN tail, in double), batch 1, full Llama-2-7B shape, S = 4096"}
    rng = np.random.default_rng(0)
    for w_, r in extras.get("rowwise", {}).items():
        rows, cols, k = r["rows"], r["cols"], 16
        a = lambda: rng.standard_normal((k, cols)).astype(np.float32)   # noqa: E731
        fn = {"rowwise_quant": (lambda x=a(): orc.rowwise_quant(x)),
              "lars_momentum": (lambda w=a(), g=a(), m_=a(): orc.lars_momentum(w, g, m_, **orc.LARS_DEFAULTS)),
              "layernorm_backward": (lambda x=a(), dy=a(): orc.layernorm_backward(x, dy, np.ones(cols, np.float32),
                                                                                  orc.LN_BWD_EPS)),
              "pearson_backward": (lambda x=a(), y=a(): orc.pearson_backward(x, y, np.ones(k, np.float32),
                                                                           orc.PEARSON_EPS)),
              "softmax_logits_backward": (lambda z=a(), dy=a(): orc.softmax_logits_backward(z, dy)),
              "weighted_var_backward": (lambda x=a(), wt=np.abs(a()), dy=a(): orc.weighted_var_backward(
                  x, wt, dy, orc.WVAR_EPS))}[w_]
        calls, el = _timed(fn, 0.5)
        r["cpu_baseline"] = {"value": round(el / calls * rows / k * 1e6, 1), "unit": "us", "cores": 1,
                             "kind": "port", "sample": f"oracle restatement, {k} of the {rows} rows, scaled"}
    for s_, r in extras.get("topk", {}).items():
        k = min(2, r["m"])
        x = rng.standard_normal((k, r["n"])).astype(np.float32)
        calls, el = _timed(lambda: orc.topk_values(x, r["k"]), 0.5)
        r["cpu_baseline"] = {"value": round(el / calls * r["m"] / k * 1e6, 1), "unit": "us", "cores": 1,
                             "kind": "port", "sample": f"oracle top-k values, {k} of the {r['m']} rows, scaled"}


def decoder_extras(torch, hbm_peak):
    """the Llama-2-7B decoder layer, one decode step, batch 1 / 4 / 16 (cluster-8 projections; the
    attention's cluster size follows the (sequence, head) count), CUDA-graph-timed; tokens/s and HBM fraction."""
    from dsmem_b200 import decoder_bench as DB

    r = DB.run(batches=(1, 4, 16), clusters=(8,), with_torch=False)
    out = {"config": r["config"], "timing": "CUDA graph of 10 steps, median of 5 replays"}
    for b, row in r["batch"].items():
        out[f"batch{b}"] = {**row["cluster8"], "bytes_per_step": row["bytes_per_step"]}
    torch.cuda.empty_cache()
    return out


def tp_check(torch, rank, world, ctx, tokens, hidden, cluster, x, w):
    """The fused call's result at 64 tokens (the one-shot form) and 1,024 (the two-shot) against the CPU oracle:
    y = RMSNorm(sum of every rank's x) * w without a residual, from a NaN-filled output (w is the same on every
    rank, as in a TP layer); every rank's y gathered to rank 0, which checks them bit-identical and within
    1e-2 * (1 + |ref|) (bf16 output). Every rank takes the same steps; None at other token counts and on ranks
    other than 0."""
    if tokens not in (64, 1024):
        return None
    import numpy as np
    import torch.distributed as dist

    y = torch.full_like(x, float("nan"))
    ctx.allreduce_rmsnorm(x, w, 1e-6, residual=None, out=y, cluster_size=cluster)
    torch.cuda.synchronize()
    xs = [torch.empty_like(x) for _ in range(world)]
    ys = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(xs, x)
    dist.all_gather(ys, y)
    if rank != 0:
        return None
    form = "one-shot" if ctx.oneshot_picked(tokens, hidden) else "two-shot"
    try:   # rank 0 alone from here: nothing may raise past this point, or the ranks' steps would part
        from oracle import oracle as orc

        def bits(t):
            return t.cpu().view(torch.int16).numpy().view(np.uint16)

        ref = orc.tp_rmsnorm(1, [bits(a) for a in xs], bits(w), 1e-6)
        got = [bits(a) for a in ys]
        same = all(np.array_equal(g, got[0]) for g in got[1:])
        bad, _, mr = orc.check(1, got[0].reshape(-1), ref.reshape(-1), 1, 1e-2)
    except Exception as err:  # noqa: BLE001 -- reported in the line
        return {"ok": False, "form": form, "error": f"{type(err).__name__}: {err}"}
    return {"ok": bool(bad == 0 and same), "form": form, "bad_elements": int(bad), "max_rel": float(mr),
            "ranks_bit_identical": bool(same),
            "oracle": "oracle.tp_rmsnorm (sum of the ranks' x in double, RMSNorm, x w), tol 1e-2 (1 + |ref|)"}


def tp_extras(torch, rank, world):
    """tensor-parallel AllReduce + RMSNorm over the N GPUs (bf16, hidden 8192, tokens 1 / 64 / 1024 /
    8192): the fused peer-memory call (its default form, each form forced, and from ordinary tensors) and the NCCL
    composition; max over ranks, CUDA-graph-timed, with the NVLink fraction; a CPU baseline on rank 0."""
    from dsmem_b200 import tp_bench as TB

    try:
        r = TB.run(reps=10, rounds=3, warmup=3, on_tokens=lambda *a: tp_check(torch, rank, world, *a))
    except Exception as err:  # noqa: BLE001 -- raised alike on every rank (argument or launch errors); the
        r = {"error": f"{type(err).__name__}: {err}"}   # headline line is still printed
    torch.cuda.empty_cache()
    if rank == 0:
        import numpy as np

        from oracle import oracle as orc

        xs = [orc.normal(1, 64 * 8192, 7 + k, 0.0, 1.0).reshape(64, 8192) for k in range(world)]
        w = orc.normal(1, 8192, 1, 1.0, 0.02)
        calls, el = _timed(lambda: orc.tp_rmsnorm(1, xs, w, 1e-6), 1.0)
        r["cpu_baseline"] = {"value": round(calls * 64 / el, 1), "unit": "tokens/s", "cores": 1, "kind": "port",
                             "sample": f"oracle sum of {world} ranks + RMSNorm (double), 64 tokens x 8192, ~1 s"}
        del np
    return r


def run_ours(args, rank, world, local):
    import torch

    import dsmem_b200 as D

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    n, p = CLUSTER_N, args.payload
    m = p // 4
    alg = D.Alg[args.alg.upper()] if args.alg.lower() != "auto" else D.Alg.AUTO
    problems = BATCH_BYTES // (n * p)
    # AUTO picks per launch shape: the batch regime of the table for a launch of `problems` clusters.
    resolved = D.autotune_pick(D.Op.ALLREDUCE, D.Dtype.F32, n, p, problems) if alg == D.Alg.AUTO else alg
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    tin = torch.rand(problems * n * m, device=dev, generator=g) * 2 - 1
    tout = torch.empty_like(tin)
    stream = torch.cuda.current_stream(dev)

    def step():
        D.collective(D.Op.ALLREDUCE, alg, tin, tout, n, p, stream=stream.cuda_stream)

    for _ in range(max(3, args.warmup)):
        step()
    D.check(stream.cuda_stream)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    D.check(stream.cuda_stream)
    ms = e0.elapsed_time(e1) / args.steps
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
        dist.barrier()
    payload_bytes = problems * n * p                     # per GPU per step
    value = world * payload_bytes / (ms * 1e-3) / 1e9    # GB/s, whole job
    hbm_peak, peak_src = peaks()
    algo_bytes = problems * n * 2 * p                    # read in + write out, one launch
    achieved = algo_bytes / (ms * 1e-3) / 1e9
    kernel_key = f"allreduce_{resolved.name.lower()}_N{n}_P{p}_f32"
    traffic = profile_traffic(kernel_key)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                "peak_source": peak_src, "algorithmic_bytes_per_launch": algo_bytes,
                "kernel": KERNEL_NAMES.get(resolved.name, f"batch_kernel<AR_{resolved.name}<{n},float,Sum>>")
                .format(n=n)}

    # End to end through the public API on HOST buffers: dsmem_collective_host streams the step's input in,
    # runs the batch and streams the result out, the copies in and out of neighbouring chunks overlapping on
    # their own copy engines (one synchronous call per step; host wall clock around the calls, after a device
    # synchronise, max over ranks). Its output is checked against the device step's result for the same
    # input; should the call fail or differ, the sequential form (H2D, launch, D2H on one stream, CUDA events)
    # is measured instead and the line says so.
    hin = torch.empty(tin.numel(), dtype=torch.float32, pin_memory=True)
    hin.copy_(tin)
    hout = torch.empty(tout.numel(), dtype=torch.float32, pin_memory=True)
    e2e_steps = max(2, min(args.steps, 5))
    e2e_mode = "dsmem_collective_host (chunked, copies overlapped)"
    try:
        D.collective_host(D.Op.ALLREDUCE, alg, hin, hout, n, p)
        pick = torch.arange(0, tout.numel(), 1021, device=dev)
        if not torch.equal(hout[pick.cpu()], tout[pick].cpu()):
            raise RuntimeError("host-buffer result differs from the device step's")
    except Exception as err:  # noqa: BLE001 -- any failure of the host-buffer path falls back, and says so
        e2e_mode = f"sequential on one stream (dsmem_collective_host: {err})"
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if e2e_mode.startswith("dsmem_collective_host"):
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            D.collective_host(D.Op.ALLREDUCE, alg, hin, hout, n, p)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
    else:
        def e2e_step():
            tin.copy_(hin, non_blocking=True)
            step()
            hout.copy_(tout, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        a1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1) / e2e_steps
        D.check(stream.cuda_stream)
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    e2e = {"value": round(world * payload_bytes / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": tin.numel() * 4, "d2h_bytes_per_step": tout.numel() * 4,
           "ms_per_step": round(e2e_ms, 3), "mode": e2e_mode}

    # shared::cluster roofline: bytes each CTA sends per problem (two-shot: 2(N-1)/N * P; the reduce-scatter
    # with the all-gather through the outputs: (N-1)/N * P) against the measured push ceiling at this size
    ceil = dsmem_ceiling(D, n)
    dsmem_bytes = problems * n * DSMEM_SHOTS.get(resolved.name, 2) * (n - 1) / n * p
    dsmem_achieved = dsmem_bytes / (ms * 1e-3) / 1e9
    roofline["dsmem"] = {"achieved": round(dsmem_achieved, 1), "peak": ceil["peak_GBps"], "unit": "GB/s",
                         "frac": round(dsmem_achieved / ceil["peak_GBps"], 4),
                         "bytes_per_launch": int(dsmem_bytes), "ceilings": ceil,
                         "peak_source": "measured live (dsmem_ceiling_dsmem_bw, best push shape, 1/slope)"}

    # the timed batch's own output, sampled, against the CPU oracle (every rank; outside the timed region)
    check = check_sample(torch, tin, tout, n, m, problems)

    extras = {}
    if world > 1 and not args.no_extras:
        # tensor-parallel AllReduce + RMSNorm across the N GPUs (every rank takes part)
        extras["tp_allreduce_rmsnorm"] = tp_extras(torch, rank, world)
    if rank == 0 and not args.no_extras:
        extras["single_cluster"] = single_cluster_latency(torch, D)
        extras["config0_batch"] = config0_batch(torch, D, hbm_peak)
        extras["rmsnorm"] = rmsnorm_config3(torch, D, hbm_peak)
        # ceilings beyond DSMEM and HBM (tcgen05 MMA, L2, shared memory), 1 / slope over two work amounts
        extras["ceilings_sm100"] = D.sm100_ceilings(reps=3)
        if world == 1:   # kept out of multi-GPU runs, where the other GPUs wait meanwhile
            extras["decoder"] = decoder_extras(torch, hbm_peak)
            extras["rowwise"] = rowwise_extras(torch, hbm_peak)
            extras["topk"] = topk_extras(torch)

    cpu = None
    if rank == 0 and world == 1:
        cpu = headline_cpu_baseline(p)
        if not args.no_extras:
            cpu_extras(extras, p)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic U(-1,1)",
            "config": {"workload": f"allreduce cluster{n} {p // 1024}KiB/CTA f32, grid-filled persistent batch",
                       "alg": resolved.name.lower(), "cluster_size": n, "bytes_per_cta": p,
                       "problems_per_gpu": problems, "input_bytes_per_gpu": problems * n * p,
                       "l2": "inputs 2 GiB per GPU > 126 MB L2 (no flush)", "parallelism": f"shard{world}"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps,
            "clocks": clocks.summary(), "check": check}
    line.update(extras)
    print(json.dumps(line), flush=True)
    if not check["ok"]:
        raise SystemExit(f"result check failed: {check}")


def main():
    args = parse()
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
