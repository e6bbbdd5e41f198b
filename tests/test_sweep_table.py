"""The AUTO table builder of dsmem_b200.sweep (host logic, no GPU): the fastest algorithm per (op, N, P, dtype,
regime), and the merge that keeps the lines a partial sweep did not measure."""
from dsmem_b200 import sweep


def _r(op, alg, n, p, dt, span, batch=None):
    r = {"op": op, "alg": alg, "n": n, "bytes": p, "dtype": dt, "span_ns": span}
    if batch is not None:
        r["batch_algbw_GBps"] = batch
    return r


def test_table_picks_fastest_per_regime():
    res = [_r("allreduce", "ring", 8, 256, "f32", 900.0, 10.0), _r("allreduce", "two_shot_push", 8, 256, "f32", 700.0, 9.0),
           _r("allreduce", "bruck", 8, 256, "f32", 800.0, 20.0), {"error": "x", "op": "allreduce"}]
    lines = sweep.table(res).splitlines()[1:]
    assert "allreduce 8 256 f32 two_shot_push single" in lines
    assert "allreduce 8 256 f32 bruck batch" in lines
    assert len(lines) == 2


def test_single_only_sweep_keeps_batch_lines():
    old = ("# header\n"
           "allreduce 8 256 f32 ring single\n"
           "allreduce 8 256 f32 rs_push_global_ag batch\n"
           "allgather 8 256 f32 ring single\n"
           "allreduce 8 256 bf16 ring single\n")
    res = [_r("allreduce", "ring", 8, 256, "f32", 900.0), _r("allreduce", "rabenseifner_credit", 8, 256, "f32", 500.0)]
    new = sweep.table(res)
    assert "batch" not in new   # a single-regime sweep has no batch figure
    merged = sweep.merge(old, new, res, ("single",)).splitlines()
    assert "allreduce 8 256 f32 rabenseifner_credit single" in merged
    assert "allreduce 8 256 f32 ring single" not in merged        # replaced: the swept (op, dtype, regime)
    assert "allreduce 8 256 f32 rs_push_global_ag batch" in merged  # kept: batch not swept
    assert "allgather 8 256 f32 ring single" in merged              # kept: op not swept
    assert "allreduce 8 256 bf16 ring single" in merged             # kept: dtype not swept


def test_full_sweep_replaces_both_regimes():
    old = "allreduce 8 256 f32 ring single\nallreduce 8 256 f32 ring batch\n"
    res = [_r("allreduce", "two_shot_push", 8, 256, "f32", 700.0, 30.0)]
    merged = sweep.merge(old, sweep.table(res), res).splitlines()
    assert "allreduce 8 256 f32 ring batch" not in merged and "allreduce 8 256 f32 two_shot_push batch" in merged
