"""The SM-to-SM traffic model (dsmem_b200.traffic.dsmem_bytes) against schedules replayed here round by round,
and against the per-CTA byte counts of the reference's catalogue table for N = 8, P = 16 KiB (SURVEY-style closed
forms, collectives/README.md:19-49): e.g. two-shot 2(N-1)/N P = 28,672 B per CTA, ring the same, recursive
doubling P log2 N = 49,152 B. CPU only; the GPU counters are compared in profiles/dsmem_traffic_b200.md."""
import math

import pytest

import dsmem_b200 as D
from dsmem_b200 import traffic as T


def replay(op, alg, n, blk):
    """Cluster-wide bytes of a few schedules, replayed as explicit transfers."""
    moves = []
    if (op, alg) == (D.Op.ALLREDUCE, D.Alg.RABENSEIFNER):
        m = blk
        for r in range(n):
            lo, hi, d = 0, m, n // 2
            while d >= 1:
                mid = (lo + hi) // 2
                up = bool(r & d)
                moves.append((hi - mid) if not up else (mid - lo))
                lo = mid if up else lo
                hi = lo + (hi - mid if not up else hi - mid)
                d //= 2
            d = 1
            while d < n:
                moves.append(hi - lo)
                lo, hi = (lo - (hi - lo), hi) if r & d else (lo, hi + (hi - lo))
                d *= 2
    elif (op, alg) == (D.Op.ALLTOALL, D.Alg.BRUCK):
        for r in range(n):
            d = 1
            while d < n:
                moves.append(sum(1 for j in range(n) if j & d) * blk)   # blocks whose index has bit d
                d *= 2
    elif (op, alg) == (D.Op.ALLGATHER, D.Alg.GATHER_BCAST_BINOMIAL):
        d = 1
        while d < n:   # gather: ranks with bit d set send their 2^k accumulated blocks to r - d
            moves += [d * blk] * (n // (2 * d))
            d *= 2
        moves += [n * blk] * (n - 1)   # broadcast of the full buffer
    elif (op, alg) == (D.Op.BROADCAST, D.Alg.BINOMIAL):
        moves += [blk] * (n - 1)
    elif (op, alg) == (D.Op.REDUCE, D.Alg.BINOMIAL):
        d = 1
        while d < n:   # ranks with r mod 2d == d send their one-block partial to r - d
            moves += [blk for r in range(n) if r % (2 * d) == d]
            d *= 2
    elif (op, alg) == (D.Op.GATHER, D.Alg.BINOMIAL):
        d = 1
        while d < n:   # ranks with r mod 2d == d send the d blocks they hold to r - d
            moves += [d * blk for r in range(n) if r % (2 * d) == d]
            d *= 2
    elif (op, alg) == (D.Op.SCATTER, D.Alg.BINOMIAL):
        held = {0: n}   # rank -> blocks it holds (ranks r .. r + held - 1)
        d = n // 2
        while d >= 1:   # ranks holding 2d blocks send the upper d to r + d
            for r in [r for r, h in held.items() if h == 2 * d]:
                moves.append(d * blk)
                held[r], held[r + d] = d, d
            d //= 2
        assert sorted(held) == list(range(n)) and all(h == 1 for h in held.values())
    return sum(moves)


@pytest.mark.parametrize("op,alg", [(D.Op.ALLREDUCE, D.Alg.RABENSEIFNER), (D.Op.ALLTOALL, D.Alg.BRUCK),
                                    (D.Op.ALLGATHER, D.Alg.GATHER_BCAST_BINOMIAL), (D.Op.BROADCAST, D.Alg.BINOMIAL),
                                    (D.Op.REDUCE, D.Alg.BINOMIAL), (D.Op.GATHER, D.Alg.BINOMIAL),
                                    (D.Op.SCATTER, D.Alg.BINOMIAL)])
@pytest.mark.parametrize("n", D.CLUSTER_SIZES)
def test_model_matches_replayed_schedule(op, alg, n):
    p = 16384
    m = D.msg_elems(op, n, p, D.Dtype.F32)
    assert T.dsmem_bytes(op, alg, n, p, D.Dtype.F32) == replay(op, alg, n, m * 4)


def test_model_per_cta_figures_at_n8_16k():
    n, p, f = 8, 16384, D.Dtype.F32
    per_cta = lambda op, alg: T.dsmem_bytes(op, alg, n, p, f) / n   # noqa: E731
    assert per_cta(D.Op.ALLREDUCE, D.Alg.TWO_SHOT_PUSH) == 2 * (n - 1) / n * p == 28672
    assert per_cta(D.Op.ALLREDUCE, D.Alg.RING) == 28672
    assert per_cta(D.Op.ALLREDUCE, D.Alg.RECURSIVE_DOUBLING) == p * math.log2(n) == 49152
    assert per_cta(D.Op.ALLREDUCE, D.Alg.RS_PUSH_GLOBAL_AG) == (n - 1) / n * p
    assert per_cta(D.Op.ALLREDUCE, D.Alg.ONE_SHOT_PULL) == (n - 1) * p
    for op in (D.Op.ALLGATHER, D.Op.REDUCESCATTER, D.Op.ALLTOALL):   # P = N M B: (N-1)/N P per CTA
        assert per_cta(op, D.Alg.DIRECT_PULL) == (n - 1) / n * p
    # rooted: every non-root block crosses once; Reduce P = M B, Gather / Scatter P = N M B
    assert per_cta(D.Op.REDUCE, D.Alg.DIRECT_PUSH) == (n - 1) / n * p
    assert per_cta(D.Op.GATHER, D.Alg.DIRECT_PUSH) == per_cta(D.Op.SCATTER, D.Alg.DIRECT_PULL) == (n - 1) / n ** 2 * p


def test_model_covers_every_registered_algorithm():
    for (op, alg) in list(D.CATALOGUE) + list(D.EXTENSIONS):
        for n in D.CLUSTER_SIZES:
            if D.query(op, alg, D.Dtype.F32, n, 16384)[0] != D.Status.OK:
                continue
            v = T.dsmem_bytes(op, alg, n, 16384, D.Dtype.F32)
            assert v is not None and v > 0, (op, alg, n)
