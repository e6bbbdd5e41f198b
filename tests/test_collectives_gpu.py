"""GPU parity of every catalogue algorithm against the CPU oracle, through the C ABI.

For each (op, alg, N) of the catalogue and each dtype, payloads P in {smallest legal, 4 KiB, 64 KiB,
192 KiB} (where legal and within shared memory), batches of 1 and of many cluster problems:
  * pattern A of the reference harness (main.cu:119): every result exact, compared bit for bit;
  * seeded U(-1,1) floats: |got - ref| <= rtol * (1 + |ref|) * ceil(log2 N) (main.cu:165) with
    rtol 1e-5 (f32) and 1e-2 (bf16); f32 also within the unscaled 1e-5 * (1 + |ref|); for bf16 the factor is
    the algorithm's chain of bf16 roundings where that is longer (rings: N - 1 hops; bf16_chain);
  * seeded U[-2^15, 2^15) int32: exact;
  * AllGather / AlltoAll (and the rooted Broadcast, Gather and Scatter): exact for every input.
Outputs are poisoned (all-ones bits) before each launch, so an element the kernel never wrote fails; for the
rooted Reduce and Gather, which write rank 0's out block only, the other ranks' blocks must still hold the poison.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402  (path set up by conftest)

CASES = [(op, alg, n) for (op, alg) in list(D.CATALOGUE) + list(D.EXTENSIONS) for n in D.CLUSTER_SIZES]
NAMES = {**D.CATALOGUE, **{k: v.split()[0] for k, v in D.EXTENSIONS.items()}}


def _np_to_torch(torch, host, dt):
    if dt == D.Dtype.BF16:
        return torch.from_numpy(host.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(host.copy())


def _torch_to_np(t, dt):
    import torch

    t = t.cpu()
    if dt == D.Dtype.BF16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


ORC_DT = {D.Dtype.F32: 0, D.Dtype.BF16: 1, D.Dtype.I32: 2}
EXACT_OPS = (D.Op.ALLGATHER, D.Op.ALLTOALL, D.Op.BROADCAST, D.Op.GATHER, D.Op.SCATTER)   # pure data movement
# the poison of run_case's outputs, as the bits _torch_to_np returns them
POISON = {D.Dtype.BF16: (np.uint16, 0xFFFF), D.Dtype.F32: (np.uint32, 0xFFFFFFFF), D.Dtype.I32: (np.int32, 2 ** 31 - 1)}
RTOL = {D.Dtype.F32: 1e-5, D.Dtype.BF16: 1e-2}


def bf16_chain(op, alg, n):
    """Roundings to bf16 along the algorithm's longest accumulation chain: every hop of a ring or shift schedule
    adds the received partial into a bf16 buffer (N - 1 hops), every round of a tree or halving schedule once
    (ceil(log2 N)); one-round algorithms accumulate in fp32 and round once. The bf16 bound is
    1e-2 * (1 + |ref|) per rounding of that chain, never below the reference's ceil(log2 N) factor (main.cu:165)."""
    chained = {(D.Op.ALLREDUCE, D.Alg.RING), (D.Op.ALLREDUCE, D.Alg.RING_CREDIT), (D.Op.REDUCESCATTER, D.Alg.RING),
               (D.Op.REDUCESCATTER, D.Alg.RING_CREDIT), (D.Op.ALLREDUCE, D.Alg.SHIFT_ACCUMULATE_BULK),
               (D.Op.ALLREDUCE, D.Alg.SHIFT_ACCUMULATE_BULK_CREDIT)}
    return max(n - 1 if (op, alg) in chained else 1, math.ceil(math.log2(n)))


def make_input(orc, dt, count, pattern, seed):
    odt = ORC_DT[dt]
    if pattern == "A":
        return orc.pattern_a(odt, count)
    if dt == D.Dtype.I32:
        return orc.uniform_int(count, seed, -32768, 32767)
    return orc.uniform_real(odt, count, seed, -1.0, 1.0)


def run_case(torch, orc, op, alg, n, dt, p, clusters, pattern, seed=0, max_resident_clusters=0):
    m = D.msg_elems(op, n, p, dt)
    nin = clusters * n * D.in_elems_per_rank(op, n, m)
    nout = clusters * n * D.out_elems_per_rank(op, n, m)
    host = make_input(orc, dt, nin, pattern, seed)
    tin = _np_to_torch(torch, host, dt).cuda()
    tdt = tin.dtype
    # poison: NaN bits for floats, INT32_MAX for int32 (no reachable sum in these tests)
    if dt == D.Dtype.BF16:
        tout = torch.full((nout,), -1, dtype=torch.int16, device="cuda").view(tdt)
    elif dt == D.Dtype.F32:
        tout = torch.full((nout,), -1, dtype=torch.int32, device="cuda").view(tdt)
    else:
        tout = torch.full((nout,), 2 ** 31 - 1, dtype=torch.int32, device="cuda")
    D.collective(op, alg, tin, tout, n, p, max_resident_clusters=max_resident_clusters)
    D.check()
    got = _torch_to_np(tout, dt)
    ref = orc.reference(int(op), ORC_DT[dt], n, m, clusters, host)
    if op in D.ROOT_OUT_ONLY:   # only rank 0's out blocks are written: the others keep the poison
        mask = orc.written(int(op), n, m, clusters)
        kind, bits = POISON[dt]
        untouched = got[~mask].view(kind)
        assert (untouched == bits).all(), f"{int((untouched != bits).sum())} elements of non-root out blocks written"
        got, ref = got[mask], ref[mask]
    exact = pattern == "A" or dt == D.Dtype.I32 or op in EXACT_OPS
    if exact:
        bad, ma, mr = orc.check(ORC_DT[dt], got, ref, 0)
        assert bad == 0, f"{bad} inexact elements (max abs {ma})"
    else:
        tol = RTOL[dt] * (bf16_chain(op, alg, n) if dt == D.Dtype.BF16 else math.ceil(math.log2(n)))
        bad, ma, mr = orc.check(ORC_DT[dt], got, ref, 1, tol)
        assert bad == 0, f"{bad} elements beyond {tol}*(1+|ref|) (max rel {mr})"
        if dt == D.Dtype.F32:
            bad2, _, mr2 = orc.check(ORC_DT[dt], got, ref, 1, 1e-5)
            assert bad2 == 0, f"f32 beyond 1e-5*(1+|ref|): max rel {mr2}"
    return mr


def payloads(op, alg, n, dt):
    out = []
    smallest = None
    for p in [16 * 2 ** k for k in range(0, 10)]:
        if D.query(op, alg, dt, n, p)[0] == D.Status.OK:
            smallest = p
            break
    for p in ([smallest] if smallest else []) + [4096, 65536, 196608]:
        if p not in out and D.query(op, alg, dt, n, p)[0] == D.Status.OK:
            out.append(p)
    return out


@pytest.mark.parametrize("op,alg,n", CASES, ids=[f"{NAMES[(o, a)]}-N{n}" for (o, a, n) in CASES])
def test_parity(cuda, orc, op, alg, n):
    torch = cuda
    ran, failures = 0, []
    for dt in D.Dtype:
        for p in payloads(op, alg, n, dt):
            batches = (1, 37) if p <= 16384 else (1, 3)
            for clusters in batches:
                for pattern in ("A", "R"):
                    try:
                        run_case(torch, orc, op, alg, n, dt, p, clusters, pattern, seed=p + clusters)
                    except (AssertionError, D.DsmemError) as e:
                        failures.append(f"{dt.name} P={p} clusters={clusters} pattern={pattern}: {e}")
                    ran += 1
    if ran == 0:
        pytest.skip("no legal configuration (reference static_assert)")
    assert not failures, "\n".join(failures)


@pytest.mark.parametrize("alg", (D.Alg.TWO_SHOT_PUSH, D.Alg.RS_PUSH_GLOBAL_AG), ids=("two_shot", "rs_push_global_ag"))
@pytest.mark.parametrize("n", D.CLUSTER_SIZES)
def test_pipelined_matches_plain(cuda, orc, n, alg):
    """The pipelined batch drivers (sub-vector units, bulk HBM copies, no per-problem cluster barrier)
    against the oracle, with the plain driver forced for comparison; many problems per resident cluster,
    every dtype, and payloads that split into several units."""
    failures = []
    try:
        for pipelined in (True, False):
            D.set_pipelined(pipelined)
            for dt in D.Dtype:
                for p in (256 * n // 8 if n >= 8 else 256, 4096, 16384, 65536, 196608):
                    if D.query(D.Op.ALLREDUCE, alg, dt, n, p)[0] != D.Status.OK:
                        continue
                    for clusters, pattern in ((2, "A"), (301, "R"), (1200, "A")):
                        if p * n * clusters > (256 << 20):
                            continue
                        try:
                            run_case(cuda, orc, D.Op.ALLREDUCE, alg, n, dt, p, clusters, pattern, seed=clusters)
                        except (AssertionError, D.DsmemError) as e:
                            failures.append(f"pipelined={pipelined} {dt.name} P={p} clusters={clusters}: {e}")
    finally:
        D.set_pipelined(True)
    assert not failures, "\n".join(failures)


def test_many_problems_per_cluster(cuda, orc):
    """Persistent clusters loop over many problems: 4000 AllReduce problems at N = 8, 16 KiB, f32."""
    for alg in (D.Alg.RING, D.Alg.RECURSIVE_DOUBLING, D.Alg.TWO_SHOT_PUSH, D.Alg.ONE_SHOT_PULL):
        run_case(cuda, orc, D.Op.ALLREDUCE, alg, 8, D.Dtype.F32, 16384, 4000, "R", seed=11)
        run_case(cuda, orc, D.Op.ALLREDUCE, alg, 8, D.Dtype.I32, 16384, 4000, "R", seed=12)


def test_resident_cap_and_repeat(cuda, orc):
    """Same result with one resident cluster (all problems serialised) and when relaunched."""
    torch = cuda
    op, alg, n, p, clusters = D.Op.REDUCESCATTER, D.Alg.RING, 4, 4096, 50
    m = D.msg_elems(op, n, p, D.Dtype.I32)
    host = make_input(orc, D.Dtype.I32, clusters * n * n * m, "R", 5)
    tin = torch.from_numpy(host).cuda()
    outs = []
    for cap in (0, 1, 3):
        for _ in range(2):
            tout = torch.empty(clusters * n * m, dtype=torch.int32, device="cuda")
            D.collective(op, alg, tin, tout, n, p, max_resident_clusters=cap)
            D.check()
            outs.append(tout.cpu().numpy())
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


ROOTED = [(o, a) for (o, a) in D.EXTENSIONS if o in (D.Op.BROADCAST, D.Op.REDUCE, D.Op.GATHER, D.Op.SCATTER)]


@pytest.mark.parametrize("op,alg", ROOTED, ids=[NAMES[k] for k in ROOTED])
def test_rooted_many_problems_per_cluster(cuda, orc, op, alg):
    """The rooted ops' persistent loop: 23 problems through 1 and 3 resident clusters (each cluster runs several
    problems in a row, so every mbarrier goes through several phases and every buffer is reused), against the
    oracle, f32 random and int32 exact, at N = 2, 8 and 16."""
    failures = []
    for n in (2, 8, 16):
        for dt, pattern in ((D.Dtype.F32, "R"), (D.Dtype.I32, "R"), (D.Dtype.BF16, "A")):
            p = 4096 if D.query(op, alg, dt, n, 4096)[0] == D.Status.OK else 256 * n
            if D.query(op, alg, dt, n, p)[0] != D.Status.OK:
                continue
            for cap in (1, 3):
                try:
                    run_case(cuda, orc, op, alg, n, dt, p, 23, pattern, seed=31 * n + cap, max_resident_clusters=cap)
                except (AssertionError, D.DsmemError) as e:
                    failures.append(f"N={n} {dt.name} P={p} resident={cap}: {e}")
    assert not failures, "\n".join(failures)


def test_stamps_and_smid(cuda):
    torch = cuda
    n, p, clusters = 8, 16384, 4
    m = D.msg_elems(D.Op.ALLREDUCE, n, p, D.Dtype.F32)
    tin = torch.randn(clusters * n * m, device="cuda")
    tout = torch.empty_like(tin)
    stamps = torch.zeros(clusters * n * 32, dtype=torch.int64, device="cuda")
    smid = torch.full((clusters * n,), -1, dtype=torch.int32, device="cuda")
    D.collective(D.Op.ALLREDUCE, D.Alg.RING, tin, tout, n, p, stamps=stamps, smid=smid)
    D.check()
    st = stamps.cpu().numpy().reshape(clusters, n, 32)
    sm = smid.cpu().numpy().reshape(clusters, n)
    rounds = 2 * (n - 1)
    for c in range(clusters):
        assert len(set(sm[c].tolist())) == n, "ranks of one cluster share an SM"
        for b in range(n):
            seq = [st[c, b, 0]] + [st[c, b, 2 + r] for r in range(rounds)] + [st[c, b, 1]]
            assert all(x > 0 for x in seq)
            assert all(seq[i] <= seq[i + 1] for i in range(len(seq) - 1)), "stamps not monotone"


def test_bounded_wait_reports_timeout(cuda, orc):
    """A wait that can never complete gives up after its limit; the kernel ends and TIMEOUT is reported."""
    D.check()   # clear
    D.selftest_timeout(2_000_000)   # 2 ms
    with pytest.raises(D.DsmemError) as e:
        D.check()
    assert e.value.status == D.Status.TIMEOUT
    D.check()   # the word was cleared; the context is still usable
    run_case(cuda, orc, D.Op.ALLREDUCE, D.Alg.RING, 4, D.Dtype.F32, 4096, 2, "A")


def test_illegal_config_rejected_before_launch(cuda):
    torch = cuda
    tin = torch.zeros(1024, device="cuda")
    tout = torch.zeros(1024, device="cuda")
    with pytest.raises(D.DsmemError) as e:
        D.collective(D.Op.ALLREDUCE, D.Alg.SHIFT_ACCUMULATE_BULK, tin, tout, 8, 512)
    assert e.value.status == D.Status.ILLEGAL_CONFIG
    with pytest.raises(D.DsmemError) as e:
        D.collective(D.Op.ALLREDUCE, D.Alg.ONE_SHOT_PULL, tin, tout, 8, 196608 * 2, num_clusters=0)
    assert e.value.status == D.Status.SMEM_LIMIT


# ---------------------------------------------------------------------------------------------------------
# BASELINE configs[0], exactly as specified: a cluster of 8 CTAs, each holding 4096 values (16 KiB per CTA);
# fp32 drawn U(-1,1) from mt19937_64 seeded 0, int32 drawn U[-1000,1000] from seed 0 (bit-exact), the ring
# and recursive-doubling AllReduce (and their mbarrier-credit forms), one cluster per launch and a grid-filling
# batch (whose first problem is the single-cluster input).
CONFIG0_ALGS = (D.Alg.RING, D.Alg.RECURSIVE_DOUBLING, D.Alg.RING_CREDIT, D.Alg.RECURSIVE_DOUBLING_CREDIT)


@pytest.mark.parametrize("clusters", (1, 296), ids=("single_cluster", "batch296"))
@pytest.mark.parametrize("alg", CONFIG0_ALGS, ids=[a.name.lower() for a in CONFIG0_ALGS])
def test_config0_exact_inputs(cuda, orc, alg, clusters):
    torch = cuda
    n, m = 8, 4096
    p = m * 4
    count = clusters * n * m
    for dt, host in ((D.Dtype.F32, orc.uniform_real(0, count, 0, -1.0, 1.0)),
                     (D.Dtype.I32, orc.uniform_int(count, 0, -1000, 1000))):
        tin = torch.from_numpy(host.copy()).cuda()
        tout = torch.full_like(tin, -1) if dt == D.Dtype.I32 else torch.full_like(tin, float("nan"))
        D.collective(D.Op.ALLREDUCE, alg, tin, tout, n, p)
        D.check()
        got = tout.cpu().numpy()
        ref = orc.reference(int(D.Op.ALLREDUCE), ORC_DT[dt], n, m, clusters, host)
        if dt == D.Dtype.I32:
            bad, ma, _ = orc.check(ORC_DT[dt], got, ref, 0)
            assert bad == 0, f"int32: {bad} elements differ (max abs {ma})"
        else:
            bad, _, mr = orc.check(ORC_DT[dt], got, ref, 1, 1e-5)
            assert bad == 0, f"fp32: {bad} elements beyond 1e-5*(1+|ref|) (max rel {mr})"


# ---------------------------------------------------------------------------------------------------------
# BASELINE configs[1]'s payload grid, swept: every power-of-two payload from the smallest legal one to
# 128 KiB, plus 192 KiB, for every (op, alg, N, dtype): one cluster per launch and, below 64 KiB, a batch of
# two (test_parity already runs 64 and 192 KiB at 1 and 3 clusters). Payloads above the one-piece
# shared-memory limit run where a pipelined driver takes them (batch regime).
GRID = [16 * 2 ** k for k in range(0, 14)] + [196608]   # 16 B ... 128 KiB, 192 KiB
PIPELINED_ALGS = {(D.Op.ALLREDUCE, D.Alg.TWO_SHOT_PUSH), (D.Op.ALLREDUCE, D.Alg.RS_PUSH_GLOBAL_AG),
                  (D.Op.REDUCESCATTER, D.Alg.DIRECT_PUSH), (D.Op.ALLTOALL, D.Alg.DIRECT_PUSH),
                  (D.Op.ALLGATHER, D.Alg.DIRECT_REPLICATED_PUSH)}


def grid_points(op, alg, n, dt):
    """(P, cluster counts) of the configs[1] grid that this (op, alg, N, dtype) can launch."""
    pts = []
    for p in GRID:
        st = D.query(op, alg, dt, n, p)[0]
        if st == D.Status.OK:
            if p in (65536, 196608):
                continue   # test_parity runs these at 1 and 3 clusters
            pts.append((p, (1, 2) if p < 65536 else (1,)))
        elif st == D.Status.SMEM_LIMIT and (op, alg) in PIPELINED_ALGS:
            pts.append((p, (2,)))
    return pts


@pytest.mark.parametrize("op,alg,n", CASES, ids=[f"{NAMES[(o, a)]}-N{n}" for (o, a, n) in CASES])
def test_payload_grid(cuda, orc, op, alg, n):
    ran, failures = 0, []
    for dt in D.Dtype:
        for p, batches in grid_points(op, alg, n, dt):
            for clusters in batches:
                try:
                    run_case(cuda, orc, op, alg, n, dt, p, clusters, "R", seed=7 * p + clusters)
                except (AssertionError, D.DsmemError) as e:
                    failures.append(f"{dt.name} P={p} clusters={clusters}: {e}")
                ran += 1
    if ran == 0:
        pytest.skip("no legal configuration (reference static_assert)")
    assert not failures, "\n".join(failures)


# (0, 0, 0): the measured defaults, which take 32 KiB units for launches of at most one wave (the 2-problem
# batches below) and 16 KiB units otherwise
STREAM_SETTINGS = ((0, 0, 0), (16384, 0, 1), (4096, 5, 3), (2048, 2, 1), (65536, 3, 2), (1024, 8, 1))
STREAMED = ((D.Op.ALLREDUCE, D.Alg.RS_PUSH_GLOBAL_AG), (D.Op.REDUCESCATTER, D.Alg.DIRECT_PUSH),
            (D.Op.ALLTOALL, D.Alg.DIRECT_PUSH), (D.Op.ALLGATHER, D.Alg.DIRECT_REPLICATED_PUSH))


@pytest.mark.parametrize("op,alg", STREAMED, ids=[f"{o.name.lower()}-{a.name.lower()}" for o, a in STREAMED])
@pytest.mark.parametrize("n", D.CLUSTER_SIZES)
def test_streamed_matches_plain(cuda, orc, op, alg, n):
    """The streamed batch drivers (warp-specialised, an input ring and a slot ring, no cluster barrier per unit)
    at several (unit, input stages, slot stages) settings -- units per problem from 1 to many, fewer units than
    stages, several problems per resident cluster -- are bit-equal to the plain driver of the same algorithm
    (AllReduce and ReduceScatter sum the N parts in the same rank order; AlltoAll and AllGather move bytes), and the
    plain result (or, above the one-piece shared-memory limit, the streamed one) is checked against the oracle."""
    torch = cuda
    failures = []
    try:
        for dt in D.Dtype:
            for p in (256 * n // 8 if n >= 8 else 256, 4096, 65536, 196608):
                if op != D.Op.ALLREDUCE and p < 16 * n:
                    continue
                if D.query(op, alg, dt, n, p)[0] not in (D.Status.OK, D.Status.SMEM_LIMIT):
                    continue
                m = D.msg_elems(op, n, p, dt)
                nin, nout = n * D.in_elems_per_rank(op, n, m), n * D.out_elems_per_rank(op, n, m)
                for clusters in (2, 301, 1200):
                    if max(nin, nout) * clusters * D.ELEM_BYTES[dt] > (256 << 20):
                        continue
                    host = make_input(orc, dt, clusters * nin, "R", clusters + p)
                    tin = _np_to_torch(torch, host, dt).cuda()
                    ref = orc.reference(int(op), ORC_DT[dt], n, m, clusters, host)
                    exact = dt == D.Dtype.I32 or op in (D.Op.ALLGATHER, D.Op.ALLTOALL)
                    tol = 0 if exact else RTOL[dt] * math.ceil(math.log2(n))

                    def empty():
                        z = torch.full((clusters * nout,), -1, dtype=torch.int32 if dt != D.Dtype.BF16 else torch.int16,
                                       device="cuda")
                        return z.view(tin.dtype)

                    plain = None
                    if D.query(op, alg, dt, n, p)[0] == D.Status.OK:
                        plain = empty()
                        D.set_pipelined(False)
                        D.collective(op, alg, tin, plain, n, p)
                        D.check()
                        D.set_pipelined(True)
                    outs = []
                    for unit, depth, lag in STREAM_SETTINGS:
                        D.set_stream_pipeline(unit, depth, lag)
                        out = empty()
                        D.collective(op, alg, tin, out, n, p)
                        D.check()
                        outs.append(out)
                    first = plain if plain is not None else outs[0]
                    bad, _, mr = orc.check(ORC_DT[dt], _torch_to_np(first, dt), ref, 0 if exact else 1, tol)
                    if bad:
                        failures.append(f"{dt.name} P={p} clusters={clusters}: {bad} off the oracle (max rel {mr})")
                    iv = torch.int16 if dt == D.Dtype.BF16 else torch.int32
                    for (unit, depth, lag), out in zip(STREAM_SETTINGS, outs):
                        if not torch.equal(out.view(iv), first.view(iv)):
                            failures.append(f"{dt.name} P={p} clusters={clusters} unit={unit} depth={depth} "
                                            f"lag={lag}: differs from the {'plain driver' if plain is not None else 'defaults'}")
    finally:
        D.set_pipelined(True)
        D.set_stream_pipeline()
    assert not failures, "\n".join(failures[:20])


# mbarrier-credit forms against their barrier-per-round originals: same rounds, partners and operand order, so
# the same bits for every dtype (random inputs, one and 37 clusters)
CREDIT_PAIRS = (
    (D.Op.ALLREDUCE, D.Alg.RING_CREDIT, D.Alg.RING),
    (D.Op.ALLREDUCE, D.Alg.RECURSIVE_DOUBLING_CREDIT, D.Alg.RECURSIVE_DOUBLING),
    (D.Op.ALLREDUCE, D.Alg.RABENSEIFNER_CREDIT, D.Alg.RABENSEIFNER),
    (D.Op.ALLREDUCE, D.Alg.BINOMIAL_CREDIT, D.Alg.REDUCE_BCAST_BINOMIAL),
    (D.Op.ALLREDUCE, D.Alg.SHIFT_ACCUMULATE_BULK_CREDIT, D.Alg.SHIFT_ACCUMULATE_BULK),
    (D.Op.ALLGATHER, D.Alg.RING_CREDIT, D.Alg.RING),
    (D.Op.ALLGATHER, D.Alg.RECURSIVE_DOUBLING_CREDIT, D.Alg.RECURSIVE_DOUBLING),
    (D.Op.ALLGATHER, D.Alg.BRUCK_CREDIT, D.Alg.BRUCK),
    (D.Op.ALLGATHER, D.Alg.BINOMIAL_CREDIT, D.Alg.GATHER_BCAST_BINOMIAL),
    (D.Op.REDUCESCATTER, D.Alg.RING_CREDIT, D.Alg.RING),
    (D.Op.REDUCESCATTER, D.Alg.RECURSIVE_HALVING_CREDIT, D.Alg.RECURSIVE_HALVING),
    (D.Op.ALLTOALL, D.Alg.PAIRWISE_XOR_CREDIT, D.Alg.PAIRWISE_XOR),
    (D.Op.ALLTOALL, D.Alg.BRUCK_CREDIT, D.Alg.BRUCK),
)


@pytest.mark.parametrize("op,credit,orig", CREDIT_PAIRS, ids=[f"{NAMES[(o, c)]}" for (o, c, _) in CREDIT_PAIRS])
def test_credit_matches_original(cuda, orc, op, credit, orig):
    torch = cuda
    ran, failures = 0, []
    for n in D.CLUSTER_SIZES:
        for dt in D.Dtype:
            for p in (256, 4096, 16384):
                if any(D.query(op, a, dt, n, p)[0] != D.Status.OK for a in (credit, orig)):
                    continue
                m = D.msg_elems(op, n, p, dt)
                for clusters in (1, 37):
                    nin = clusters * n * D.in_elems_per_rank(op, n, m)
                    nout = clusters * n * D.out_elems_per_rank(op, n, m)
                    host = make_input(orc, dt, nin, "R", seed=11 * p + n + clusters)
                    tin = _np_to_torch(torch, host, dt).cuda()
                    outs = []
                    for a in (credit, orig):
                        t = torch.full((nout,), -1, dtype=torch.int16 if dt == D.Dtype.BF16 else torch.int32,
                                       device="cuda").view(tin.dtype)
                        D.collective(op, a, tin, t, n, p)
                        D.check()
                        outs.append(_torch_to_np(t, dt).view(np.uint8))
                    if not np.array_equal(outs[0], outs[1]):
                        failures.append(f"N={n} {dt.name} P={p} clusters={clusters}: differs from {orig.name}")
                    ran += 1
    if ran == 0:
        pytest.skip("no configuration legal for both forms")
    assert not failures, "\n".join(failures)
