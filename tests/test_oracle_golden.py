"""The C oracle against golden vectors produced by the reference's own host code.

tests/golden/reference_golden.npz was written by tests/golden/make_golden.py from binaries that compile
collectives/harness/main.cu (fill_input :118-126, reference :129-149) straight from the reference
sources. Each record pins (1) the oracle's input generator (SHA-256 of the input array) and (2) the
oracle's reference reduction (bit-identical float64 output: same double summation order).
"""
import hashlib
import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "reference_golden.npz"
OPS = (0, 1, 2, 3)
NS = (2, 4, 8, 16)
M = 64


def records():
    for op in OPS:
        for n in NS:
            for t in ("float", "int"):
                for pattern in ("A", "B") if t == "float" else ("A",):
                    yield op, n, t, pattern


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("op,n,t,pattern", list(records()))
def test_oracle_matches_reference_golden(orc, golden, op, n, t, pattern):
    dtype = orc.F32 if t == "float" else orc.I32
    count = n * orc.in_elems(op, n, M)
    inp = orc.pattern_a(dtype, count) if pattern == "A" else orc.pattern_b(dtype, count)
    key = f"op{op}_N{n}_M{M}_{t}_{pattern}"
    assert hashlib.sha256(inp.tobytes()).digest() == golden[key + "_in_sha256"].tobytes(), "fill_input differs"
    ref = orc.reference(op, dtype, n, M, 1, inp)
    want = golden[key + "_ref"]
    assert ref.shape == want.shape
    assert np.array_equal(ref.view(np.uint64), want.view(np.uint64)), "reference() output differs"


def test_golden_covers_every_record(golden):
    assert len(golden.files) == 2 * len(list(records()))


def test_batched_reference_is_per_cluster(orc):
    """Batches are independent problems: cluster c of a batch equals a single-problem run."""
    for op in OPS:
        n, m, clusters = 4, 32, 5
        per = n * orc.in_elems(op, n, m)
        inp = orc.pattern_b(orc.F32, clusters * per)
        ref = orc.reference(op, orc.F32, n, m, clusters, inp)
        per_out = n * orc.out_elems(op, n, m)
        for c in range(clusters):
            one = orc.reference(op, orc.F32, n, m, 1, inp[c * per:(c + 1) * per])
            assert np.array_equal(one, ref[c * per_out:(c + 1) * per_out])


def test_check_modes(orc):
    ref = np.array([1.0, 2.5, -3.0, 1e-3], np.float64)
    out = ref.astype(np.float32)
    assert orc.check(orc.F32, out, ref, 0)[0] == 0
    out2 = out.copy()
    out2[1] += 1e-3
    assert orc.check(orc.F32, out2, ref, 0)[0] == 1
    assert orc.check(orc.F32, out2, ref, 1, 1e-3)[0] == 0
    assert orc.check(orc.F32, out2, ref, 1, 1e-4)[0] == 1
    nan = out.copy()
    nan[0] = np.nan
    assert orc.check(orc.F32, nan, ref, 1, 1.0)[0] == 1   # NaN never passes
