"""Known-answer tests of the oracle's input generators.

* mt19937_64: the C++ standard's known answer ([rand.predef]: the 10000th output of a
  default-constructed std::mt19937_64, seed 5489, is 9981545732273789042).
* The benchmark draws (U(-1,1) floats and U[-1000,1000] ints from seed 0) use
  std::uniform_real_distribution / std::uniform_int_distribution on mt19937_64; the oracle's C
  restatement is compared with the standard library compiled here.
"""
import shutil
import subprocess

import numpy as np
import pytest


def test_mt19937_64_known_answer(orc):
    g = orc.mt64(5489)
    v = 0
    for _ in range(10000):
        v = orc.mt64_next(g)
    assert v == 9981545732273789042


CPP = r"""
#include <cstdio>
#include <random>
int main() {
    std::mt19937_64 g(0);
    std::uniform_real_distribution<double> u(-1.0, 1.0);
    for (int i = 0; i < 2000; ++i) std::printf("%.17g\n", u(g));
    std::mt19937_64 h(0);
    std::uniform_int_distribution<int> d(-1000, 1000);
    for (int i = 0; i < 2000; ++i) std::printf("%d\n", d(h));
    std::mt19937_64 k(7);
    std::uniform_int_distribution<int> e(-32768, 32767);
    for (int i = 0; i < 2000; ++i) std::printf("%d\n", e(k));
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_draws_match_standard_library(orc, tmp_path):
    src = tmp_path / "draws.cpp"
    src.write_text(CPP)
    exe = tmp_path / "draws"
    subprocess.run(["g++", "-O1", "-std=c++17", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    reals = np.array([float(x) for x in out[:2000]])
    ints = np.array([int(x) for x in out[2000:4000]])
    ints2 = np.array([int(x) for x in out[4000:]])
    # float32 draws of the oracle are the double draws rounded to float
    got = orc.uniform_real(orc.F32, 2000, 0, -1.0, 1.0)
    assert np.array_equal(got, reals.astype(np.float32))
    assert np.array_equal(orc.uniform_int(2000, 0, -1000, 1000), ints)
    assert np.array_equal(orc.uniform_int(2000, 7, -32768, 32767), ints2)


def test_bf16_rounding_is_nearest_even(orc):
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40], np.float32)
    bits = orc.f32_to_bf16(x)
    for v, b in zip(x, bits):
        assert orc.lib().orc_f32_to_bf16(float(v)) == int(b)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: rounds to the even mantissa (1.0)
    assert orc.bf16_to_f32(bits[1]) == 1.0


def test_broadcast_reference_is_rank0_vector(orc):
    """The broadcast restatement (B200 extension op 4): every rank's output is rank 0's input, per cluster."""
    n, m, clusters = 4, 8, 3
    inp = np.arange(clusters * n * m, dtype=np.int32)
    ref = orc.reference(4, 2, n, m, clusters, inp)
    for c in range(clusters):
        for b in range(n):
            got = ref[(c * n + b) * m:(c * n + b + 1) * m]
            assert (got == inp[c * n * m:c * n * m + m]).all()


def test_rooted_references(orc):
    """The rooted restatements (B200 extension ops 5-7): REDUCE gives rank 0 the sum of the ranks' vectors,
    GATHER gives rank 0 the vectors in rank order, and neither writes the other ranks' out blocks (written()
    marks them); SCATTER gives rank b block b of rank 0's input. Per cluster, int32 exact and f32."""
    n, m, clusters = 4, 8, 3
    for dt in (0, 2):
        for op in (orc.REDUCE, orc.GATHER, orc.SCATTER):
            ie, oe = orc.in_elems(op, n, m), orc.out_elems(op, n, m)
            count = clusters * n * ie
            inp = (orc.uniform_int(count, 5, -1000, 1000) if dt == 2 else orc.uniform_real(0, count, 5, -1.0, 1.0))
            ref = orc.reference(op, dt, n, m, clusters, inp).reshape(clusters, n, oe)
            x = inp.astype(np.float64).reshape(clusters, n, ie)
            mask = orc.written(op, n, m, clusters).reshape(clusters, n, oe)
            if op == orc.REDUCE:
                assert np.allclose(ref[:, 0], x.sum(axis=1), rtol=0, atol=1e-12)
            elif op == orc.GATHER:
                assert np.array_equal(ref[:, 0], x.reshape(clusters, n * m))
            else:
                assert np.array_equal(ref, x[:, 0].reshape(clusters, n, m))
            if op == orc.SCATTER:
                assert mask.all()
            else:
                assert mask[:, 0].all() and not mask[:, 1:].any()
