"""Host-side tests of the C ABI (no GPU): exported symbols, names, file stems, legality and shared-memory
classification against the reference build matrix, AUTO tables.

Legality restates the reference files' static_asserts (collectives/<file>.cu) and the per-file shared
memory of collectives/docs/TESTING.md:28-39 (in elements of T); the B200 build adds a 128-byte mbarrier
area and, uniformly, 16-byte whole messages (every M of the reference matrix satisfies it).
"""
import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "dsmem_b200.h"


def declared_functions(path):
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dsmem_[a-z0-9_]+)\s*\(", text)))


def test_header_compiles_as_c_and_cxx_and_links(dsmem, tmp_path):
    """A C caller and a C++ caller that take the address of every declared entry point compile against
    include/dsmem_b200.h (C99 and C++11, warnings as errors), link against lib/libdsmem_b200.so with unmangled
    names, and load and run (no GPU call is made)."""
    import os
    import shutil
    import subprocess

    names = declared_functions(HEADER)
    body = ",\n".join(f"        (fn)&{n}" for n in names)
    src = ('#include "dsmem_b200.h"\n#include <stdio.h>\ntypedef void (*fn)(void);\nint main(void) {\n'
           f"    fn table[] = {{\n{body}\n    }};\n"
           '    printf("%d\\n", (int)(sizeof table / sizeof table[0]));\n    return 0;\n}\n')
    libdir = str(dsmem.LIB_PATH.parent)
    cuda_lib = "/usr/local/cuda/lib64"
    for compiler, std, ext in (("gcc", "-std=c99", "c"), ("g++", "-std=c++11", "cpp")):
        if shutil.which(compiler) is None:
            pytest.skip(f"{compiler} not found")
        path = tmp_path / f"abi.{ext}"
        path.write_text(src)
        exe = tmp_path / f"abi_{ext}"
        subprocess.run([compiler, std, "-Wall", "-Wextra", "-Werror", f"-I{HEADER.parent}", str(path), "-o", str(exe),
                        f"-L{libdir}", "-ldsmem_b200", f"-Wl,-rpath-link,{cuda_lib}"], check=True)
        env = dict(os.environ, LD_LIBRARY_PATH=":".join([libdir, cuda_lib, os.environ.get("LD_LIBRARY_PATH", "")]))
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, env=env).stdout
        assert int(out) == len(names)


def test_library_exports_every_declared_symbol(dsmem):
    names = declared_functions(HEADER)
    assert len(names) >= 15
    lib = ctypes.CDLL(str(dsmem.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_names_and_stems(dsmem):
    L = dsmem.lib()
    assert L.dsmem_op_name(0) == b"allreduce"
    assert L.dsmem_alg_name(int(dsmem.Alg.TWO_SHOT_PUSH)) == b"two_shot_push"
    assert L.dsmem_dtype_name(1) == b"bf16"
    assert dsmem.version().startswith("dsmem_b200")
    for (op, alg), stem in dsmem.CATALOGUE.items():
        assert dsmem.file_stem(op, alg) == stem
        assert dsmem.lookup(stem) == (op, alg)
        assert dsmem.lookup(stem + ".cu") == (op, alg)
        assert (dsmem.COLLECTIVES_DIR / f"{stem}.cu").exists(), f"missing harness-compatible file {stem}.cu"
    assert len(dsmem.CATALOGUE) == 29
    assert dsmem.file_stem(dsmem.Op.ALLTOALL, dsmem.Alg.RING) is None
    with pytest.raises(dsmem.DsmemError):
        dsmem.lookup("allreduce__nope__x")


def pow2(n):
    return n & (n - 1) == 0


def grid2d(n):
    r = 4 if n >= 16 else (2 if n >= 4 else 1)
    return r, n // r


# (op, alg) -> (constraint(N, M, B), smem elements(N, M)) restated from the reference files
def rules(dsmem):
    A, O = dsmem.Alg, dsmem.Op
    m16 = lambda n, m, b: (m * b) % 16 == 0
    return {
        (O.ALLREDUCE, A.RECURSIVE_DOUBLING): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: 3 * m),
        (O.ALLREDUCE, A.SHIFT_ACCUMULATE_BULK): (lambda n, m, b: n == 4 and m16(n, m, b), lambda n, m: 3 * m),
        (O.ALLREDUCE, A.SHIFT_ACCUMULATE_ATOMIC): (lambda n, m, b: n in (2, 4) and m16(n, m, b), lambda n, m: 2 * m),
        (O.ALLREDUCE, A.DIRECT_REPLICATED_PUSH): (m16, lambda n, m: (n + 2) * m),
        (O.ALLREDUCE, A.PULL_REDUCE_SCATTER_PUSH_ALLGATHER): (lambda n, m, b: 32 % n == 0 and m % n == 0 and m16(n, m, b),
                                                              lambda n, m: m),
        (O.ALLREDUCE, A.RING): (lambda n, m, b: m % n == 0 and ((m // n) * b) % 16 == 0, lambda n, m: m + m // n),
        (O.ALLREDUCE, A.RABENSEIFNER): (lambda n, m, b: pow2(n) and m % n == 0 and ((m // n) * b) % 16 == 0,
                                        lambda n, m: m + m // 2),
        (O.ALLREDUCE, A.ONE_SHOT_PULL): (m16, lambda n, m: 2 * m),
        (O.ALLREDUCE, A.TWO_SHOT_PUSH): (lambda n, m, b: m % n == 0 and ((m // n) * b) % 16 == 0, lambda n, m: 2 * m),
        (O.ALLREDUCE, A.REDUCE_BCAST_BINOMIAL): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: 2 * m),
        (O.ALLREDUCE, A.ATOMIC_ALL_PUSH): (m16, lambda n, m: 2 * m),
        (O.ALLREDUCE, A.MESH_2D): (lambda n, m, b: m % grid2d(n)[1] == 0 and ((m // grid2d(n)[1]) * b) % 16 == 0,
                                   lambda n, m: m + (sum(grid2d(n)) + 1) * (m // grid2d(n)[1])),
        (O.ALLGATHER, A.RECURSIVE_DOUBLING): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: n * m),
        (O.ALLGATHER, A.DIRECT_SHIFT): (m16, lambda n, m: n * m),
        (O.ALLGATHER, A.DIRECT_REPLICATED_PUSH): (m16, lambda n, m: (n + 1) * m),
        (O.ALLGATHER, A.RING): (m16, lambda n, m: n * m),
        (O.ALLGATHER, A.BRUCK): (m16, lambda n, m: n * m),
        (O.ALLGATHER, A.DIRECT_PULL): (m16, lambda n, m: (n + 1) * m),
        (O.ALLGATHER, A.GATHER_BCAST_BINOMIAL): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: n * m),
        (O.REDUCESCATTER, A.RING): (m16, lambda n, m: n * m + m),
        (O.REDUCESCATTER, A.RECURSIVE_HALVING): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: n * m + n * m // 2),
        (O.REDUCESCATTER, A.DIRECT_PUSH): (m16, lambda n, m: 2 * n * m + m),
        (O.REDUCESCATTER, A.DIRECT_PULL): (m16, lambda n, m: n * m + m),
        (O.ALLTOALL, A.PAIRWISE_EXCHANGE): (lambda n, m, b: n == 2 and m16(n, m, b), lambda n, m: n * m + m),
        (O.ALLTOALL, A.DIRECT_PUSH): (m16, lambda n, m: 2 * n * m),
        (O.ALLTOALL, A.PAIRWISE_XOR): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: 2 * n * m),
        (O.ALLTOALL, A.SHIFT): (m16, lambda n, m: 2 * n * m),
        (O.ALLTOALL, A.BRUCK): (lambda n, m, b: pow2(n) and m16(n, m, b), lambda n, m: n * m + n * m // 2),
        (O.ALLTOALL, A.DIRECT_PULL): (m16, lambda n, m: 2 * n * m),
    }


SMEM_LIMIT = 232448
PAYLOADS = [2 ** k for k in range(4, 18)] + [192 * 1024, 48, 96, 200, 1000]


def test_legality_and_smem_match_reference_matrix(dsmem):
    R = rules(dsmem)
    FP32_ACCUMULATORS = (dsmem.Alg.SHIFT_ACCUMULATE_ATOMIC, dsmem.Alg.ATOMIC_ALL_PUSH)
    assert set(R) == set(dsmem.CATALOGUE)
    checked = 0
    for (op, alg), (legal_fn, smem_fn) in R.items():
        for dt in dsmem.Dtype:
            b = dsmem.ELEM_BYTES[dt]
            for n in dsmem.CLUSTER_SIZES:
                for p in PAYLOADS:
                    unit = b * (1 if op == dsmem.Op.ALLREDUCE else n)
                    status, smem, legal = dsmem.query(op, alg, dt, n, p)
                    if p % unit:
                        assert status == dsmem.Status.ILLEGAL_CONFIG and not legal
                        continue
                    m = p // unit
                    if not legal_fn(n, m, b):
                        assert status == dsmem.Status.ILLEGAL_CONFIG, (op, alg, dt, n, p)
                        continue
                    want = 128 + smem_fn(n, m) * b
                    if alg in FP32_ACCUMULATORS and dt == dsmem.Dtype.BF16:
                        want = 128 + smem_fn(n, m) * 4   # bf16 remote-atomic sums accumulate in fp32
                    assert smem == want, (op.name, alg.name, dt.name, n, p, smem, want)
                    if want > SMEM_LIMIT:
                        assert status == dsmem.Status.SMEM_LIMIT
                    else:
                        assert status == dsmem.Status.OK and legal
                    checked += 1
    assert checked > 2000


def test_rooted_ops_legality_smem_and_names(dsmem):
    """The rooted extensions (no reference file): names, payload convention (Reduce P = M B, Gather and Scatter
    P = N M B), legality (16-byte rank blocks) and the window each algorithm declares, sized for rank 0's
    buffers; AUTO's built-in order prefers the direct push where it fits."""
    L, O, A = dsmem.lib(), dsmem.Op, dsmem.Alg
    assert [L.dsmem_op_name(int(o)) for o in (O.REDUCE, O.GATHER, O.SCATTER)] == [b"reduce", b"gather", b"scatter"]
    lg = {2: 1, 4: 2, 8: 3, 16: 4}
    window = {  # elements of the window, from N and M
        (O.REDUCE, A.DIRECT_PUSH): lambda n, m: n * m, (O.REDUCE, A.DIRECT_PULL): lambda n, m: m,
        (O.REDUCE, A.BINOMIAL): lambda n, m: (1 + lg[n]) * m,
        **{(o, a): (lambda n, m: n * m) for o in (O.GATHER, O.SCATTER) for a in (A.DIRECT_PUSH, A.DIRECT_PULL, A.BINOMIAL)},
    }
    for (op, alg), win in window.items():
        assert (op, alg) in dsmem.EXTENSIONS
        for dt in dsmem.Dtype:
            b = dsmem.ELEM_BYTES[dt]
            for n in dsmem.CLUSTER_SIZES:
                for p in PAYLOADS:
                    unit = b * (1 if op == O.REDUCE else n)
                    status, smem, legal = dsmem.query(op, alg, dt, n, p)
                    m = p // unit
                    if p % unit or (m * b) % 16:
                        assert status == dsmem.Status.ILLEGAL_CONFIG and not legal, (op, alg, dt, n, p)
                        continue
                    assert smem == 128 + win(n, m) * b, (op.name, alg.name, dt.name, n, p, smem)
                    assert status == (dsmem.Status.OK if smem <= SMEM_LIMIT else dsmem.Status.SMEM_LIMIT)
    empty_pick = dsmem.autotune_pick(O.GATHER, dsmem.Dtype.F32, 8, 16384)
    assert empty_pick in (A.DIRECT_PUSH, A.DIRECT_PULL, A.BINOMIAL)


def test_auto_defaults_and_table(dsmem, tmp_path):
    Op, Alg, Dt = dsmem.Op, dsmem.Alg, dsmem.Dtype
    empty = tmp_path / "empty.txt"
    empty.write_text("")
    dsmem.autotune_load(empty)   # the built-in order alone (no measured table)
    assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 16384) == Alg.TWO_SHOT_PUSH
    # two-shot needs N | M with 16-B chunks; 64 B at N = 8 is not legal for it
    pick = dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 64)
    assert pick != Alg.TWO_SHOT_PUSH and dsmem.query(Op.ALLREDUCE, pick, Dt.F32, 8, 64)[2]
    table = tmp_path / "tune.txt"
    table.write_text("# op N bytes dtype alg\nallreduce 8 256 f32 ring\nallreduce 8 65536 f32 one_shot_pull\n")
    dsmem.autotune_load(table)
    try:
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 4096) == Alg.RING
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 65536) == Alg.ONE_SHOT_PULL
        # 128 KiB: one-shot pull would need 256 KiB of shared memory, so AUTO falls back to a fitting one
        big = dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 131072)
        assert big != Alg.ONE_SHOT_PULL and dsmem.query(Op.ALLREDUCE, big, Dt.F32, 8, 131072)[0] == dsmem.Status.OK
        # below the smallest entry: built-in default order
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 128) != Alg.AUTO
        # an entry whose algorithm is illegal at that size falls back to the defaults
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.BF16, 8, 4096) == Alg.TWO_SHOT_PUSH
        # regimes: a `batch` line serves batches; one cluster per launch keeps the `single` line
        table.write_text("allreduce 8 256 f32 ring single\nallreduce 8 256 f32 rabenseifner batch\n")
        dsmem.autotune_load(table)
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 4096, num_clusters=1) == Alg.RING
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 4096, num_clusters=64) == Alg.RABENSEIFNER
        table.write_text("allreduce 8 256 f32 ring batch\n")   # no `single` line: the batch one serves
        dsmem.autotune_load(table)
        assert dsmem.autotune_pick(Op.ALLREDUCE, Dt.F32, 8, 4096, num_clusters=1) == Alg.RING
        bad = tmp_path / "bad_regime.txt"
        bad.write_text("allreduce 8 256 f32 ring sometimes\n")
        with pytest.raises(dsmem.DsmemError):
            dsmem.autotune_load(bad)
    finally:
        dsmem.autotune_load(empty)
    bad = tmp_path / "bad.txt"
    bad.write_text("allreduce 8 256 f32 no_such_alg\n")
    with pytest.raises(dsmem.DsmemError):
        dsmem.autotune_load(bad)
    bad.write_text("alltoall 8 256 f32 ring\n")   # ring does not exist for alltoall
    with pytest.raises(dsmem.DsmemError):
        dsmem.autotune_load(bad)


def test_invalid_arguments(dsmem):
    st, _, legal = dsmem.query(dsmem.Op.ALLREDUCE, dsmem.Alg.RING, dsmem.Dtype.F32, 3, 4096)
    assert st == dsmem.Status.INVALID_ARGUMENT and not legal
    st, _, _ = dsmem.query(dsmem.Op.ALLTOALL, dsmem.Alg.RING, dsmem.Dtype.F32, 4, 4096)
    assert st == dsmem.Status.ILLEGAL_CONFIG
    with pytest.raises(dsmem.DsmemError) as e:
        dsmem.launch(dsmem.Op.ALLREDUCE, dsmem.Alg.RING, dsmem.Dtype.F32, 8, 4096, 16, 32, 1)
    assert e.value.status == dsmem.Status.INVALID_ARGUMENT or e.value.status == dsmem.Status.CUDA


def test_shipped_autotune_table_parses(dsmem, tmp_path):
    """The table measured on B200 and shipped next to lib/ loads, and every entry names a legal algorithm."""
    path = dsmem.PKG_DIR / "autotune_b200.tsv"
    if not path.exists():
        pytest.skip("no measured table shipped")
    dsmem.autotune_load(path)
    try:
        lines = [ln.split() for ln in path.read_text().splitlines() if ln.strip() and not ln.startswith("#")]
        assert lines
        ops = {"allreduce": dsmem.Op.ALLREDUCE, "allgather": dsmem.Op.ALLGATHER,
               "reducescatter": dsmem.Op.REDUCESCATTER, "alltoall": dsmem.Op.ALLTOALL,
               "broadcast": dsmem.Op.BROADCAST, "reduce": dsmem.Op.REDUCE, "gather": dsmem.Op.GATHER,
               "scatter": dsmem.Op.SCATTER}
        dts = {"f32": dsmem.Dtype.F32, "bf16": dsmem.Dtype.BF16, "i32": dsmem.Dtype.I32}
        pipelined = {(dsmem.Op.ALLREDUCE, dsmem.Alg.TWO_SHOT_PUSH), (dsmem.Op.ALLREDUCE, dsmem.Alg.RS_PUSH_GLOBAL_AG),
                     (dsmem.Op.REDUCESCATTER, dsmem.Alg.DIRECT_PUSH), (dsmem.Op.ALLTOALL, dsmem.Alg.DIRECT_PUSH),
                     (dsmem.Op.ALLGATHER, dsmem.Alg.DIRECT_REPLICATED_PUSH)}
        by_name = {dsmem.lib().dsmem_alg_name(int(x)).decode(): x for x in dsmem.Alg}
        for op, n, p, dt, alg, regime in lines:
            a = by_name[alg]
            st = dsmem.query(ops[op], a, dts[dt], int(n), int(p))[0]
            # payloads above the one-piece limit run on the pipelined / streamed driver (one problem or many)
            assert st == dsmem.Status.OK or (st == dsmem.Status.SMEM_LIMIT and (ops[op], a) in pipelined)
            got = dsmem.autotune_pick(ops[op], dts[dt], int(n), int(p), num_clusters=64 if regime == "batch" else 1)
            assert got == a
    finally:
        empty = tmp_path / "empty.txt"
        empty.write_text("")
        dsmem.autotune_load(empty)


def test_capi_host_collective_argument_checks(dsmem):
    """Host-side checks of dsmem_collective_host, which return before any device call."""
    lib = dsmem.lib()
    fake = ctypes.c_void_p(0x10000)
    null = ctypes.c_void_p(None)
    s, op, alg, dt = dsmem.Status, dsmem.Op, dsmem.Alg, dsmem.Dtype
    assert lib.dsmem_collective_host(op.ALLREDUCE, alg.AUTO, dt.F32, 8, 65536, null, fake, 4, 0) == s.INVALID_ARGUMENT
    assert lib.dsmem_collective_host(op.ALLREDUCE, alg.AUTO, dt.F32, 3, 65536, fake, fake, 4, 0) == s.INVALID_ARGUMENT
    assert lib.dsmem_collective_host(op.ALLGATHER, alg.AUTO, dt.F32, 8, 100, fake, fake, 4, 0) == s.ILLEGAL_CONFIG
    assert lib.dsmem_collective_host(op.ALLREDUCE, alg.AUTO, dt.F32, 8, 65536, fake, fake, -1, 0) == s.INVALID_ARGUMENT
    assert lib.dsmem_collective_host(op.ALLREDUCE, alg.AUTO, dt.F32, 8, 65536, fake, fake, 0, 0) == s.OK


def test_rowwise_and_topk_plans_fit(dsmem):
    """The row-wise and top-k launch planners (host logic, no device call): every planned launch fits the 227 KiB
    of dynamic shared memory per CTA, has at least one ring stage and one look-ahead group at most, and returns
    SMEM_LIMIT exactly where one row slice of every input (top-k: one segment) cannot fit."""
    lib = dsmem.lib()
    s = dsmem.Status
    smem, rpg, stages, ahead = ctypes.c_size_t(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    # row slices resident per CTA: staged inputs (+ LayerNorm's gamma slice) for quant, LARS, LN, Pearson,
    # softmax, weighted variance
    n_inputs = [1, 3, 3, 2, 2, 3]
    for wl in range(6):
        for n in (1, 2, 4, 8, 16):
            for cols in (1, 3, 5, 100, 1003, 4096, 16384, 40000, 65536, 131072):
                st = lib.dsmem_rowwise_query(wl, cols, n, ctypes.byref(smem), ctypes.byref(rpg), ctypes.byref(stages),
                                             ctypes.byref(ahead))
                slice_bytes = (((cols + n - 1) // n + 3) // 4 * 4) * 4
                if n_inputs[wl] * slice_bytes > 227 * 1024 - 1024:
                    assert st == s.SMEM_LIMIT, (wl, n, cols, st)
                    continue
                assert st == s.OK, (wl, n, cols, st)
                assert 0 < smem.value <= 232448
                assert rpg.value in (1, 2, 4, 8) and 1 <= stages.value <= 8
                assert ahead.value == min(1, stages.value - 1)
    assert lib.dsmem_rowwise_query(6, 100, 8, None, None, None, None) == s.INVALID_ARGUMENT
    assert lib.dsmem_rowwise_query(0, 100, 3, None, None, None, None) == s.INVALID_ARGUMENT
    for n in (2, 4, 8, 16):
        for length in (1, 7, 32768, 65536, 244650, 400000):
            st = lib.dsmem_topk_query(length, n, ctypes.byref(smem))
            if st == s.OK:
                assert smem.value <= 232448
            else:
                assert st == s.SMEM_LIMIT and ((length + n - 1) // n) * 4 > 150 * 1024, (n, length)
    assert lib.dsmem_topk_query(244650, 8, ctypes.byref(smem)) == s.OK            # the reference's m8_n240k
    assert lib.dsmem_topk_query(244650, 4, ctypes.byref(smem)) == s.SMEM_LIMIT
    assert lib.dsmem_topk_query(100, 3, ctypes.byref(smem)) == s.INVALID_ARGUMENT
