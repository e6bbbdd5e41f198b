"""The 29 reference-harness plugin files (h100-dsmem-collectives_b200/collectives/<op>__<alg>__<src>.cu) as
builds, checked on the CPU.

* Every (file, N in {2,4,8,16}, float / int) is either built into lib/libdsmem_shims.so or recorded as the
  reference's skip, and the skips are exactly the configurations the C ABI classifies as illegal
  (ILLEGAL_CONFIG -> SKIP:static_assert) or too large (SMEM_LIMIT -> SKIP:smem) at the same payload.
* The library exports the launcher of every build, and its CollectiveSmem size equals dsmem_query's.
* Where the reference checkout is mounted: each file compiles inside the reference's own harness
  (collectives/harness/main.cu with the flags of collectives/harness/driver.py:233-239, for sm_100a) exactly
  when our build of it compiles, and fails on the same kind of static_assert otherwise.
"""
import concurrent.futures as cf
import ctypes
import subprocess

import pytest

import dsmem_b200 as D
from dsmem_b200 import shims
from conftest import reference_root

OPS = {"allreduce": D.Op.ALLREDUCE, "allgather": D.Op.ALLGATHER, "reducescatter": D.Op.REDUCESCATTER,
       "alltoall": D.Op.ALLTOALL}
ELEM = {"float": D.Dtype.F32, "int": D.Dtype.I32}


@pytest.fixture(scope="module")
def manifest():
    return shims.build()


def test_every_file_is_built_or_skipped_as_the_abi_classifies(manifest):
    stems = shims.files()
    assert len(stems) == 29
    seen = {}
    for rec in manifest["builds"]:
        seen[(rec["stem"], rec["n"], rec["elem"])] = "ok"
    for rec in manifest["skipped"]:
        seen[(rec["stem"], rec["n"], rec["elem"])] = rec["skip"]
    assert len(seen) == 29 * 4 * 2
    want_kind = {D.Status.OK: "ok", D.Status.ILLEGAL_CONFIG: "static_assert", D.Status.SMEM_LIMIT: "smem"}
    for (stem, n, elem), kind in seen.items():
        op, alg = D.lookup(stem)
        st = D.query(op, alg, ELEM[elem], n, shims.PAYLOAD)[0]
        assert want_kind[st] == kind, f"{stem} N={n} {elem}: build says {kind}, dsmem_query says {st.name}"


def test_library_exports_every_build(manifest):
    lib = ctypes.CDLL(str(shims.LIB_PATH))
    for rec in manifest["builds"]:
        for suffix in ("_launch", "_smem", "_take_error"):
            assert hasattr(lib, rec["tag"] + suffix), rec["tag"] + suffix
        op, alg = D.lookup(rec["stem"])
        want = D.query(op, alg, ELEM[rec["elem"]], rec["n"], shims.PAYLOAD)[1]
        assert shims.smem_bytes(rec["tag"]) >= want, rec["tag"]


def _compile_in_reference_harness(ref, stem, n, elem, tmp):
    op = shims.op_of(stem)
    cmd = [shims.NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O0", f"-I{ref}/common/h100mb",
           f'-DCOLLECTIVE_FILE="{shims.COLLECTIVES_DIR / (stem + ".cu")}"', f'-DCOLL_NAME="{stem}"',
           f"-DCOLL_OP={int(OPS[op])}", f"-DCLUSTER_N={n}", f"-DMSG_ELEMS={shims.msg_elems(stem, n)}",
           f"-DELEM_T={elem}", "-c", str(ref / "collectives" / "harness" / "main.cu"),
           "-o", str(tmp / f"{stem}_{n}_{elem}.o")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0:
        return "ok", ""
    if "static assertion failed" in r.stderr:
        return ("smem" if "SMEM_LIMIT" in r.stderr else "static_assert"), ""
    return "error", r.stderr[-2000:]


def test_files_compile_inside_the_reference_harness(manifest, tmp_path):
    ref = reference_root()
    if ref is None or not (ref / "collectives" / "harness" / "main.cu").exists():
        pytest.skip("reference checkout not mounted")
    ours = {(r["stem"], r["n"], r["elem"]): "ok" for r in manifest["builds"]}
    ours.update({(r["stem"], r["n"], r["elem"]): r["skip"] for r in manifest["skipped"]})
    todo = [(s, 8, "float") for s in shims.files()] + [(s, 16, "int") for s in shims.files()]
    with cf.ThreadPoolExecutor(max_workers=8) as ex:
        got = list(ex.map(lambda a: _compile_in_reference_harness(ref, *a, tmp_path), todo))
    bad = [f"{a}: harness {k} ({msg}), ours {ours[a]}" for a, (k, msg) in zip(todo, got) if k != ours[a]]
    assert not bad, "\n".join(bad)
