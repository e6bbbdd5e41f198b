"""The 29 reference-harness plugin files (collectives/<op>__<alg>__<src>.cu), built and launched the way the
reference harness builds and launches them (collectives/harness/driver.py:233-239, main.cu:63-66, 207-214,
273): one build per (file, cluster size N, element type) with compile-time CLUSTER_N / MSG_ELEMS / ELEM_T,
one cluster of N CTAs per launch, 256 threads, dynamic shared memory sizeof(CollectiveSmem).

    python -m dsmem_b200.shims          build lib/libdsmem_shims.so and lib/shims_manifest.json

Every (file, N in {2,4,8,16}, float / int) is compiled from csrc/shim_launcher.cu. A build that fails on a
static_assert is recorded as the reference's skip (SKIP:static_assert, or SKIP:smem for the CollectiveSmem
limit, driver.py:210-230); any other compiler error fails the build. The message size per build is the
configs[0] point of the sweep, 16 KiB per CTA: M = 4096 elements for AllReduce and 4096 / N for the other
ops (whose payload is N * M elements).
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes
import json
import os
import pathlib
import subprocess

PKG_DIR = pathlib.Path(__file__).resolve().parent.parent
COLLECTIVES_DIR = PKG_DIR / "collectives"
LAUNCHER = PKG_DIR / "csrc" / "shim_launcher.cu"
INCLUDE_DIR = PKG_DIR.parent / "include"
BUILD_DIR = PKG_DIR / "_build" / "shims"
LIB_PATH = PKG_DIR / "lib" / "libdsmem_shims.so"
MANIFEST_PATH = PKG_DIR / "lib" / "shims_manifest.json"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", f"-I{INCLUDE_DIR}", f"-I{COLLECTIVES_DIR}"]
CLUSTER_SIZES = (2, 4, 8, 16)
ELEM_TYPES = ("float", "int")
PAYLOAD = 16384   # bytes per CTA of every build


def files():
    """Stems of the plugin files, in name order."""
    return sorted(p.stem for p in COLLECTIVES_DIR.glob("*__*__*.cu"))


def op_of(stem):
    return stem.split("__")[0]


def msg_elems(stem, n):
    """MSG_ELEMS of the build: P = 16 KiB per CTA (AllReduce M * 4 B, the others N * M * 4 B)."""
    return PAYLOAD // 4 if op_of(stem) == "allreduce" else PAYLOAD // (4 * n)


def tag(stem, n, elem):
    return f"shim_{stem}__N{n}_{elem}"


def _deps():
    return [LAUNCHER, COLLECTIVES_DIR / "dsmem_b200_algos.cuh", COLLECTIVES_DIR / "dsmem_primitives.cuh",
            INCLUDE_DIR / "dsmem_b200.h"]


def _compile(stem, n, elem):
    """Compile one build; returns (tag, "ok" | "static_assert" | "smem", message)."""
    t = tag(stem, n, elem)
    obj, skip = BUILD_DIR / f"{t}.o", BUILD_DIR / f"{t}.skip"
    src = COLLECTIVES_DIR / f"{stem}.cu"
    newest = max(p.stat().st_mtime for p in _deps() + [src])
    for f in (obj, skip):
        if f.exists() and f.stat().st_mtime >= newest:
            return (t, "ok", "") if f is obj else (t, *skip.read_text().split("\n", 1))
    for f in (obj, skip):
        f.unlink(missing_ok=True)
    cmd = [NVCC, *FLAGS, f'-DCOLLECTIVE_FILE="{src}"', f"-DCLUSTER_N={n}", f"-DMSG_ELEMS={msg_elems(stem, n)}",
           f"-DELEM_T={elem}", f"-DSHIM_TAG={t}", "-c", str(LAUNCHER), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0:
        return t, "ok", ""
    err = r.stderr
    if "static assertion failed" in err:
        kind = "smem" if "SMEM_LIMIT" in err else "static_assert"
        line = next((x for x in err.splitlines() if "static assertion failed" in x), "").strip()
        line = line.replace(f"{PKG_DIR}/", "")
        skip.write_text(f"{kind}\n{line}")
        return t, kind, line
    raise RuntimeError(f"shim build {t} failed:\n{err}")


def build(jobs=None):
    """Compile every (file, N, element type), link lib/libdsmem_shims.so, write the manifest; returns it."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
    todo = [(s, n, e) for s in files() for n in CLUSTER_SIZES for e in ELEM_TYPES]
    with cf.ThreadPoolExecutor(max_workers=jobs or min(16, os.cpu_count() or 8)) as ex:
        results = list(ex.map(lambda a: _compile(*a), todo))
    builds, skipped = [], []
    for (stem, n, elem), (t, kind, msg) in zip(todo, results):
        rec = {"stem": stem, "op": op_of(stem), "n": n, "elem": elem, "msg_elems": msg_elems(stem, n), "tag": t}
        if kind == "ok":
            builds.append(rec)
        else:
            skipped.append({**rec, "skip": kind, "message": msg})
    objs = [str(BUILD_DIR / f"{b['tag']}.o") for b in builds]
    newest = max(pathlib.Path(o).stat().st_mtime for o in objs)
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest or not MANIFEST_PATH.exists():
        subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB_PATH), *objs,
                        "-lcudart"], check=True)
    man = {"payload_bytes_per_cta": PAYLOAD, "threads": 256, "builds": builds, "skipped": skipped}
    text = json.dumps(man, indent=1)
    if not MANIFEST_PATH.exists() or MANIFEST_PATH.read_text() != text:
        MANIFEST_PATH.write_text(text)
    return man


def manifest():
    if not MANIFEST_PATH.exists():
        raise RuntimeError(f"{MANIFEST_PATH} is missing: run `python -m dsmem_b200.shims` (there is no fallback)")
    return json.loads(MANIFEST_PATH.read_text())


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m dsmem_b200.shims` (there is no fallback)")
        _lib = ctypes.CDLL(str(LIB_PATH))
    return _lib


def launch(t, in_ptr, out_ptr, ts_ptr=0, smid_ptr=0, stream=0):
    """Launch build `t` (a manifest tag) on raw device pointers; raises on a CUDA error."""
    fn = getattr(lib(), f"{t}_launch")
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5
    r = fn(in_ptr, out_ptr, ts_ptr or None, smid_ptr or None, stream or None)
    if r != 0:
        raise RuntimeError(f"{t}: cudaError {r}")


def smem_bytes(t):
    fn = getattr(lib(), f"{t}_smem")
    fn.restype = ctypes.c_size_t
    return fn()


def take_error(t):
    """Synchronise and read-and-clear build `t`'s device error word (DSMEM_ERRBIT_*; 0 = none)."""
    fn = getattr(lib(), f"{t}_take_error")
    fn.restype = ctypes.c_uint
    return fn()


if __name__ == "__main__":
    m = build()
    print(f"{len(m['builds'])} builds, {len(m['skipped'])} skipped -> {LIB_PATH}")
