"""Generate tests/golden/reference_golden.npz from the reference's OWN host code.

Runs the binaries built by `make -C oracle ref` (oracle/ref_golden.cu: the reference harness
collectives/harness/main.cu compiled with its main() renamed) for every op x N in {2,4,8,16} x
{float, int} at M = 64, patterns A (float, int) and B (float only, as main.cu:189 allows), and stores
for each record the SHA-256 of the input the reference's fill_input() produced (main.cu:118-126) and the
reference() output (main.cu:129-149) in float64.

Run here, where the reference is mounted:  make -C oracle ref -j8 && python tests/golden/make_golden.py
The fixture is committed; tests never need the reference at run time.
"""
import hashlib
import pathlib
import struct
import subprocess
import sys
import tempfile

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
REF_BIN = ROOT / "oracle" / "_ref"
OUT = pathlib.Path(__file__).resolve().parent / "reference_golden.npz"


def read_record(path):
    raw = pathlib.Path(path).read_bytes()
    op, n, m, is_int, n_in, n_out = struct.unpack_from("<6q", raw, 0)
    off = 48
    dt = np.int32 if is_int else np.float32
    inp = np.frombuffer(raw, dtype=dt, count=n_in, offset=off)
    off += inp.nbytes
    ref = np.frombuffer(raw, dtype=np.float64, count=n_out, offset=off)
    return op, n, m, bool(is_int), inp, ref


def main():
    arrays = {}
    with tempfile.TemporaryDirectory() as tmp:
        for op in range(4):
            for n in (2, 4, 8, 16):
                for t in ("float", "int"):
                    exe = REF_BIN / f"ref_op{op}_N{n}_M64_{t}"
                    if not exe.exists():
                        sys.exit(f"missing {exe}: run `make -C oracle ref -j8` first")
                    for pattern in ("A", "B") if t == "float" else ("A",):
                        rec = pathlib.Path(tmp) / "rec.bin"
                        subprocess.run([str(exe), "golden", pattern, str(rec)], check=True)
                        op_, n_, m_, is_int, inp, ref = read_record(rec)
                        assert (op_, n_, m_, is_int) == (op, n, 64, t == "int")
                        key = f"op{op}_N{n}_M64_{t}_{pattern}"
                        arrays[key + "_in_sha256"] = np.frombuffer(hashlib.sha256(inp.tobytes()).digest(), np.uint8)
                        arrays[key + "_ref"] = ref.copy()
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays) // 2} records)")


if __name__ == "__main__":
    main()
