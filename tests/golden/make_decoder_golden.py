"""Generate tests/golden/decoder_golden.npz from the reference's OWN fp32 decoder-layer reference.

roofline/harness/workloads/clusterfusion_llama2_7b_decoder.py:160-180 (`reference_fp32`) is plain torch: RMSNorm of
inp + res, QKV projection, NEOX RoPE, attention over the cache plus the new token, O projection, and with the layer
scope the tail h = x + o, RMSNorm, SwiGLU FFN. This script imports that module where the reference is mounted and
runs the function on the CPU at a small shape (2 heads x 16, hidden 32, FFN 48, 7 cached tokens). Every input is
exactly representable in fp16 (the reference's dtype) and in bf16 (the oracle's), so both compute from identical
values.

    python tests/golden/make_decoder_golden.py      # needs the reference checkout ($REF, else BASELINE.json's
                                                    # reference_path)

The fixture is committed; tests never need the reference at run time.
"""
import os
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "decoder_golden.npz"

def _reference_root():
    import json

    ref = os.environ.get("REF") or json.loads((HERE.parents[1] / "BASELINE.json").read_text()).get("reference_path")
    if not ref or not pathlib.Path(ref).is_dir():
        raise SystemExit("set REF to the reference checkout")
    return pathlib.Path(ref)


REF = _reference_root()


def main():
    import torch

    sys.path.insert(0, str(REF / "roofline" / "harness" / "workloads"))
    sys.path.insert(0, str(REF / "roofline" / "harness"))
    argv, sys.argv = sys.argv, [sys.argv[0]]
    try:
        import clusterfusion_llama2_7b_decoder as ref
    finally:
        sys.argv = argv
    H, D, S, ffn = 2, 16, 7, 48
    hid = H * D
    g = np.random.default_rng(7)

    def grid(shape, lo, hi, step):
        """Values k * step with |k| <= 128: exact in bf16 (8 significant bits) and in fp16."""
        return (g.integers(lo, hi + 1, shape) * step).astype(np.float32)

    a = {
        "inp": grid((1, hid), -128, 128, 2.0 ** -7),
        "res": grid((1, hid), -128, 128, 2.0 ** -7),
        "w_rms": (1.0 + grid((hid,), -16, 16, 2.0 ** -7)).astype(np.float32),
        "wqkv": grid((3 * hid, hid), -64, 64, 2.0 ** -8),
        "wo": grid((hid, hid), -64, 64, 2.0 ** -8),
        "w_post": (1.0 + grid((hid,), -16, 16, 2.0 ** -7)).astype(np.float32),
        "wgu": grid((2 * ffn, hid), -64, 64, 2.0 ** -8),
        "wd": grid((hid, ffn), -64, 64, 2.0 ** -8),
        "kc": grid((S, H, D), -128, 128, 2.0 ** -7),
        "vc": grid((S, H, D), -128, 128, 2.0 ** -7),
    }
    ang = (S + 1) * 10000.0 ** (-np.arange(D // 2) / (D // 2))
    a["cos"] = np.concatenate([np.cos(ang), np.cos(ang)]).astype(np.float32)
    a["sin"] = np.concatenate([np.sin(ang), np.sin(ang)]).astype(np.float32)
    h16 = {k: torch.from_numpy(v).to(torch.float16) for k, v in a.items() if k not in ("cos", "sin")}
    for k, v in h16.items():
        assert np.array_equal(v.float().numpy(), a[k]), f"{k} not exact in fp16"
        assert not (a[k].view(np.uint32) & 0xFFFF).any(), f"{k} not exact in bf16"
    st = types.SimpleNamespace(H=H, D=D, S=S, hid=hid, ffn=ffn, layer=True, w_rms=h16["w_rms"], wqkv=h16["wqkv"],
                               wo=h16["wo"], w_post=h16["w_post"], wgu=h16["wgu"], wd=h16["wd"], kc=h16["kc"],
                               vc=h16["vc"], cos3=torch.from_numpy(a["cos"]).view(1, 1, D),
                               sin3=torch.from_numpy(a["sin"]).view(1, 1, D))
    o, k, v, out = ref.reference_fp32(st, h16["inp"], h16["res"])
    np.savez_compressed(OUT, **a, eps=np.float64(ref.EPS), shape=np.array([H, D, S, ffn]),
                        o=o.numpy().reshape(-1), k_new=k.numpy().reshape(-1), v_new=v.numpy().reshape(-1),
                        out=out.numpy().reshape(-1))
    print("wrote", OUT)


if __name__ == "__main__":
    main()
