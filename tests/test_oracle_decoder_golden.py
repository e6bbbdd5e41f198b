"""The decoder-layer oracle (orc_decoder_layer) against the reference's own fp32 reference.

tests/golden/decoder_golden.npz was written by tests/golden/make_decoder_golden.py, which imports
roofline/harness/workloads/clusterfusion_llama2_7b_decoder.py and runs its `reference_fp32` (:160-180, with the
layer-scope FFN tail) on the CPU at a small shape, from inputs exact in both fp16 and bf16. The oracle accumulates
in double, the reference in fp32: outputs agree to 1e-4 of their largest magnitude.
"""
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "decoder_golden.npz"


def test_decoder_oracle_matches_reference_fp32(orc):
    g = np.load(GOLDEN)
    H, D, S, ffn = (int(v) for v in g["shape"])
    bf = lambda k: orc.f32_to_bf16(g[k])  # noqa: E731 -- exact: the fixture's inputs are bf16 values
    kc = bf("kc").reshape(1, S, H, D)
    vc = bf("vc").reshape(1, S, H, D)
    got = orc.decoder_layer(bf("inp"), bf("res"), bf("w_rms"), bf("wqkv"), bf("wo"), bf("w_post"), bf("wgu"), bf("wd"),
                            kc, vc, g["cos"], g["sin"], S, float(g["eps"]), H, head_dim=D)
    assert got["out"].shape == (1, H * D) and g["wd"].shape == (H * D, ffn)
    for name, ref in (("o", g["o"]), ("k_new", g["k_new"]), ("v_new", g["v_new"]), ("out", g["out"])):
        r = np.asarray(ref, np.float64)
        err = np.max(np.abs(got[name].ravel() - r))
        assert err <= 1e-4 * np.max(np.abs(r)), f"{name}: max err {err:.3e} vs scale {np.max(np.abs(r)):.3e}"
