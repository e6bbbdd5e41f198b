"""Decoder layer against the CPU oracle, through the C ABI.

Oracle: oracle.decoder_layer, the double-precision restatement of reference_fp32 with the FFN tail
(roofline/harness/workloads/clusterfusion_llama2_7b_decoder.py:160-180). Tolerances of that file (:78-79):
the attention-block output o within max abs 2e-2, MAE 1e-3 and relative L2 1e-2; the new k, v (after
RoPE) and the layer output within relative L2 1e-2 and max abs 2e-2 * max|ref|. The kernel rounds the
stage boundaries (x, xn, the attention output, h, hn, SiLU(gate)*up) to bf16; the oracle does not.
Shapes: reduced (hidden 1024, 8 heads, ffn 2816, 300 cached tokens) at batch 1, 3, 16 and cluster 4 / 8,
and the full Llama-2-7B layer (hidden 4096, 32 heads, ffn 11008, 4096 cached tokens) at batch 1, 4 and 16.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402

TOL_O = {"max_abs": 2e-2, "mae": 1e-3, "rel_l2": 1e-2}
TOL_REL = {"rel_l2": 1e-2, "rel_max": 2e-2}


def errs(got, ref):
    d = got.astype(np.float64) - ref
    rm = float(np.abs(ref).max())
    return {"max_abs": float(np.abs(d).max()), "mae": float(np.abs(d).mean()),
            "rel_l2": float(np.linalg.norm(d) / max(np.linalg.norm(ref), 1e-30)), "rel_max": float(np.abs(d).max()) / max(rm, 1e-30)}


def make_layer(orc, B, hidden, heads, ffn, S, cap, seed):
    r = lambda n, s, std: orc.normal(1, n, seed * 100 + s, 0.0, std)   # noqa: E731
    L = {
        "inp": r(B * hidden, 1, 1.0).reshape(B, hidden), "res": r(B * hidden, 2, 1.0).reshape(B, hidden),
        "w_rms": orc.normal(1, hidden, seed * 100 + 3, 1.0, 0.02), "w_post": orc.normal(1, hidden, seed * 100 + 4, 1.0, 0.02),
        "wqkv": r(3 * hidden * hidden, 5, 0.02).reshape(3 * hidden, hidden),
        "wo": r(hidden * hidden, 6, 0.02).reshape(hidden, hidden),
        "wgu": r(2 * ffn * hidden, 7, 0.02).reshape(2 * ffn, hidden),
        "wd": r(hidden * ffn, 8, 0.02).reshape(hidden, ffn),
        "kc": r(B * cap * heads * 128, 9, 1.0).reshape(B, cap, heads, 128),
        "vc": r(B * cap * heads * 128, 10, 1.0).reshape(B, cap, heads, 128),
    }
    # RoPE at position S, theta 10000 (NEOX halves)
    inv = 10000.0 ** (-np.arange(0, 128, 2, dtype=np.float64) / 128)
    ang = S * inv
    L["cos"] = np.concatenate([np.cos(ang), np.cos(ang)]).astype(np.float32)
    L["sin"] = np.concatenate([np.sin(ang), np.sin(ang)]).astype(np.float32)
    return L


def run_layer(torch, orc, B, hidden, heads, ffn, S, cap, n, seed=0):
    L = make_layer(orc, B, hidden, heads, ffn, S, cap, seed)
    bf = lambda a: torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()   # noqa: E731
    t = {k: (bf(v) if v.dtype == np.uint16 else torch.from_numpy(v).cuda()) for k, v in L.items()}
    o = torch.empty(B, hidden, dtype=torch.bfloat16, device="cuda")
    kn, vn = torch.empty_like(o), torch.empty_like(o)
    out, h = D.decoder_layer(t["inp"], t["res"], t["w_rms"], t["wqkv"], t["wo"], t["w_post"], t["wgu"], t["wd"],
                             t["kc"], t["vc"], t["cos"], t["sin"], S, eps=1e-5, cluster_size=n, o_out=o, k_new=kn,
                             v_new=vn)
    torch.cuda.synchronize()
    D.decoder_check()
    D.rmsnorm_check()
    ref = orc.decoder_layer(L["inp"], L["res"], L["w_rms"], L["wqkv"], L["wo"], L["w_post"], L["wgu"], L["wd"],
                            L["kc"], L["vc"], L["cos"], L["sin"], S, 1e-5, heads)
    f = lambda x: x.float().cpu().numpy()   # noqa: E731
    got = {"out": f(out), "h": f(h), "o": f(o), "k_new": f(kn), "v_new": f(vn)}
    # the cache row S now holds the step's k and v
    kc_row = t["kc"][:, S].reshape(B, hidden)
    assert torch.equal(kc_row, kn), "cache row S differs from k_new"
    return {k: errs(got[k], ref[k]) for k in got}


def check(e):
    fails = []
    eo = e["o"]
    if not (eo["max_abs"] <= TOL_O["max_abs"] and eo["mae"] <= TOL_O["mae"] and eo["rel_l2"] <= TOL_O["rel_l2"]):
        fails.append(f"o {eo}")
    for k in ("k_new", "v_new", "out", "h"):
        if not (e[k]["rel_l2"] <= TOL_REL["rel_l2"] and e[k]["rel_max"] <= TOL_REL["rel_max"]):
            fails.append(f"{k} {e[k]}")
    return fails


@pytest.mark.parametrize("B,n", [(1, 8), (3, 4), (16, 8), (9, 4)])
def test_decoder_reduced_shape(cuda, orc, B, n):
    fails = check(run_layer(cuda, orc, B, 1024, 8, 2816, 300, 320, n, seed=B))
    assert not fails, "\n".join(fails)


@pytest.mark.parametrize("B,n", [(1, 8), (4, 8), (16, 8), (16, 4)])
def test_decoder_llama2_7b(cuda, orc, B, n):
    """The full Llama-2-7B layer at configs[3]'s batches 1, 4 and 16 (batch 16's attention runs at cluster 2,
    its (sequence, head) count being above 96), plus batch 16 with cluster-4 projections."""
    fails = check(run_layer(cuda, orc, B, 4096, 32, 11008, 4096, 4097, n, seed=7 + B))
    assert not fails, "\n".join(fails)


def test_decoder_rejects_bad_shapes(cuda):
    torch = cuda
    z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16, device="cuda")   # noqa: E731
    c = torch.zeros(128, device="cuda")
    with pytest.raises(D.DsmemError) as e:   # ffn not a multiple of 64
        D.decoder_layer(z(1, 1024), z(1, 1024), z(1024), z(3072, 1024), z(1024, 1024), z(1024), z(2 * 100, 1024),
                        z(1024, 100), z(1, 8, 8, 128), z(1, 8, 8, 128), c, c, 3)
    assert e.value.status == D.Status.ILLEGAL_CONFIG
    with pytest.raises(D.DsmemError) as e:   # no room for the new token
        D.decoder_layer(z(1, 1024), z(1, 1024), z(1024), z(3072, 1024), z(1024, 1024), z(1024), z(2 * 256, 1024),
                        z(1024, 256), z(1, 8, 8, 128), z(1, 8, 8, 128), c, c, 8)
    assert e.value.status == D.Status.INVALID_ARGUMENT
