"""CPU model of the top-k kernel's selection (ext_topk.cu), checked against the oracle on adversarial rows.

The model restates the kernel's steps with numpy:
- the 11-bit coarse key of the fp16-rounded value, with NaN pinned to the top (+NaN) or bottom (-NaN) bin;
- the cut bin of the cluster-wide histogram;
- fine rounds. When both neighbouring fp16 values of the bin are finite and the key span fits 21 bits, the
  rounds run on the key relative to the bin's exact range (two digits); otherwise they run on three absolute
  digits of the fp32 key (bits 21..31, 10..20, 0..9);
- exact ties shared among the cluster's segments in rank order.
It runs the same arithmetic on the same keys as the kernel, so a flaw in the method (a wrong range bound, a
digit schedule that loses bits, a tie share that does not add up to k) shows here without a GPU.
"""
import numpy as np
import pytest


def key32(v):
    v = np.asarray(v, np.float32)
    b = v.view(np.uint32).astype(np.uint64)
    k = np.where(b & 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000)
    nan = np.isnan(v)
    return np.where(nan, np.where(b >> 31, 0, 0xFFFFFFFF), k).astype(np.uint64)


def coarse(v):
    v = np.asarray(v, np.float32)
    with np.errstate(over="ignore"):
        h = v.astype(np.float16).view(np.uint16).astype(np.uint32)
    k16 = np.where(h & 0x8000, (~h) & 0xFFFF, h | 0x8000)
    ck = (k16 >> 5).astype(np.uint64)
    nan = np.isnan(v)
    return np.where(nan, np.where(v.view(np.uint32) >> 31, 0, 0x7FF), ck).astype(np.uint64)


def half16_value(k16):
    h = (k16 & 0x7FFF) if (k16 & 0x8000) else ((~k16) & 0xFFFF)
    return np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]


def find_cut(hist, r):
    acc = 0
    for d in range(len(hist) - 1, -1, -1):
        if acc + hist[d] >= r:
            return d, acc, r - acc, int(hist[d])
        acc += int(hist[d])
    raise AssertionError("histogram holds fewer than r elements")


def model_topk(x, k, n_cta):
    """Indices the kernel selects for one row (the order within the row is not modelled)."""
    n = x.size
    seg = ((n + n_cta - 1) // n_cta + 3) // 4 * 4
    ck, kk = coarse(x), key32(x)
    tau, _, r, in_bin = find_cut(np.bincount(ck.astype(np.int64), minlength=2048), k)
    full = r == in_bin
    base, shifts, masks, nfine = 0, [21, 10, 0], [0x7FF, 0x7FF, 0x3FF], 3
    kb = tau << 5
    ok = kb > 0 and kb + 32 <= 0xFFFF
    if ok:
        lo, hi = half16_value(kb - 1), half16_value(kb + 32)
        ok = not (np.isnan(lo) or np.isnan(hi))
    if ok:
        klo = int(key32(lo)[()]) + 1
        span = int(key32(hi)[()]) - klo
        bits = 1 if span <= 1 else int(span - 1).bit_length()
        if bits <= 21:
            base = klo
            s1 = bits - 11 if bits > 11 else 0
            shifts, masks, nfine = [s1, 0], [0x7FF, (1 << s1) - 1], (2 if s1 > 0 else 1)
    cand = ck == tau
    u = (kk.astype(np.int64) - base) & 0xFFFFFFFF
    if cand.any():   # the kernel's relative keys stay below 2^21 inside the cut bin
        assert base == 0 or u[cand].max() < (1 << 21)
    shift, prefix = 32, 0
    for fr in range(nfine):
        if full:
            break
        sh = shifts[fr]
        m = cand.copy()
        if shift < 32:
            m &= (u >> shift) == prefix
        d, _, r, in_bin = find_cut(np.bincount(((u[m] >> sh) & masks[fr]).astype(np.int64), minlength=2048), r)
        prefix = (0 if shift == 32 else (prefix << (shift - sh)) & 0xFFFFFFFF) | d
        shift, full = sh, r == in_bin
    sel = ck > tau
    tie = np.zeros(n, bool)
    if shift == 32:
        sel |= cand
    else:
        p = u >> shift
        sel |= cand & (p > prefix)
        eq = cand & (p == prefix)
        if full:
            sel |= eq
        else:
            tie = eq
    out = list(np.nonzero(sel)[0])
    taken = 0
    for b in range(n_cta):   # exact ties in rank order, then index order within a segment
        if taken >= r or full or shift == 32:
            break
        idx = np.nonzero(tie[b * seg:(b + 1) * seg])[0] + b * seg
        take = idx[: r - taken]
        out += list(take)
        taken += take.size
    return np.array(out, np.int64)


def rows():
    g = np.random.default_rng(21)
    yield "randn", g.standard_normal(20000).astype(np.float32)
    yield "fp16 grid", g.standard_normal(20000).astype(np.float16).astype(np.float32)
    yield "ten values", g.integers(0, 10, 20000).astype(np.float32)
    yield "one value", np.full(5000, 1.5, np.float32)
    yield "tiny", (g.standard_normal(20000) * 1e-30).astype(np.float32)          # subnormal fp16 and below
    yield "huge", (g.standard_normal(20000) * 1e30).astype(np.float32)           # beyond fp16: the inf bins
    yield "ulps", (np.float32(1) + np.arange(30000, dtype=np.float32) * np.float32(2.0 ** -23))
    x = g.standard_normal(20000).astype(np.float32)
    x[::7] = np.inf
    x[1::7] = -np.inf
    yield "infinities", x
    x = g.standard_normal(20000).astype(np.float32)
    x[::997] = np.nan
    x[5::991] = -np.nan
    yield "nan", x
    yield "signed zeros", np.where(g.random(4000) < 0.5, -0.0, 0.0).astype(np.float32)


@pytest.mark.parametrize("name,x", list(rows()))
def test_model_selects_the_top_k(orc, name, x):
    for k in (1, 2, 37, 2048, x.size):
        for n_cta in (2, 8):
            idx = model_topk(x, k, n_cta)
            assert idx.size == k and np.unique(idx).size == k, (name, k, n_cta, idx.size)
            got = np.sort(x[idx])[::-1]
            exp = np.sort(orc.topk_values(x[None, :], k)[0])[::-1]
            assert np.array_equal(got, exp, equal_nan=True), (name, k, n_cta)
