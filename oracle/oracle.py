"""ctypes wrapper of oracle/_build/liboracle.so -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import this module. It restates the
reference harness's host code (collectives/harness/main.cu:118-173) in C; see dsmem_oracle.h.
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"

F32, BF16, I32 = 0, 1, 2
ALLREDUCE, ALLGATHER, REDUCESCATTER, ALLTOALL = 0, 1, 2, 3
BROADCAST = 4   # B200 extension: rank 0's vector to every rank (no reference file)
REDUCE, GATHER, SCATTER = 5, 6, 7   # B200 extensions rooted at rank 0 (no reference file)
NP_DTYPE = {F32: np.float32, BF16: np.uint16, I32: np.int32}  # bf16 carried as raw uint16 bits

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        vp, sz, i, d, u64, i64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_double, ctypes.c_uint64, ctypes.c_int64
        L.orc_fill_pattern_a.argtypes = [i, vp, sz]
        L.orc_fill_pattern_b.argtypes = [i, vp, sz]
        L.orc_fill_uniform_real.argtypes = [i, vp, sz, u64, d, d]
        L.orc_fill_uniform_int.argtypes = [vp, sz, u64, i64, i64]
        L.orc_fill_normal.argtypes = [i, vp, sz, u64, d, d]
        L.orc_reference.argtypes = [i, i, i, sz, ctypes.c_longlong, vp, vp]
        L.orc_check.argtypes = [i, sz, vp, vp, i, d, ctypes.POINTER(d), ctypes.POINTER(d)]
        L.orc_check.restype = ctypes.c_longlong
        L.orc_rmsnorm.argtypes = [i, sz, sz, vp, vp, vp, d, vp, vp]
        L.orc_sum_ranks.argtypes = [i, sz, sz, ctypes.POINTER(vp), vp]
        L.orc_tp_rmsnorm.argtypes = [i, sz, sz, sz, ctypes.POINTER(vp), vp, vp, d, vp]
        ll = ctypes.c_longlong
        L.orc_decoder_layer.argtypes = [i, i, i, i, i, ll, ll] + [vp] * 10 + [vp, vp, d] + [vp] * 5
        L.orc_mt64_seed.argtypes = [vp, u64]
        L.orc_mt64_next.argtypes = [vp]
        L.orc_mt64_next.restype = u64
        L.orc_uniform_int.argtypes = [vp, i64, i64]
        L.orc_uniform_int.restype = i64
        L.orc_uniform_real.argtypes = [vp, d, d]
        L.orc_uniform_real.restype = d
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_rowwise_quant.argtypes = [sz, sz, vp, vp, vp]
        L.orc_quantize_i8.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_quantize_i8.restype = i
        L.orc_lars_momentum.argtypes = [sz, sz, vp, vp, vp, d, d, d, d, d, vp, vp]
        L.orc_lars_update.argtypes = [d, d, d, d, d]
        L.orc_lars_update.restype = d
        L.orc_layernorm_backward.argtypes = [sz, sz, vp, vp, vp, d, vp]
        L.orc_pearson_backward.argtypes = [sz, sz, vp, vp, vp, d, vp, vp]
        L.orc_softmax_logits_backward.argtypes = [sz, sz, vp, vp, vp]
        L.orc_weighted_var_backward.argtypes = [sz, sz, vp, vp, vp, d, vp]
        L.orc_wvar_backward_value.argtypes = [d] * 8
        L.orc_wvar_backward_value.restype = d
        L.orc_topk_values.argtypes = [sz, sz, sz, vp, vp]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def in_elems(op, n, m):
    return m if op in (ALLREDUCE, ALLGATHER, BROADCAST, REDUCE, GATHER) else n * m


def out_elems(op, n, m):
    return m if op in (ALLREDUCE, REDUCESCATTER, BROADCAST, REDUCE, SCATTER) else n * m


def written(op, n, m, clusters):
    """Boolean mask over a batch's output: the elements the collective writes. REDUCE and GATHER write rank 0's out
    block of each problem only (the other blocks keep their contents); every other op writes every element."""
    oe = out_elems(op, n, m)
    mask = np.ones(clusters * n * oe, dtype=bool)
    if op in (REDUCE, GATHER):
        mask.reshape(clusters, n, oe)[:, 1:, :] = False
    return mask


def pattern_a(dtype, count):
    a = np.empty(count, NP_DTYPE[dtype])
    lib().orc_fill_pattern_a(dtype, _p(a), count)
    return a


def pattern_b(dtype, count):
    a = np.empty(count, NP_DTYPE[dtype])
    lib().orc_fill_pattern_b(dtype, _p(a), count)
    return a


def uniform_real(dtype, count, seed, lo=-1.0, hi=1.0):
    a = np.empty(count, NP_DTYPE[dtype])
    lib().orc_fill_uniform_real(dtype, _p(a), count, seed, lo, hi)
    return a


def uniform_int(count, seed, lo, hi):
    a = np.empty(count, np.int32)
    lib().orc_fill_uniform_int(_p(a), count, seed, lo, hi)
    return a


def normal(dtype, count, seed, mean=0.0, std=1.0):
    a = np.empty(count, NP_DTYPE[dtype])
    lib().orc_fill_normal(dtype, _p(a), count, seed, mean, std)
    return a


def reference(op, dtype, n, m, clusters, inp):
    inp = np.ascontiguousarray(inp)
    assert inp.size >= clusters * n * in_elems(op, n, m)
    ref = np.empty(clusters * n * out_elems(op, n, m), np.float64)
    lib().orc_reference(op, dtype, n, m, clusters, _p(inp), _p(ref))
    return ref


def check(dtype, out, ref, mode, tol=0.0):
    """(n_bad, max_abs, max_rel); mode 0 exact in the element type, 1 |err| <= tol*(1+|ref|)."""
    out = np.ascontiguousarray(out)
    ref = np.ascontiguousarray(ref, dtype=np.float64)
    assert out.size == ref.size, (out.size, ref.size)
    ma, mr = ctypes.c_double(0), ctypes.c_double(0)
    bad = lib().orc_check(dtype, out.size, _p(out), _p(ref), mode, tol, ctypes.byref(ma), ctypes.byref(mr))
    return int(bad), ma.value, mr.value


def rmsnorm(dtype, x, w, eps, res=None):
    rows, hidden = x.shape
    y = np.empty((rows, hidden), np.float64)
    pre = np.empty((rows, hidden), np.float64) if res is not None else None
    lib().orc_rmsnorm(dtype, rows, hidden, _p(np.ascontiguousarray(x)),
                      _p(np.ascontiguousarray(res)) if res is not None else None, _p(np.ascontiguousarray(w)), eps,
                      _p(y), _p(pre) if pre is not None else None)
    return y, pre


def sum_ranks(dtype, xs):
    xs = [np.ascontiguousarray(x) for x in xs]
    arr = (ctypes.c_void_p * len(xs))(*[x.ctypes.data for x in xs])
    out = np.empty(xs[0].size, np.float64)
    lib().orc_sum_ranks(dtype, len(xs), xs[0].size, arr, _p(out))
    return out


def tp_rmsnorm(dtype, xs, w, eps, res=None):
    """y (double) = RMSNorm(sum of the ranks' xs (+ res)) * w; xs: list of [rows, hidden] arrays."""
    xs = [np.ascontiguousarray(x) for x in xs]
    rows, hidden = xs[0].shape
    arr = (ctypes.c_void_p * len(xs))(*[x.ctypes.data for x in xs])
    y = np.empty((rows, hidden), np.float64)
    lib().orc_tp_rmsnorm(dtype, len(xs), rows, hidden, arr, _p(np.ascontiguousarray(res)) if res is not None else None,
                         _p(np.ascontiguousarray(w)), eps, _p(y))
    return y


def decoder_layer(inp, res, w_rms, wqkv, wo, w_post, wgu, wd, kc, vc, cos, sin, seq_len, eps, heads, head_dim=128):
    """Decoder-layer oracle (double): bf16 bit arrays in; returns dict of out, h, o, k_new, v_new (float64
    [batch, hidden]). kc / vc: [batch, cap, heads, head_dim] with seq_len valid tokens."""
    batch, hidden = inp.shape
    ffn = wd.shape[1]
    cap = kc.shape[1]
    arrs = [np.ascontiguousarray(a) for a in (inp, res, w_rms, wqkv, wo, w_post, wgu, wd, kc, vc)]
    cs = [np.ascontiguousarray(a, dtype=np.float32) for a in (cos, sin)]
    outs = {k: np.empty((batch, hidden), np.float64) for k in ("out", "h", "o", "k_new", "v_new")}
    lib().orc_decoder_layer(batch, hidden, heads, head_dim, ffn, seq_len, cap, *[_p(a) for a in arrs],
                            *[_p(c) for c in cs], eps, *[_p(outs[k]) for k in ("out", "h", "o", "k_new", "v_new")])
    return outs


# ------------------------------------------------------------------ row-wise reduction-reuse workloads
# The constants the reference kernels compile in (kernels/*__reduction_reuse__credit.cu), as float32 values.
LARS_DEFAULTS = dict(mu=float(np.float32(0.9)), wd=float(np.float32(0.01)), lr=float(np.float32(1.0e-3)),
                     eta=float(np.float32(0.02)), eps=float(np.float32(1e-6)))   # lars_momentum :29-33
LN_BWD_EPS = float(np.float32(1e-5))     # layernorm_backward :29
PEARSON_EPS = float(np.float32(1e-5))    # pearson_backward :29
WVAR_EPS = float(np.float32(1.0e-6))     # weighted_var_backward :29


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rowwise_quant(x):
    """(q int8 [rows, cols], scales float32 [rows]), bit-exact fp32 restatement."""
    x = _f32(x)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.int8)
    sc = np.empty(rows, np.float32)
    lib().orc_rowwise_quant(rows, cols, _p(x), _p(q), _p(sc))
    return q, sc


def lars_momentum(w, g, m, mu, wd, lr, eta, eps):
    w, g, m = _f32(w), _f32(g), _f32(m)
    rows, cols = w.shape
    wo, mo = np.empty((rows, cols)), np.empty((rows, cols))
    lib().orc_lars_momentum(rows, cols, _p(w), _p(g), _p(m), mu, wd, lr, eta, eps, _p(wo), _p(mo))
    return wo, mo


def layernorm_backward(x, dy, gamma, eps):
    x, dy, gamma = _f32(x), _f32(dy), _f32(gamma)
    rows, cols = x.shape
    dx = np.empty((rows, cols))
    lib().orc_layernorm_backward(rows, cols, _p(x), _p(dy), _p(gamma), eps, _p(dx))
    return dx


def pearson_backward(x, y, grad, eps):
    x, y, grad = _f32(x), _f32(y), _f32(grad)
    rows, cols = x.shape
    dx, dy = np.empty((rows, cols)), np.empty((rows, cols))
    lib().orc_pearson_backward(rows, cols, _p(x), _p(y), _p(grad), eps, _p(dx), _p(dy))
    return dx, dy


def softmax_logits_backward(z, dy):
    z, dy = _f32(z), _f32(dy)
    rows, cols = z.shape
    dx = np.empty((rows, cols))
    lib().orc_softmax_logits_backward(rows, cols, _p(z), _p(dy), _p(dx))
    return dx


def weighted_var_backward(x, w, dy, eps):
    x, w, dy = _f32(x), _f32(w), _f32(dy)
    rows, cols = x.shape
    dx = np.empty((rows, cols))
    lib().orc_weighted_var_backward(rows, cols, _p(x), _p(w), _p(dy), eps, _p(dx))
    return dx


def topk_values(x, k):
    """The k largest values of each row of x (float32 [rows, n]), sorted descending (torch.topk's order)."""
    x = _f32(x)
    rows, n = x.shape
    vals = np.empty((rows, k), np.float32)
    lib().orc_topk_values(rows, n, k, _p(x), _p(vals))
    return vals


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f):
    """Round-to-nearest-even float32 -> bf16 bits (numpy, vectorised)."""
    u = np.asarray(f, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


class MT64(ctypes.Structure):
    _fields_ = [("mt", ctypes.c_uint64 * 312), ("idx", ctypes.c_int)]


def mt64(seed):
    g = MT64()
    lib().orc_mt64_seed(ctypes.byref(g), seed)
    return g


def mt64_next(g):
    return lib().orc_mt64_next(ctypes.byref(g))
