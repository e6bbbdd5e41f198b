"""The allocation-free two-shot AllReduce entry point (dsmem_allreduce_two_shot_noalloc).

Some callers cannot let a library allocate device memory: a framework whose caching allocator has reserved
the GPU's memory and accounts for every byte, or a program with a fixed memory map. This entry point keeps
its scratch in a static device array instead. Through the C ABI, this file checks that:
  * two calls in a row give the regular entry point's result (dsmem_collective_launch, two-shot push, plain
    driver) bit for bit -- same shots, same summation order -- and the oracle's within the parity tolerance;
  * after the first call on the device (its set-up), calls of every other dtype and cluster size leave the
    device's free memory unchanged (set-up resolved all twelve kernels);
  * a call made without a status array can have its device error bits read back by a zero-problem call;
  * batches above the static limit are refused.
It is collected last (test_zz_*) and also passes when run alone in a fresh process.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402

ORC_DT = {D.Dtype.F32: 0, D.Dtype.BF16: 1, D.Dtype.I32: 2}


def _host(orc, dt, count, seed):
    if dt == D.Dtype.I32:
        return orc.uniform_int(count, seed, -32768, 32767)
    return orc.uniform_real(ORC_DT[dt], count, seed, -1.0, 1.0)


def _dev(torch, host, dt):
    if dt == D.Dtype.BF16:
        return torch.from_numpy(host.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(host.copy()).cuda()


def _np(t, dt):
    import torch

    t = t.cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if dt == D.Dtype.BF16 else t.numpy()


def _regular(x, n, p):
    """The existing entry point, plain driver (the no-alloc kernel's summation order)."""
    r = x.new_empty(x.shape)
    D.set_pipelined(False)
    try:
        D.collective(D.Op.ALLREDUCE, D.Alg.TWO_SHOT_PUSH, x, r, n, p)
        D.check()
    finally:
        D.set_pipelined(True)
    return r


def _check_oracle(orc, got, host, dt, n, m, clusters):
    ref = orc.reference(int(D.Op.ALLREDUCE), ORC_DT[dt], n, m, clusters, host)
    if dt == D.Dtype.I32:
        bad, ma, _ = orc.check(ORC_DT[dt], got, ref, 0)
        assert bad == 0, f"{bad} int32 elements differ from the oracle (max abs {ma})"
    else:
        tol = (1e-5 if dt == D.Dtype.F32 else 1e-2) * math.ceil(math.log2(n))
        bad, _, mr = orc.check(ORC_DT[dt], got, ref, 1, tol)
        assert bad == 0, f"{bad} elements beyond {tol}*(1+|ref|) of the oracle (max rel {mr})"


@pytest.mark.parametrize("dt", list(D.Dtype))
def test_noalloc_matches_regular_entry_point_twice(cuda, orc, dt):
    torch = cuda
    n, p, clusters = 8, 16384, 300
    m = D.msg_elems(D.Op.ALLREDUCE, n, p, dt)
    hosts = [_host(orc, dt, clusters * n * m, seed) for seed in (101, 202)]
    ins = [_dev(torch, h, dt) for h in hosts]
    outs = [torch.empty_like(x) for x in ins]
    stream = torch.cuda.current_stream().cuda_stream
    # first call on the device (a no-op for the result): the set-up, if no earlier test made it
    D.allreduce_two_shot_noalloc(D.dtype_of(ins[0]), n, p, ins[0].data_ptr(), outs[0].data_ptr(), 1, stream)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for x, y in zip(ins, outs):   # two calls in a row, nothing allocated in between
        status = D.allreduce_two_shot_noalloc(D.dtype_of(x), n, p, x.data_ptr(), y.data_ptr(), clusters, stream)
        assert status == [0] * clusters
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc entry point changed free device memory"
    for h, x, y in zip(hosts, ins, outs):
        got, want = _np(y, dt), _np(_regular(x, n, p), dt)
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), \
            f"{int((got != want).sum())} elements differ from the regular entry point's bits"
        _check_oracle(orc, got, h, dt, n, m, clusters)


def test_noalloc_other_dtypes_and_cluster_sizes_allocate_nothing(cuda, orc):
    """The set-up (first call on the device) resolves every kernel, so later calls of other dtypes and cluster
    sizes load no code and leave the free memory unchanged; each result is the regular entry point's."""
    torch = cuda
    p, clusters = 4096, 40
    cases = [(dt, n) for dt in D.Dtype for n in D.CLUSTER_SIZES]
    data = []
    for k, (dt, n) in enumerate(cases):
        m = D.msg_elems(D.Op.ALLREDUCE, n, p, dt)
        h = _host(orc, dt, clusters * n * m, 300 + k)
        x = _dev(torch, h, dt)
        data.append((dt, n, m, h, x, torch.empty_like(x)))
    stream = torch.cuda.current_stream().cuda_stream
    dt0, n0, _, _, x0, y0 = data[0]
    D.allreduce_two_shot_noalloc(dt0, n0, p, x0.data_ptr(), y0.data_ptr(), 1, stream)   # set-up (if first)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for dt, n, _, _, x, y in reversed(data):
        assert D.allreduce_two_shot_noalloc(dt, n, p, x.data_ptr(), y.data_ptr(), clusters, stream) == [0] * clusters
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, \
        "a call of another dtype / cluster size after the set-up changed free device memory"
    for dt, n, m, h, x, y in data:
        got, want = _np(y, dt), _np(_regular(x, n, p), dt)
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), f"{dt.name} N={n}: differs from regular"
        _check_oracle(orc, got, h, dt, n, m, clusters)


def test_noalloc_without_status_then_read_back(cuda, orc):
    """status_out = NULL returns right after the launch; a zero-problem call then reads the error bits back."""
    torch = cuda
    dt, n, p, clusters = D.Dtype.F32, 16, 8192, 150
    m = D.msg_elems(D.Op.ALLREDUCE, n, p, dt)
    h = _host(orc, dt, clusters * n * m, 77)
    x = _dev(torch, h, dt)
    ys = [torch.empty_like(x), torch.empty_like(x)]
    stream = torch.cuda.current_stream().cuda_stream
    for y in ys:
        assert D.allreduce_two_shot_noalloc(dt, n, p, x.data_ptr(), y.data_ptr(), clusters, stream,
                                            want_status=False) is None
    st, bits = D.noalloc_last_error(stream)
    assert st == D.Status.OK and bits == 0
    want = _np(_regular(x, n, p), dt)
    for y in ys:
        assert np.array_equal(_np(y, dt).view(np.uint8), want.view(np.uint8))
    _check_oracle(orc, _np(ys[1], dt), h, dt, n, m, clusters)


def test_noalloc_rejects_batches_beyond_static_scratch(cuda):
    torch = cuda
    x = torch.zeros(64, device="cuda")
    with pytest.raises(D.DsmemError) as e:
        D.allreduce_two_shot_noalloc(D.Dtype.F32, 8, 256, x.data_ptr(), x.data_ptr(), D.NOALLOC_MAX_PROBLEMS + 1)
    assert e.value.status == D.Status.SCRATCH_LIMIT
