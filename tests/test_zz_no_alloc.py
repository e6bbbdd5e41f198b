"""The allocation-free two-shot AllReduce entry point (dsmem_allreduce_two_shot_noalloc).

It serves callers that must not call cudaMalloc (stream capture in progress, a framework allocator that
owns the device memory, a fixed memory map): its scratch is a static device array instead of memory the
library allocates. This file checks, through the C ABI, that two calls in a row give the same results as
the regular entry point (dsmem_collective_launch, two-shot push, plain driver) within the tolerance of the
other parity tests, that they leave the device's free memory unchanged, and that batches above the static
limit are refused. It is collected last (test_zz_*) and also passes when run alone in a fresh process.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402

ORC_DT = {D.Dtype.F32: 0, D.Dtype.BF16: 1, D.Dtype.I32: 2}


def _inputs(torch, orc, dt, count, seed):
    if dt == D.Dtype.I32:
        host = orc.uniform_int(count, seed, -32768, 32767)
        return torch.from_numpy(host).cuda()
    host = orc.uniform_real(ORC_DT[dt], count, seed, -1.0, 1.0)
    if dt == D.Dtype.BF16:
        return torch.from_numpy(host.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(host).cuda()


def _np(t, dt):
    import torch

    t = t.cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if dt == D.Dtype.BF16 else t.numpy()


@pytest.mark.parametrize("dt", list(D.Dtype))
def test_noalloc_matches_regular_entry_point_twice(cuda, orc, dt):
    torch = cuda
    n, p, clusters = 8, 16384, 300
    m = D.msg_elems(D.Op.ALLREDUCE, n, p, dt)
    ins = [_inputs(torch, orc, dt, clusters * n * m, seed) for seed in (101, 202)]
    outs = [torch.empty_like(x) for x in ins]
    refs = [torch.empty_like(x) for x in ins]
    stream = torch.cuda.current_stream().cuda_stream
    # first call on the device: its set-up (the runtime loads the library's device code and static array,
    # the entry point looks up the array's address); later calls must not touch device memory at all
    D.allreduce_two_shot_noalloc(D.dtype_of(ins[0]), n, p, ins[0].data_ptr(), outs[0].data_ptr(), 1, stream)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for x, y in zip(ins, outs):   # two calls in a row, nothing allocated in between
        status = D.allreduce_two_shot_noalloc(D.dtype_of(x), n, p, x.data_ptr(), y.data_ptr(), clusters, stream)
        assert status == [0] * clusters
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc entry point changed free device memory"
    D.set_pipelined(False)
    try:
        for x, r in zip(ins, refs):
            D.collective(D.Op.ALLREDUCE, D.Alg.TWO_SHOT_PUSH, x, r, n, p)
        D.check()
    finally:
        D.set_pipelined(True)
    for y, r in zip(outs, refs):
        got = _np(y, dt)
        if dt == D.Dtype.BF16:
            want = orc.bf16_to_f32(_np(r, dt)).astype(np.float64)
        else:
            want = _np(r, dt).astype(np.float64)
        if dt == D.Dtype.I32:
            assert np.array_equal(got, _np(r, dt))
        else:
            tol = (1e-5 if dt == D.Dtype.F32 else 1e-2) * math.ceil(math.log2(n))
            bad, _, mr = orc.check(ORC_DT[dt], got, want, 1, tol)
            assert bad == 0, f"{bad} elements differ from the regular entry point (max rel {mr})"


def test_noalloc_rejects_batches_beyond_static_scratch(cuda):
    torch = cuda
    x = torch.zeros(64, device="cuda")
    with pytest.raises(D.DsmemError) as e:
        D.allreduce_two_shot_noalloc(D.Dtype.F32, 8, 256, x.data_ptr(), x.data_ptr(), D.NOALLOC_MAX_PROBLEMS + 1)
    assert e.value.status == D.Status.SCRATCH_LIMIT
