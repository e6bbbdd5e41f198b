"""GPU tests of the host-buffer entry point dsmem_collective_host: its results equal the device-buffer batch
launch on the same inputs (bit for bit: every chunk runs the algorithm AUTO picks for the whole batch), for every
op, ragged last chunks, page-locked and pageable host memory."""
import pytest

pytestmark = pytest.mark.gpu

import dsmem_b200 as D  # noqa: E402

CASES = [  # op, N, bytes per CTA, problems, problems per chunk (0: the default ~64 MiB)
    (D.Op.ALLREDUCE, 8, 65536, 300, 64),
    (D.Op.ALLREDUCE, 8, 16384, 33, 0),
    (D.Op.ALLREDUCE, 2, 4096, 5, 1),
    (D.Op.ALLGATHER, 4, 16384, 50, 7),
    (D.Op.REDUCESCATTER, 8, 65536, 20, 3),
    (D.Op.ALLTOALL, 8, 16384, 17, 5),
    (D.Op.BROADCAST, 8, 4096, 9, 2),
]


@pytest.mark.parametrize("op,n,p,problems,chunk", CASES)
@pytest.mark.parametrize("pinned", [True, False])
def test_host_matches_device(cuda, op, n, p, problems, chunk, pinned):
    torch = cuda
    m = D.msg_elems(op, n, p, D.Dtype.F32)
    per_in = n * D.in_elems_per_rank(op, n, m)
    per_out = n * D.out_elems_per_rank(op, n, m)
    g = torch.Generator(device="cuda")
    g.manual_seed(problems * 131 + n)
    din = torch.rand(problems * per_in, device="cuda", generator=g) * 2 - 1
    dout = torch.empty(problems * per_out, device="cuda")
    D.collective(op, D.Alg.AUTO, din, dout, n, p)
    D.check()
    hin = torch.empty(din.numel(), pin_memory=pinned)
    hin.copy_(din)
    hout = torch.full((dout.numel(),), float("nan"), pin_memory=pinned)
    D.collective_host(op, D.Alg.AUTO, hin, hout, n, p, chunk_clusters=chunk)
    assert torch.equal(hout, dout.cpu()), f"{op.name} N={n} P={p} problems={problems} chunk={chunk}"


@pytest.mark.parametrize("op,n,p,problems,chunk", [(D.Op.REDUCE, 8, 4096, 37, 5), (D.Op.GATHER, 4, 16384, 50, 7),
                                                    (D.Op.SCATTER, 16, 16384, 21, 4)])
def test_host_rooted_matches_device(cuda, op, n, p, problems, chunk):
    """The rooted ops on host buffers: rank 0's out blocks (every block for the Scatter) equal the device launch's,
    and for the Reduce and Gather the other ranks' host blocks keep their contents (only rank 0's are copied back)."""
    torch = cuda
    m = D.msg_elems(op, n, p, D.Dtype.F32)
    per_in = n * D.in_elems_per_rank(op, n, m)
    oe = D.out_elems_per_rank(op, n, m)
    g = torch.Generator(device="cuda")
    g.manual_seed(problems * 17 + n)
    din = torch.rand(problems * per_in, device="cuda", generator=g) * 2 - 1
    dout = torch.full((problems * n * oe,), 7.0, device="cuda")
    D.collective(op, D.Alg.AUTO, din, dout, n, p)
    D.check()
    hin = torch.empty(din.numel(), pin_memory=True)
    hin.copy_(din)
    hout = torch.full((dout.numel(),), float("nan"), pin_memory=True)
    D.collective_host(op, D.Alg.AUTO, hin, hout, n, p, chunk_clusters=chunk)
    got, want = hout.view(problems, n, oe), dout.cpu().view(problems, n, oe)
    if op in D.ROOT_OUT_ONLY:
        assert torch.equal(got[:, 0], want[:, 0]), f"{op.name}: rank 0's blocks differ"
        assert torch.isnan(got[:, 1:]).all(), f"{op.name}: a non-root host block was overwritten"
        assert (want[:, 1:] == 7.0).all(), f"{op.name}: a non-root device block was written"
    else:
        assert torch.equal(got, want), f"{op.name}: host result differs from the device launch"


def test_host_rejects_device_tensors(cuda):
    torch = cuda
    x = torch.zeros(8 * 1024, device="cuda")
    with pytest.raises(ValueError):
        D.collective_host(D.Op.ALLREDUCE, D.Alg.AUTO, x, x, 8, 4096)
