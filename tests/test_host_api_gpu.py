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


def test_host_rejects_device_tensors(cuda):
    torch = cuda
    x = torch.zeros(8 * 1024, device="cuda")
    with pytest.raises(ValueError):
        D.collective_host(D.Op.ALLREDUCE, D.Alg.AUTO, x, x, 8, 4096)
