"""Host logic of bench.py's TP result check on CPU: two gloo ranks (127.0.0.1), no GPU.

bench.tp_check gathers every rank's x and y to rank 0 and checks y against the oracle's TP formula and the
ranks' outputs against each other. Here each rank's fused call is a stand-in (an all-reduce of x in fp32, then
RMSNorm and the weight in torch), so the check must pass; with a mistake planted in rank 1's output it must
fail and say that the ranks differ. Every rank takes the same collective steps either way (the test ends).
"""
import os
import socket

import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeCtx:
    """Stands in for TPContext: y = RMSNorm(sum over ranks of x) * w, computed in fp32 on the CPU."""

    def __init__(self, rank, plant):
        self.rank, self.plant = rank, plant

    def allreduce_rmsnorm(self, x, w, eps, residual=None, out=None, cluster_size=8):
        import torch
        import torch.distributed as dist

        h = x.float()
        dist.all_reduce(h)
        y = h * torch.rsqrt((h * h).mean(dim=1, keepdim=True) + eps) * w.float()
        out.copy_(y.to(torch.bfloat16))
        if self.plant and self.rank == 1:
            out[0, 0] = out[0, 0] + 1.0
        return out

    def oneshot_picked(self, tokens, hidden):
        return tokens <= 64


def _worker(rank, world, port, plant, q):
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "h100-dsmem-collectives_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.synchronize = lambda *a, **k: None   # no device here
    try:
        g = torch.Generator().manual_seed(1234 + rank)
        x = torch.randn(64, 1024, generator=g).to(torch.bfloat16)
        w = (1 + 0.02 * torch.randn(1024, generator=torch.Generator().manual_seed(1))).to(torch.bfloat16)
        res = bench.tp_check(torch, rank, world, _FakeCtx(rank, plant), 64, 1024, 8, x, w)
        skipped = bench.tp_check(torch, rank, world, _FakeCtx(rank, plant), 8, 1024, 8, x[:8], w)
        q.put((rank, res, skipped))
    finally:
        dist.destroy_process_group()


def _run(plant):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, plant, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, res, skipped = q.get(timeout=180)
        got[r] = (res, skipped)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return got


def test_tp_check_passes_on_a_correct_result():
    got = _run(plant=False)
    res0, skipped0 = got[0]
    assert got[1] == (None, None)   # only rank 0 reports
    assert skipped0 is None          # token counts other than 64 and 1,024 are not checked
    assert res0["ok"] and res0["ranks_bit_identical"] and res0["bad_elements"] == 0, res0
    assert res0["form"] == "one-shot"


def test_tp_check_fails_on_a_planted_mistake():
    res0, _ = _run(plant=True)[0]
    assert not res0["ok"] and not res0["ranks_bit_identical"], res0
