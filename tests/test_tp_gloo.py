"""Host logic of the tensor-parallel path on CPU: two gloo ranks (127.0.0.1), no GPU.

* the IPC-handle exchange returns every rank's bytes in rank order on every rank;
* the row ownership of the fused kernel (reduce-scatter by rows) tiles [0, rows) exactly once;
* the oracle's TP formula equals the sum of the ranks followed by the single-GPU RMSNorm formula.
"""
import os
import socket

import numpy as np
import torch.multiprocessing as mp

from dsmem_b200 import tp as T


def test_owned_rows_tile_the_tensor():
    for rows in (0, 1, 7, 64, 1024, 8191):
        for tp in (1, 2, 4, 8):
            covered = []
            for r in range(tp):
                lo, hi = T.owned_rows(rows, tp, r)
                covered.extend(range(lo, hi))
            assert covered == list(range(rows))


def test_tp_oracle_is_sum_then_rmsnorm(orc):
    xs = [orc.normal(1, 3 * 128, s).reshape(3, 128) for s in range(4)]
    w = orc.normal(1, 128, 99, 1.0, 0.02)
    res = orc.normal(1, 3 * 128, 98).reshape(3, 128)
    y = orc.tp_rmsnorm(1, xs, w, 1e-6, res)
    h = sum(orc.bf16_to_f32(x).astype(np.float64) for x in xs) + orc.bf16_to_f32(res)
    ref = h / np.sqrt((h * h).mean(axis=1, keepdims=True) + 1e-6) * orc.bf16_to_f32(w)
    assert np.allclose(y, ref, rtol=1e-12, atol=1e-12)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = bytes([rank]) * T.HANDLE_BYTES
        q.put((rank, T.exchange_bytes(local)))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert got[r] == [bytes([k]) * T.HANDLE_BYTES for k in range(world)]
