"""Every reference-harness plugin build (lib/libdsmem_shims.so: 29 files x N in {2,4,8,16} x float / int, minus
the reference's skips) launched as collectives/harness/main.cu launches it -- one cluster of N CTAs, 256 threads,
sizeof(CollectiveSmem) of dynamic shared memory (main.cu:207-214, 273) -- on the harness's two input patterns,
against the CPU oracle (the restatement of main.cu:118-173, pinned to the reference's own fill_input() /
reference()):
  * pattern A (main.cu:119): every result an integer below 2^24, so exact for float and int;
  * pattern B (main.cu:121-124, mt19937_64(20261025), U(-1,1)): float within 1e-5 * (1 + |ref|) * ceil(log2 N)
    (main.cu:165), int exact; AllGather / AlltoAll exact.
Outputs are poisoned before each launch; the in-kernel stamps (entry <= every round <= exit) and the SM ids (N
distinct SMs) are checked as main.cu records them, and the build's device error word must stay clear.
This exercises dsb::run_single, the one-cluster driver these files delegate to.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from dsmem_b200 import shims  # noqa: E402

OPS = {"allreduce": 0, "allgather": 1, "reducescatter": 2, "alltoall": 3}
ORC_DT = {"float": 0, "int": 2}


def _elems(op, n, m):
    ins = m if op in ("allreduce", "allgather") else n * m
    outs = m if op in ("allreduce", "reducescatter") else n * m
    return n * ins, n * outs


@pytest.mark.parametrize("stem", shims.files())
def test_shim_builds_match_the_oracle(cuda, orc, stem):
    torch = cuda
    builds = [b for b in shims.manifest()["builds"] if b["stem"] == stem]
    if not builds:
        pytest.skip("every configuration is a reference skip")
    failures = []
    for b in builds:
        op, n, m, elem = b["op"], b["n"], b["msg_elems"], b["elem"]
        nin, nout = _elems(op, n, m)
        for pattern in ("A", "B"):
            host = orc.pattern_a(ORC_DT[elem], nin) if pattern == "A" else orc.pattern_b(ORC_DT[elem], nin)
            tin = torch.from_numpy(host.copy()).cuda()
            poison = 2 ** 31 - 1 if elem == "int" else -1
            tout = torch.full((nout,), poison, dtype=torch.int32, device="cuda")
            if elem == "float":
                tout = tout.view(torch.float32)
            ts = torch.zeros(n * 32, dtype=torch.int64, device="cuda")
            smid = torch.full((n,), -1, dtype=torch.int32, device="cuda")
            try:
                shims.launch(b["tag"], tin.data_ptr(), tout.data_ptr(), ts.data_ptr(), smid.data_ptr())
                err = shims.take_error(b["tag"])   # synchronises
                assert err == 0, f"device error word {err:#x}"
                got = tout.cpu().numpy()
                ref = orc.reference(OPS[op], ORC_DT[elem], n, m, 1, host)
                exact = pattern == "A" or elem == "int" or op in ("allgather", "alltoall")
                if exact:
                    bad, ma, _ = orc.check(ORC_DT[elem], got, ref, 0)
                    assert bad == 0, f"{bad} elements inexact (max abs {ma})"
                else:
                    tol = 1e-5 * math.ceil(math.log2(n))
                    bad, _, mr = orc.check(ORC_DT[elem], got, ref, 1, tol)
                    assert bad == 0, f"{bad} elements beyond {tol}*(1+|ref|) (max rel {mr})"
                st = ts.cpu().numpy().reshape(n, 32)
                assert (st[:, 0] > 0).all() and (st[:, 1] >= st[:, 0]).all(), "entry / exit stamps"
                rounds = st[:, 2:]
                for b_ in range(n):
                    r = rounds[b_][rounds[b_] > 0]
                    assert ((r >= st[b_, 0]) & (r <= st[b_, 1])).all(), "round stamps outside entry..exit"
                assert len(set(smid.cpu().numpy().tolist())) == n, "ranks of the cluster share an SM"
            except (AssertionError, RuntimeError) as e:
                failures.append(f"N={n} {elem} pattern {pattern}: {e}")
    assert not failures, "\n".join(failures)
