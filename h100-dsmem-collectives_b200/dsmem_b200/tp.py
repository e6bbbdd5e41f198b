"""Tensor-parallel AllReduce + RMSNorm across the GPUs of one node (one process per GPU).

`TPContext` owns this rank's communication buffer (signal words, an x region and a y region), shares its
CUDA IPC handle with the other ranks over the caller's process group (any torch.distributed backend:
the handles are small host objects), and maps the peers' buffers. `allreduce_rmsnorm` then runs the
fused kernel of include/dsmem_b200.h (dsmem_tp_allreduce_rmsnorm): y = RMSNorm(sum over ranks of x
(+ residual)) * w on every rank, bf16.

`nccl_allreduce_rmsnorm` is the baseline composition (ncclAllReduce, then the cluster RMSNorm) through the
same C ABI, with a communicator made by `NcclComm`.
"""
from __future__ import annotations

import ctypes

from . import DsmemError, Dtype, Status, _ok, lib

HANDLE_BYTES = 64     # DSMEM_TP_HANDLE_BYTES
NCCL_UID_BYTES = 128
LL_SLOT_MAX = 4 << 20          # bytes of one LL sender slot at most (min(2 * capacity, 4 MiB))
ONESHOT_DEFAULT = 16 << 20     # the context's default one-shot limit


def exchange_bytes(local: bytes, group=None) -> list:
    """Every rank's `local` bytes, in rank order (torch.distributed.all_gather_object over `group`)."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(local), group=group)
    for i, b in enumerate(out):
        if not isinstance(b, (bytes, bytearray)) or len(b) != len(local):
            raise ValueError(f"rank {i} sent {type(b).__name__} of {len(b) if b is not None else 0} bytes")
    return [bytes(b) for b in out]


def owned_rows(rows: int, tp: int, rank: int) -> tuple:
    """Rows [lo, hi) whose reduction and normalisation rank `rank` performs (the kernel's split)."""
    if not 0 <= rank < tp:
        raise ValueError("rank out of range")
    return rank * rows // tp, (rank + 1) * rows // tp


def tp_bytes(tokens: int, hidden: int) -> int:
    """Capacity of each of the x / y regions for a [tokens, hidden] bf16 tensor."""
    return int(tokens) * int(hidden) * 2


class TPContext:
    """This rank's mapping of every rank's TP buffer. Collective: every rank of `group` constructs it."""

    def __init__(self, capacity_bytes: int, rank: int | None = None, world: int | None = None, group=None,
                 exchange=None):
        import torch.distributed as dist

        self.rank = dist.get_rank(group) if rank is None else int(rank)
        self.world = dist.get_world_size(group) if world is None else int(world)
        self._ctx = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        _ok(lib().dsmem_tp_alloc(int(capacity_bytes), ctypes.byref(self._ctx), handle), "dsmem_tp_alloc")
        try:
            handles = (exchange or (lambda b: exchange_bytes(b, group)))(handle.raw)
            if len(handles) != self.world:
                raise ValueError(f"{len(handles)} handles for {self.world} ranks")
            joined = ctypes.create_string_buffer(b"".join(handles), HANDLE_BYTES * self.world)
            _ok(lib().dsmem_tp_open(self._ctx, self.rank, self.world, joined), "dsmem_tp_open")
        except BaseException:
            lib().dsmem_tp_close(self._ctx)
            self._ctx = None
            raise
        x, y, cap = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_size_t()
        _ok(lib().dsmem_tp_buffers(self._ctx, ctypes.byref(x), ctypes.byref(y), ctypes.byref(cap)), "dsmem_tp_buffers")
        self._x, self._y, self.capacity = x.value, y.value, cap.value
        self._limit = ONESHOT_DEFAULT

    def buffers(self, tokens: int, hidden: int):
        """bf16 CUDA tensors [tokens, hidden] viewing the x and y regions (zero-copy input / output)."""
        import torch

        if tp_bytes(tokens, hidden) > self.capacity:
            raise DsmemError(Status.SCRATCH_LIMIT, "TPContext.buffers")

        class _View:
            def __init__(self, ptr):
                self.__cuda_array_interface__ = {"shape": (tokens, hidden), "typestr": "<i2", "data": (ptr, False),
                                                 "version": 3}

        dev = torch.device("cuda", torch.cuda.current_device())
        return tuple(torch.as_tensor(_View(p), device=dev).view(torch.bfloat16) for p in (self._x, self._y))

    def allreduce_rmsnorm(self, x, w, eps=1e-6, residual=None, out=None, cluster_size=8, stream=None):
        """y = RMSNorm(sum over ranks of x (+ residual)) * w on this rank. x [tokens, hidden] bf16 CUDA
        (None: already in the x region of `buffers`); out None leaves y in the y region (returned)."""
        import torch

        if x is not None:
            tokens, hidden = x.shape
        elif out is not None:
            tokens, hidden = out.shape
        else:
            raise ValueError("give x or out (the shape)")
        for t in [w] + [t for t in (x, residual, out) if t is not None]:
            if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("bf16 contiguous CUDA tensors expected")
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        _ok(lib().dsmem_tp_allreduce_rmsnorm(self._ctx, int(Dtype.BF16), x.data_ptr() if x is not None else None,
                                             residual.data_ptr() if residual is not None else None, w.data_ptr(),
                                             float(eps), tokens, hidden, int(cluster_size),
                                             out.data_ptr() if out is not None else None, ctypes.c_void_p(s or None)),
            f"dsmem_tp_allreduce_rmsnorm({tokens}x{hidden}, tp={self.world}, cluster {cluster_size})")
        return out if out is not None else self.buffers(tokens, hidden)[1]

    def set_wait_limit_ns(self, ns):
        """Limit of each cross-GPU flag wait of this context's calls (dsmem_tp_set_wait_limit_ns; default 2 s)."""
        _ok(lib().dsmem_tp_set_wait_limit_ns(self._ctx, int(ns)), "dsmem_tp_set_wait_limit_ns")

    def set_oneshot_limit(self, nbytes):
        """Use the one-shot form while the LL bytes this rank sends, (tp - 1) * rows * hidden * 4, stay within
        `nbytes` (dsmem_tp_set_oneshot_limit; 0: always the two-shot; default 16 MiB)."""
        _ok(lib().dsmem_tp_set_oneshot_limit(self._ctx, int(nbytes)), "dsmem_tp_set_oneshot_limit")
        self._limit = int(nbytes)

    def oneshot_fits(self, tokens, hidden):
        """Whether a [tokens, hidden] tensor fits one LL slot of this context (the one-shot form's room)."""
        return int(tokens) * int(hidden) * 4 <= min(2 * self.capacity, LL_SLOT_MAX)

    def oneshot_picked(self, tokens, hidden):
        """Whether a call of this shape runs the one-shot form under the current limit (the C ABI's rule)."""
        ll = int(tokens) * int(hidden) * 4
        return self.world > 1 and self.oneshot_fits(tokens, hidden) and (self.world - 1) * ll <= self._limit

    def status(self):
        """(status, error bits, detail) of the device error words, read and cleared (dsmem_tp_check); no raise."""
        bits, detail = ctypes.c_uint(0), ctypes.c_uint(0)
        st = lib().dsmem_tp_check(self._ctx, ctypes.byref(bits), ctypes.byref(detail))
        return Status(st), bits.value, detail.value

    def check(self):
        """Raise DsmemError(TIMEOUT/BOUNDS) if a device-side wait or check fired since the last call."""
        bits, detail = ctypes.c_uint(0), ctypes.c_uint(0)
        st = lib().dsmem_tp_check(self._ctx, ctypes.byref(bits), ctypes.byref(detail))
        _ok(st, f"dsmem_tp_check (detail {detail.value:#x})")

    def close(self):
        if self._ctx is not None:
            _ok(lib().dsmem_tp_close(self._ctx), "dsmem_tp_close")
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class NcclComm:
    """An NCCL communicator made through the C ABI (for dsmem_tp_allreduce_rmsnorm_nccl). Collective."""

    def __init__(self, rank: int | None = None, world: int | None = None, group=None, exchange=None):
        import torch.distributed as dist

        self.rank = dist.get_rank(group) if rank is None else int(rank)
        self.world = dist.get_world_size(group) if world is None else int(world)
        uid = ctypes.create_string_buffer(NCCL_UID_BYTES)
        if self.rank == 0:
            _ok(lib().dsmem_nccl_unique_id(uid), "dsmem_nccl_unique_id")
        uids = (exchange or (lambda b: exchange_bytes(b, group)))(uid.raw)
        root = ctypes.create_string_buffer(uids[0], NCCL_UID_BYTES)
        self._comm = ctypes.c_void_p()
        _ok(lib().dsmem_nccl_comm_init(self.world, self.rank, root, ctypes.byref(self._comm)), "dsmem_nccl_comm_init")

    def allreduce_rmsnorm(self, x, w, sum_buf, out, eps=1e-6, residual=None, cluster_size=8, stream=None):
        import torch

        tokens, hidden = x.shape
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        _ok(lib().dsmem_tp_allreduce_rmsnorm_nccl(self._comm, int(Dtype.BF16), x.data_ptr(),
                                                  residual.data_ptr() if residual is not None else None, w.data_ptr(),
                                                  float(eps), tokens, hidden, int(cluster_size), sum_buf.data_ptr(),
                                                  out.data_ptr(), ctypes.c_void_p(s or None)),
            "dsmem_tp_allreduce_rmsnorm_nccl")
        return out

    def close(self):
        if self._comm:
            _ok(lib().dsmem_nccl_comm_destroy(self._comm), "dsmem_nccl_comm_destroy")
            self._comm = ctypes.c_void_p()
