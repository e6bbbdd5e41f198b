"""dsmem_b200 -- Python host API of the B200 (sm_100a) DSMEM collective catalogue.

A thin ctypes layer over the C ABI in include/dsmem_b200.h (lib/libdsmem_b200.so). It mirrors the
reference's plugin interface: one collective = (op, alg, dtype, cluster size N, payload per CTA P),
the reference's compile-time knobs COLL_OP / <alg> / ELEM_T / CLUSTER_N / MSG_ELEMS
(collectives/harness/main.cu:1-10) as run-time arguments, run on a batch of independent cluster problems.
Errors are raised as DsmemError carrying the C status; there is no fallback: without the compiled
library every call fails.

Device memory and streams come from the caller (torch tensors in the convenience wrappers; raw device
pointers in `launch`).
"""
from __future__ import annotations

import ctypes
import enum
import pathlib

PKG_DIR = pathlib.Path(__file__).resolve().parent.parent
LIB_PATH = PKG_DIR / "lib" / "libdsmem_b200.so"
INCLUDE_DIR = PKG_DIR.parent / "include"
COLLECTIVES_DIR = PKG_DIR / "collectives"


class Op(enum.IntEnum):
    ALLREDUCE = 0
    ALLGATHER = 1
    REDUCESCATTER = 2
    ALLTOALL = 3
    BROADCAST = 4   # B200 extension (no reference file): rank 0's vector to every rank
    REDUCE = 5      # B200 extension: op over the ranks' vectors into rank 0 (other ranks' out not written)
    GATHER = 6      # B200 extension: the ranks' vectors into rank 0, in rank order (other ranks' out not written)
    SCATTER = 7     # B200 extension: block r of rank 0's input to rank r


class Alg(enum.IntEnum):
    AUTO = 0
    RING = 1
    RECURSIVE_DOUBLING = 2
    SHIFT_ACCUMULATE_BULK = 3
    SHIFT_ACCUMULATE_ATOMIC = 4
    DIRECT_REPLICATED_PUSH = 5
    PULL_REDUCE_SCATTER_PUSH_ALLGATHER = 6
    RABENSEIFNER = 7
    ONE_SHOT_PULL = 8
    TWO_SHOT_PUSH = 9
    REDUCE_BCAST_BINOMIAL = 10
    ATOMIC_ALL_PUSH = 11
    MESH_2D = 12
    DIRECT_SHIFT = 13
    BRUCK = 14
    DIRECT_PULL = 15
    GATHER_BCAST_BINOMIAL = 16
    RECURSIVE_HALVING = 17
    DIRECT_PUSH = 18
    PAIRWISE_EXCHANGE = 19
    PAIRWISE_XOR = 20
    SHIFT = 21
    RS_PUSH_GLOBAL_AG = 22   # B200 extension (no reference file): DSMEM reduce-scatter, all-gather via the outputs
    RING_CREDIT = 23         # B200 extension: ring AllReduce, a buffer + mbarrier per round (N <= 8)
    RECURSIVE_DOUBLING_CREDIT = 24   # B200 extension: recursive doubling, a buffer + mbarrier per round
    BINOMIAL = 25            # broadcast, reduce, gather, scatter (B200 extensions)
    BRUCK_CREDIT = 26        # B200 extension: allgather Bruck, a buffer range + mbarrier per round
    RECURSIVE_HALVING_CREDIT = 27   # B200 extension: reducescatter halving, a buffer + mbarrier per round
    RABENSEIFNER_CREDIT = 28  # B200 extension: Rabenseifner AllReduce, a buffer + mbarrier per round
    PAIRWISE_XOR_CREDIT = 29  # B200 extension: pairwise XOR AlltoAll, an mbarrier per round
    BINOMIAL_CREDIT = 30      # B200 extension: binomial reduce/gather + broadcast, a buffer + mbarrier per round
    SHIFT_ACCUMULATE_BULK_CREDIT = 31   # B200 extension: shift-accumulate bulk AllReduce (N = 4), per-round buffers


class Dtype(enum.IntEnum):
    F32 = 0
    BF16 = 1
    I32 = 2


class Status(enum.IntEnum):
    OK = 0
    ILLEGAL_CONFIG = 1
    SMEM_LIMIT = 2
    TIMEOUT = 3
    CUDA = 4
    INVALID_ARGUMENT = 5
    BOUNDS = 6
    NCCL = 7
    SCRATCH_LIMIT = 8


ELEM_BYTES = {Dtype.F32: 4, Dtype.BF16: 2, Dtype.I32: 4}
CLUSTER_SIZES = (2, 4, 8, 16)
STAMPS_PER_RANK = 32  # dsmem_primitives.cuh kStamps

# (op, alg) -> reference file stem collectives/<op>__<alg>__<src>.cu  (collectives/README.md:19-49)
CATALOGUE = {
    (Op.ALLREDUCE, Alg.RECURSIVE_DOUBLING): "allreduce__recursive_doubling__clusterfusion",
    (Op.ALLREDUCE, Alg.SHIFT_ACCUMULATE_BULK): "allreduce__shift_accumulate_bulk__clusterfusion",
    (Op.ALLREDUCE, Alg.SHIFT_ACCUMULATE_ATOMIC): "allreduce__shift_accumulate_atomic__clusterfusion",
    (Op.ALLREDUCE, Alg.DIRECT_REPLICATED_PUSH): "allreduce__direct_replicated_push__credit",
    (Op.ALLREDUCE, Alg.PULL_REDUCE_SCATTER_PUSH_ALLGATHER): "allreduce__pull_reduce_scatter_push_allgather__hpcops",
    (Op.ALLREDUCE, Alg.RING): "allreduce__ring__nccl",
    (Op.ALLREDUCE, Alg.RABENSEIFNER): "allreduce__rabenseifner__mpich",
    (Op.ALLREDUCE, Alg.ONE_SHOT_PULL): "allreduce__one_shot_pull__trtllm",
    (Op.ALLREDUCE, Alg.TWO_SHOT_PUSH): "allreduce__two_shot_push__trtllm",
    (Op.ALLREDUCE, Alg.REDUCE_BCAST_BINOMIAL): "allreduce__reduce_bcast_binomial__mpich",
    (Op.ALLREDUCE, Alg.ATOMIC_ALL_PUSH): "allreduce__atomic_all_push__generic",
    (Op.ALLREDUCE, Alg.MESH_2D): "allreduce__2d_mesh__generic",
    (Op.ALLGATHER, Alg.RECURSIVE_DOUBLING): "allgather__recursive_doubling__clusterfusion",
    (Op.ALLGATHER, Alg.DIRECT_SHIFT): "allgather__direct_shift__clusterfusion",
    (Op.ALLGATHER, Alg.DIRECT_REPLICATED_PUSH): "allgather__direct_replicated_push__credit",
    (Op.ALLGATHER, Alg.RING): "allgather__ring__nccl",
    (Op.ALLGATHER, Alg.BRUCK): "allgather__bruck__mpich",
    (Op.ALLGATHER, Alg.DIRECT_PULL): "allgather__direct_pull__generic",
    (Op.ALLGATHER, Alg.GATHER_BCAST_BINOMIAL): "allgather__gather_bcast_binomial__mpich",
    (Op.REDUCESCATTER, Alg.RING): "reducescatter__ring__nccl",
    (Op.REDUCESCATTER, Alg.RECURSIVE_HALVING): "reducescatter__recursive_halving__mpich",
    (Op.REDUCESCATTER, Alg.DIRECT_PUSH): "reducescatter__direct_push__generic",
    (Op.REDUCESCATTER, Alg.DIRECT_PULL): "reducescatter__direct_pull__generic",
    (Op.ALLTOALL, Alg.PAIRWISE_EXCHANGE): "alltoall__pairwise_exchange__fa4",
    (Op.ALLTOALL, Alg.DIRECT_PUSH): "alltoall__direct_push__generic",
    (Op.ALLTOALL, Alg.PAIRWISE_XOR): "alltoall__pairwise_xor__mpich",
    (Op.ALLTOALL, Alg.SHIFT): "alltoall__shift__generic",
    (Op.ALLTOALL, Alg.BRUCK): "alltoall__bruck__mpich",
    (Op.ALLTOALL, Alg.DIRECT_PULL): "alltoall__direct_pull__generic",
}


# Algorithms of this build with no reference file (selectable, and candidates for AUTO).
EXTENSIONS = {
    (Op.ALLREDUCE, Alg.RS_PUSH_GLOBAL_AG): "allreduce__rs_push_global_ag (B200 extension)",
    (Op.ALLREDUCE, Alg.RING_CREDIT): "allreduce__ring_credit (B200 extension)",
    (Op.ALLREDUCE, Alg.RECURSIVE_DOUBLING_CREDIT): "allreduce__recursive_doubling_credit (B200 extension)",
    (Op.ALLGATHER, Alg.RING_CREDIT): "allgather__ring_credit (B200 extension)",
    (Op.ALLGATHER, Alg.RECURSIVE_DOUBLING_CREDIT): "allgather__recursive_doubling_credit (B200 extension)",
    (Op.ALLGATHER, Alg.BRUCK_CREDIT): "allgather__bruck_credit (B200 extension)",
    (Op.REDUCESCATTER, Alg.RING_CREDIT): "reducescatter__ring_credit (B200 extension)",
    (Op.REDUCESCATTER, Alg.RECURSIVE_HALVING_CREDIT): "reducescatter__recursive_halving_credit (B200 extension)",
    (Op.ALLREDUCE, Alg.RABENSEIFNER_CREDIT): "allreduce__rabenseifner_credit (B200 extension)",
    (Op.ALLREDUCE, Alg.BINOMIAL_CREDIT): "allreduce__reduce_bcast_binomial_credit (B200 extension)",
    (Op.ALLREDUCE, Alg.SHIFT_ACCUMULATE_BULK_CREDIT): "allreduce__shift_accumulate_bulk_credit (B200 extension)",
    (Op.ALLGATHER, Alg.BINOMIAL_CREDIT): "allgather__gather_bcast_binomial_credit (B200 extension)",
    (Op.ALLTOALL, Alg.PAIRWISE_XOR_CREDIT): "alltoall__pairwise_xor_credit (B200 extension)",
    (Op.ALLTOALL, Alg.BRUCK_CREDIT): "alltoall__bruck_credit (B200 extension)",
    (Op.BROADCAST, Alg.DIRECT_PUSH): "broadcast__direct_push (B200 extension)",
    (Op.BROADCAST, Alg.DIRECT_PULL): "broadcast__direct_pull (B200 extension)",
    (Op.BROADCAST, Alg.BINOMIAL): "broadcast__binomial (B200 extension)",
    (Op.REDUCE, Alg.DIRECT_PUSH): "reduce__direct_push (B200 extension)",
    (Op.REDUCE, Alg.DIRECT_PULL): "reduce__direct_pull (B200 extension)",
    (Op.REDUCE, Alg.BINOMIAL): "reduce__binomial (B200 extension)",
    (Op.GATHER, Alg.DIRECT_PUSH): "gather__direct_push (B200 extension)",
    (Op.GATHER, Alg.DIRECT_PULL): "gather__direct_pull (B200 extension)",
    (Op.GATHER, Alg.BINOMIAL): "gather__binomial (B200 extension)",
    (Op.SCATTER, Alg.DIRECT_PUSH): "scatter__direct_push (B200 extension)",
    (Op.SCATTER, Alg.DIRECT_PULL): "scatter__direct_pull (B200 extension)",
    (Op.SCATTER, Alg.BINOMIAL): "scatter__binomial (B200 extension)",
}
# Ops whose collective writes rank 0's out block only (the other ranks' out blocks keep their contents).
ROOT_OUT_ONLY = (Op.REDUCE, Op.GATHER)


class DecoderParams(ctypes.Structure):
    """dsmem_decoder_params of include/dsmem_b200.h."""
    _fields_ = [("batch", ctypes.c_int), ("hidden", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("ffn", ctypes.c_int), ("seq_len", ctypes.c_longlong), ("cache_capacity", ctypes.c_longlong),
                ("cluster_size", ctypes.c_int), ("eps", ctypes.c_float)] + \
               [(k, ctypes.c_void_p) for k in ("inp", "res", "w_rms", "wqkv", "wo", "w_post", "wgu", "wd", "kcache",
                                               "vcache", "cos", "sin", "workspace")] + \
               [("workspace_bytes", ctypes.c_size_t)] + \
               [(k, ctypes.c_void_p) for k in ("out", "h_out", "o_out", "k_new", "v_new")]


class DsmemError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = Status(status)
        super().__init__(f"{what}: {self.status.name} ({_status_string(status)})")


_lib = None


def lib():
    """Load lib/libdsmem_b200.so (build it with `make -C h100-dsmem-collectives_b200 -j8`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR} -j8` "
                           "(there is no CPU fallback)")
    L = ctypes.CDLL(str(LIB_PATH))
    c_int, c_size, c_vp, c_ll, c_ull = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_ulonglong
    sig = {
        "dsmem_collective_launch": (c_int, [c_int, c_int, c_int, c_int, c_size, c_vp, c_vp, c_int, c_vp, c_vp]),
        "dsmem_collective_launch_ex": (c_int, [c_int, c_int, c_int, c_int, c_size, c_vp, c_vp, c_ll, c_vp, c_vp,
                                               c_int, c_vp]),
        "dsmem_query": (c_int, [c_int, c_int, c_int, c_int, c_size, ctypes.POINTER(c_size), ctypes.POINTER(c_int)]),
        "dsmem_max_active_clusters": (c_int, [c_int, c_int, c_int, c_int, c_size, ctypes.POINTER(c_int)]),
        "dsmem_autotune_table_load": (c_int, [ctypes.c_char_p]),
        "dsmem_autotune_pick": (c_int, [c_int, c_int, c_int, c_size]),
        "dsmem_autotune_pick_ex": (c_int, [c_int, c_int, c_int, c_size, c_ll]),
        "dsmem_last_error": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_last_error_detail": (c_int, [c_int] + [ctypes.POINTER(ctypes.c_uint)] * 3),
        "dsmem_check": (c_int, [c_vp]),
        "dsmem_op_name": (ctypes.c_char_p, [c_int]),
        "dsmem_alg_name": (ctypes.c_char_p, [c_int]),
        "dsmem_dtype_name": (ctypes.c_char_p, [c_int]),
        "dsmem_status_string": (ctypes.c_char_p, [c_int]),
        "dsmem_file_stem": (ctypes.c_char_p, [c_int, c_int]),
        "dsmem_lookup": (c_int, [ctypes.c_char_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
        "dsmem_set_wait_limit_ns": (c_int, [c_ull]),
        "dsmem_selftest_timeout": (c_int, [c_ull, c_vp]),
        "dsmem_set_pipelined": (c_int, [c_int]),
        "dsmem_set_pipeline_unit_bytes": (c_int, [c_size]),
        "dsmem_set_stream_pipeline": (c_int, [c_size, c_int, c_int]),
        "dsmem_allreduce_two_shot_noalloc": (c_int, [c_int, c_int, c_size, c_vp, c_vp, c_int,
                                                     ctypes.POINTER(ctypes.c_uint), c_vp]),
        "dsmem_rmsnorm_launch": (c_int, [c_int, c_vp, c_vp, ctypes.c_float, c_ll, c_int, c_int, c_vp, c_vp]),
        "dsmem_rmsnorm_residual_launch": (c_int, [c_int, c_vp, c_vp, c_vp, ctypes.c_float, c_ll, c_int, c_int,
                                                  c_vp, c_vp, c_vp]),
        "dsmem_rmsnorm_check": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_rowwise_quant_launch": (c_int, [c_vp, c_vp, c_vp, c_ll, c_int, c_int, c_vp]),
        "dsmem_lars_momentum_launch": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_int] + [ctypes.c_float] * 5
                                       + [c_int, c_vp]),
        "dsmem_layernorm_backward_launch": (c_int, [c_vp, c_vp, c_vp, c_vp, c_ll, c_int, ctypes.c_float, c_int, c_vp]),
        "dsmem_pearson_backward_launch": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_int, ctypes.c_float, c_int,
                                                  c_vp]),
        "dsmem_softmax_logits_backward_launch": (c_int, [c_vp, c_vp, c_vp, c_ll, c_int, c_int, c_vp]),
        "dsmem_weighted_var_backward_launch": (c_int, [c_vp, c_vp, c_vp, c_vp, c_ll, c_int, ctypes.c_float, c_int,
                                                       c_vp]),
        "dsmem_rowwise_check": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_rowwise_query": (c_int, [c_int, c_int, c_int, ctypes.POINTER(c_size), ctypes.POINTER(c_int),
                                        ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
        "dsmem_topk_query": (c_int, [c_int, c_int, ctypes.POINTER(c_size)]),
        "dsmem_topk_launch": (c_int, [c_vp, c_ll, c_int, c_int, c_vp, c_int, c_vp]),
        "dsmem_collective_host": (c_int, [c_int, c_int, c_int, c_int, c_size, c_vp, c_vp, c_ll, c_ll]),
        "dsmem_topk_check": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_ceiling_tcgen05": (c_int, [c_int, c_int, c_int, ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_int)]),
        "dsmem_ceiling_l2_bw": (c_int, [ctypes.c_longlong, c_int, c_int, ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_double)]),
        "dsmem_ceiling_smem_bw": (c_int, [c_int, c_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
        "dsmem_ceiling_dsmem_bw": (c_int, [c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(c_ll), ctypes.POINTER(c_int)]),
        "dsmem_version": (ctypes.c_char_p, []),
        "dsmem_tp_alloc": (c_int, [c_size, ctypes.POINTER(c_vp), c_vp]),
        "dsmem_tp_open": (c_int, [c_vp, c_int, c_int, c_vp]),
        "dsmem_tp_buffers": (c_int, [c_vp, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), ctypes.POINTER(c_size)]),
        "dsmem_tp_allreduce_rmsnorm": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, ctypes.c_float, c_ll, c_int, c_int,
                                               c_vp, c_vp]),
        "dsmem_tp_check": (c_int, [c_vp, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_tp_close": (c_int, [c_vp]),
        "dsmem_tp_set_wait_limit_ns": (c_int, [c_vp, c_ull]),
        "dsmem_tp_emulate": (c_int, [c_int, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), c_int, c_vp, c_vp,
                                     ctypes.c_float, c_ll, c_int, c_int, c_vp]),
        "dsmem_tp_emulate_oneshot": (c_int, [c_int, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), c_int, c_vp, c_vp,
                                             ctypes.c_float, c_ll, c_int, c_int, c_vp]),
        "dsmem_tp_emulate_check": (c_int, [ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_tp_set_oneshot_limit": (c_int, [c_vp, c_size]),
        "dsmem_decoder_workspace_bytes": (c_size, [c_int, c_int, c_int]),
        "dsmem_decoder_layer_launch": (c_int, [ctypes.POINTER(DecoderParams), c_vp]),
        "dsmem_decoder_check": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
        "dsmem_nccl_unique_id": (c_int, [c_vp]),
        "dsmem_nccl_comm_init": (c_int, [c_int, c_int, c_vp, ctypes.POINTER(c_vp)]),
        "dsmem_nccl_comm_destroy": (c_int, [c_vp]),
        "dsmem_tp_allreduce_rmsnorm_nccl": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, ctypes.c_float, c_ll, c_int, c_int,
                                                    c_vp, c_vp, c_vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _status_string(status):
    try:
        return lib().dsmem_status_string(int(status)).decode()
    except Exception:  # noqa: BLE001 - message only
        return "?"


def _ok(status, what):
    if status != 0:
        raise DsmemError(status, what)


# ----------------------------------------------------------------------------------- layouts
_ONE_BLOCK_PAYLOAD = (Op.ALLREDUCE, Op.BROADCAST, Op.REDUCE)   # P = M * sizeof(T); the other ops P = N * M * sizeof(T)


def msg_elems(op, n, bytes_per_cta, dtype):
    """M (elements per rank block) of payload P (nccl-tests convention, main.cu:97)."""
    unit = ELEM_BYTES[Dtype(dtype)] * (1 if Op(op) in _ONE_BLOCK_PAYLOAD else n)
    if bytes_per_cta % unit:
        raise ValueError(f"payload {bytes_per_cta} B is not a multiple of {unit} B")
    return bytes_per_cta // unit


def payload_bytes(op, n, m, dtype):
    return m * ELEM_BYTES[Dtype(dtype)] * (1 if Op(op) in _ONE_BLOCK_PAYLOAD else n)


def in_elems_per_rank(op, n, m):
    return m if Op(op) in (Op.ALLREDUCE, Op.ALLGATHER, Op.BROADCAST, Op.REDUCE, Op.GATHER) else n * m


def out_elems_per_rank(op, n, m):
    return m if Op(op) in (Op.ALLREDUCE, Op.REDUCESCATTER, Op.BROADCAST, Op.REDUCE, Op.SCATTER) else n * m


def algorithms(op):
    """Algorithms of the catalogue for `op`, in reference file order."""
    return [a for (o, a) in CATALOGUE if o == Op(op)]


# ----------------------------------------------------------------------------------- C ABI calls
def launch(op, alg, dtype, cluster_size, bytes_per_cta, in_ptr, out_ptr, num_clusters, stamps_ptr=0, smid_ptr=0,
           max_resident_clusters=0, stream=0):
    """dsmem_collective_launch_ex on raw device pointers (asynchronous on `stream`)."""
    st = lib().dsmem_collective_launch_ex(int(op), int(alg), int(dtype), int(cluster_size), int(bytes_per_cta),
                                          ctypes.c_void_p(in_ptr), ctypes.c_void_p(out_ptr), int(num_clusters),
                                          ctypes.c_void_p(stamps_ptr or None), ctypes.c_void_p(smid_ptr or None),
                                          int(max_resident_clusters), ctypes.c_void_p(stream or None))
    _ok(st, f"dsmem_collective_launch({Op(op).name}, {Alg(alg).name}, {Dtype(dtype).name}, N={cluster_size}, "
            f"P={bytes_per_cta})")


def query(op, alg, dtype, cluster_size, bytes_per_cta):
    """(status, smem_bytes, legal) without touching the GPU."""
    smem = ctypes.c_size_t(0)
    legal = ctypes.c_int(0)
    st = lib().dsmem_query(int(op), int(alg), int(dtype), int(cluster_size), int(bytes_per_cta), ctypes.byref(smem),
                           ctypes.byref(legal))
    return Status(st), smem.value, bool(legal.value)


def max_active_clusters(op, alg, dtype, cluster_size, bytes_per_cta):
    n = ctypes.c_int(0)
    _ok(lib().dsmem_max_active_clusters(int(op), int(alg), int(dtype), int(cluster_size), int(bytes_per_cta),
                                        ctypes.byref(n)), "dsmem_max_active_clusters")
    return n.value


def check(stream=0):
    """Synchronise `stream` and raise DsmemError(TIMEOUT/BOUNDS) if a device-side check fired."""
    _ok(lib().dsmem_check(ctypes.c_void_p(stream or None)), "dsmem_check")


def last_error(device=0):
    bits = ctypes.c_uint(0)
    _ok(lib().dsmem_last_error(int(device), ctypes.byref(bits)), "dsmem_last_error")
    return bits.value


def last_error_detail(device=0):
    """Read and clear the error words: {"bits", "timeout": None or {"barrier", "rank", "unit", "cluster"}}."""
    bits, detail, cluster = ctypes.c_uint(0), ctypes.c_uint(0), ctypes.c_uint(0)
    _ok(lib().dsmem_last_error_detail(int(device), ctypes.byref(bits), ctypes.byref(detail), ctypes.byref(cluster)),
        "dsmem_last_error_detail")
    d = detail.value
    timeout = None
    if d & 0x80000000:
        timeout = {"barrier": (d >> 24) & 0x7F, "rank": (d >> 16) & 0xFF, "unit": d & 0xFFFF, "cluster": cluster.value}
    return {"bits": bits.value, "timeout": timeout}


def set_wait_limit_ns(ns):
    _ok(lib().dsmem_set_wait_limit_ns(int(ns)), "dsmem_set_wait_limit_ns")


def set_pipelined(enable):
    """Use (True, default) or bypass (False) the pipelined batch drivers."""
    _ok(lib().dsmem_set_pipelined(1 if enable else 0), "dsmem_set_pipelined")


def set_pipeline_unit_bytes(nbytes):
    """Largest sub-vector per CTA of the pipelined drivers (default 16 KiB)."""
    _ok(lib().dsmem_set_pipeline_unit_bytes(int(nbytes)), "dsmem_set_pipeline_unit_bytes")


def set_stream_pipeline(unit_bytes=0, depth=0, lag=0):
    """Sub-vector size, input stages (0: by cluster size) and slot stages (units of reduce-scatter in flight) of the
    streamed rs_push_global_ag driver; no arguments restore the measured defaults (which adapt to one-wave launches)."""
    _ok(lib().dsmem_set_stream_pipeline(int(unit_bytes), int(depth), int(lag)), "dsmem_set_stream_pipeline")


def autotune_load(path):
    _ok(lib().dsmem_autotune_table_load(str(path).encode()), f"dsmem_autotune_table_load({path})")


def autotune_pick(op, dtype, cluster_size, bytes_per_cta, num_clusters=1):
    """The algorithm AUTO runs for a launch of num_clusters problems (measured table, then built-in order)."""
    return Alg(lib().dsmem_autotune_pick_ex(int(op), int(dtype), int(cluster_size), int(bytes_per_cta),
                                            int(num_clusters)))


def file_stem(op, alg):
    s = lib().dsmem_file_stem(int(op), int(alg))
    return s.decode() if s else None


def lookup(stem):
    op, alg = ctypes.c_int(0), ctypes.c_int(0)
    _ok(lib().dsmem_lookup(stem.encode(), ctypes.byref(op), ctypes.byref(alg)), f"dsmem_lookup({stem})")
    return Op(op.value), Alg(alg.value)


def selftest_timeout(limit_ns, stream=0):
    """Launch the bounded-wait self-test kernel (see dsmem_selftest_timeout)."""
    _ok(lib().dsmem_selftest_timeout(int(limit_ns), ctypes.c_void_p(stream or None)), "dsmem_selftest_timeout")


NOALLOC_MAX_PROBLEMS = 65536


def allreduce_two_shot_noalloc(dtype, cluster_size, bytes_per_cta, in_ptr, out_ptr, num_clusters, stream=0,
                               want_status=True):
    """Two-shot batch AllReduce that allocates no device memory (dsmem_allreduce_two_shot_noalloc), for
    callers that cannot let a library allocate device memory (a framework allocator that has reserved the
    GPU's memory, a fixed memory map). With want_status the call synchronises and returns the per-problem
    error bits (a list); otherwise it returns None right after the launch (see noalloc_last_error)."""
    status = (ctypes.c_uint * max(1, num_clusters))() if want_status else None
    st = lib().dsmem_allreduce_two_shot_noalloc(int(dtype), int(cluster_size), int(bytes_per_cta),
                                                ctypes.c_void_p(in_ptr), ctypes.c_void_p(out_ptr), int(num_clusters),
                                                status, ctypes.c_void_p(stream or None))
    _ok(st, f"dsmem_allreduce_two_shot_noalloc(N={cluster_size}, P={bytes_per_cta}, clusters={num_clusters})")
    return list(status)[:num_clusters] if want_status else None


def noalloc_last_error(stream=0):
    """The device error bits of the previous allocation-free call on this device (a num_clusters = 0 call of
    dsmem_allreduce_two_shot_noalloc: synchronises `stream`). Returns (status, bits) without raising."""
    word = (ctypes.c_uint * 1)()
    st = lib().dsmem_allreduce_two_shot_noalloc(int(Dtype.F32), 8, 16, None, None, 0, word,
                                                ctypes.c_void_p(stream or None))
    return Status(st), word[0]


def rmsnorm(x, w, eps=1e-6, cluster_size=8, out=None, residual=None, pre_norm=None, stream=None):
    """Cluster-fused RMSNorm of the rows of x (torch CUDA tensor [rows, hidden], bf16 or f32):
    y = h * rsqrt(mean(h^2) + eps) * w with h = x (+ residual, stored to pre_norm if given)."""
    import torch

    if x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA [rows, hidden] tensor")
    dt = dtype_of(x)
    rows, hidden = x.shape
    if out is None:
        out = torch.empty_like(x)
    s = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    for t in (w, out) + ((residual,) if residual is not None else ()) + ((pre_norm,) if pre_norm is not None else ()):
        if t.dtype != x.dtype or not t.is_contiguous() or not t.is_cuda:
            raise ValueError("w/out/residual/pre_norm must be contiguous CUDA tensors of x's dtype")
    if residual is None:
        st = lib().dsmem_rmsnorm_launch(int(dt), x.data_ptr(), w.data_ptr(), float(eps), rows, hidden,
                                        int(cluster_size), out.data_ptr(), ctypes.c_void_p(s or None))
    else:
        st = lib().dsmem_rmsnorm_residual_launch(int(dt), x.data_ptr(), residual.data_ptr(), w.data_ptr(), float(eps),
                                                 rows, hidden, int(cluster_size),
                                                 pre_norm.data_ptr() if pre_norm is not None else None,
                                                 out.data_ptr(), ctypes.c_void_p(s or None))
    _ok(st, f"dsmem_rmsnorm({dt.name}, {rows}x{hidden}, cluster {cluster_size})")
    return out


def rmsnorm_check(device=0):
    """Raise DsmemError(TIMEOUT) if an RMSNorm kernel's bounded wait gave up since the last check."""
    bits = ctypes.c_uint(0)
    _ok(lib().dsmem_rmsnorm_check(int(device), ctypes.byref(bits)), "dsmem_rmsnorm_check")
    if bits.value & 1:
        raise DsmemError(Status.TIMEOUT, "rmsnorm")


# ----------------------------------------------------------------------------------- row-wise workloads
# One cluster of cluster_size CTAs per row, one DSMEM exchange per row (dsmem_<name>_launch of
# include/dsmem_b200.h); fp32 CUDA tensors [rows, cols], outputs allocated when not given.
def _rw_prep(xs, outs, stream):
    import torch

    x0 = xs[0]
    if x0.dim() != 2 or not x0.is_cuda:
        raise ValueError("inputs must be CUDA [rows, cols] tensors")
    for t in list(xs) + [o for o in outs if o is not None]:
        if not t.is_cuda or not t.is_contiguous() or t.device != x0.device:
            raise ValueError("row-wise tensors must be contiguous and on one CUDA device")
    for t in xs:
        if t.dtype != torch.float32:
            raise ValueError("row-wise inputs are float32")
    s = stream if stream is not None else torch.cuda.current_stream(x0.device).cuda_stream
    return x0.shape[0], x0.shape[1], ctypes.c_void_p(s or None)


def rowwise_quant(x, cluster_size=8, q=None, scales=None, stream=None):
    """Row-wise int8 quantisation (rowwise_quant__reduction_reuse__credit.cu): returns (q int8, scales f32)."""
    import torch

    q = torch.empty(x.shape, dtype=torch.int8, device=x.device) if q is None else q
    scales = torch.empty(x.shape[0], dtype=torch.float32, device=x.device) if scales is None else scales
    rows, cols, s = _rw_prep([x], [q, scales], stream)
    _ok(lib().dsmem_rowwise_quant_launch(x.data_ptr(), q.data_ptr(), scales.data_ptr(), rows, cols, int(cluster_size),
                                         s), f"dsmem_rowwise_quant({rows}x{cols}, cluster {cluster_size})")
    return q, scales


def lars_momentum(weight, grad, momentum, cluster_size=8, momentum_coeff=0.9, weight_decay=0.01, lr=1.0e-3,
                  trust_coeff=0.02, eps=1e-6, weight_out=None, momentum_out=None, stream=None):
    """LARS momentum update (lars_momentum__reduction_reuse__credit.cu; defaults = its compiled-in constants):
    returns (weight_out, momentum_out)."""
    import torch

    weight_out = torch.empty_like(weight) if weight_out is None else weight_out
    momentum_out = torch.empty_like(weight) if momentum_out is None else momentum_out
    rows, cols, s = _rw_prep([weight, grad, momentum], [weight_out, momentum_out], stream)
    _ok(lib().dsmem_lars_momentum_launch(weight.data_ptr(), grad.data_ptr(), momentum.data_ptr(), weight_out.data_ptr(),
                                         momentum_out.data_ptr(), rows, cols, float(momentum_coeff),
                                         float(weight_decay), float(lr), float(trust_coeff), float(eps),
                                         int(cluster_size), s),
        f"dsmem_lars_momentum({rows}x{cols}, cluster {cluster_size})")
    return weight_out, momentum_out


def layernorm_backward(x, dy, gamma, eps=1e-5, cluster_size=8, dx=None, stream=None):
    """dx of LayerNorm (layernorm_backward__reduction_reuse__credit.cu); gamma [cols]."""
    import torch

    dx = torch.empty_like(x) if dx is None else dx
    rows, cols, s = _rw_prep([x, dy], [dx], stream)
    if gamma.numel() != cols or gamma.dtype != torch.float32 or not gamma.is_contiguous():
        raise ValueError("gamma must be a contiguous float32 [cols] tensor")
    _ok(lib().dsmem_layernorm_backward_launch(x.data_ptr(), dy.data_ptr(), gamma.data_ptr(), dx.data_ptr(), rows,
                                              cols, float(eps), int(cluster_size), s),
        f"dsmem_layernorm_backward({rows}x{cols}, cluster {cluster_size})")
    return dx


def pearson_backward(x, y, grad, eps=1e-5, cluster_size=8, dx=None, dy=None, stream=None):
    """(dx, dy) of the row-wise Pearson correlation (pearson_backward__reduction_reuse__credit.cu); grad [rows]."""
    import torch

    dx = torch.empty_like(x) if dx is None else dx
    dy = torch.empty_like(x) if dy is None else dy
    rows, cols, s = _rw_prep([x, y], [dx, dy], stream)
    if grad.numel() != rows or grad.dtype != torch.float32 or not grad.is_contiguous():
        raise ValueError("grad must be a contiguous float32 [rows] tensor")
    _ok(lib().dsmem_pearson_backward_launch(x.data_ptr(), y.data_ptr(), grad.data_ptr(), dx.data_ptr(), dy.data_ptr(),
                                            rows, cols, float(eps), int(cluster_size), s),
        f"dsmem_pearson_backward({rows}x{cols}, cluster {cluster_size})")
    return dx, dy


def softmax_logits_backward(logits, dy, cluster_size=8, dx=None, stream=None):
    """dx = p * (dy - sum(p * dy)), p = softmax(logits) per row (softmax_logits_backward__reduction_reuse__credit.cu)."""
    import torch

    dx = torch.empty_like(logits) if dx is None else dx
    rows, cols, s = _rw_prep([logits, dy], [dx], stream)
    _ok(lib().dsmem_softmax_logits_backward_launch(logits.data_ptr(), dy.data_ptr(), dx.data_ptr(), rows, cols,
                                                   int(cluster_size), s),
        f"dsmem_softmax_logits_backward({rows}x{cols}, cluster {cluster_size})")
    return dx


def weighted_var_backward(x, weights, dy, eps=1e-6, cluster_size=8, dx=None, stream=None):
    """dx of the row-wise weighted variance (weighted_var_backward__reduction_reuse__credit.cu)."""
    import torch

    dx = torch.empty_like(x) if dx is None else dx
    rows, cols, s = _rw_prep([x, weights, dy], [dx], stream)
    _ok(lib().dsmem_weighted_var_backward_launch(x.data_ptr(), weights.data_ptr(), dy.data_ptr(), dx.data_ptr(), rows,
                                                 cols, float(eps), int(cluster_size), s),
        f"dsmem_weighted_var_backward({rows}x{cols}, cluster {cluster_size})")
    return dx


def rowwise_check(device=0):
    """Raise DsmemError if a row-wise kernel's bounded wait gave up (TIMEOUT) or a copy failed its bounds check."""
    bits = ctypes.c_uint(0)
    _ok(lib().dsmem_rowwise_check(int(device), ctypes.byref(bits)), "dsmem_rowwise_check")
    if bits.value & 1:
        raise DsmemError(Status.TIMEOUT, "rowwise")
    if bits.value:
        raise DsmemError(Status.BOUNDS, "rowwise")


def topk(logits, k=2048, cluster_size=8, out=None, stream=None):
    """Exact top-k indices of every row of fp32 logits [rows, n] (dsmem_topk_launch; hpc-ops'
    topk_filtered_cluster8_exact_kernel). Returns int32 [rows, k], each row's indices in unspecified order."""
    import torch

    if logits.dim() != 2 or not logits.is_cuda or not logits.is_contiguous() or logits.dtype != torch.float32:
        raise ValueError("logits must be a contiguous float32 CUDA [rows, n] tensor")
    rows, n = logits.shape
    if out is None:
        out = torch.empty((rows, k), dtype=torch.int32, device=logits.device)
    if out.dtype != torch.int32 or not out.is_contiguous() or out.shape != (rows, k):
        raise ValueError("out must be a contiguous int32 [rows, k] tensor")
    s = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
    _ok(lib().dsmem_topk_launch(logits.data_ptr(), rows, n, int(k), out.data_ptr(), int(cluster_size),
                                ctypes.c_void_p(s or None)), f"dsmem_topk({rows}x{n}, k {k}, cluster {cluster_size})")
    return out


def topk_check(device=0):
    """Raise DsmemError if the top-k kernel's bounded wait gave up (TIMEOUT) or an output slot was out of range."""
    bits = ctypes.c_uint(0)
    _ok(lib().dsmem_topk_check(int(device), ctypes.byref(bits)), "dsmem_topk_check")
    if bits.value & 1:
        raise DsmemError(Status.TIMEOUT, "topk")
    if bits.value:
        raise DsmemError(Status.BOUNDS, "topk")


def decoder_layer(inp, res, w_rms, wqkv, wo, w_post, wgu, wd, kcache, vcache, cos, sin, seq_len, eps=1e-5,
                  cluster_size=8, out=None, h_out=None, o_out=None, k_new=None, v_new=None, workspace=None,
                  stream=None):
    """One decode step of the Llama-2-7B-shaped layer (dsmem_decoder_layer_launch). bf16 CUDA tensors:
    inp, res [B, hidden]; weights in nn.Linear layout; kcache / vcache [B, cap, heads, 128] with seq_len
    valid tokens (the step's k, v are stored at index seq_len); cos / sin fp32 [128]. Returns (out, h_out)."""
    import torch

    B, hidden = inp.shape
    heads, head_dim = kcache.shape[2], kcache.shape[3]
    ffn = wd.shape[1]
    out = torch.empty_like(inp) if out is None else out
    h_out = torch.empty_like(inp) if h_out is None else h_out
    need = lib().dsmem_decoder_workspace_bytes(B, hidden, ffn)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=inp.device)
    p = DecoderParams(batch=B, hidden=hidden, heads=heads, head_dim=head_dim, ffn=ffn, seq_len=int(seq_len),
                      cache_capacity=kcache.shape[1], cluster_size=int(cluster_size), eps=float(eps))
    for k, t in (("inp", inp), ("res", res), ("w_rms", w_rms), ("wqkv", wqkv), ("wo", wo), ("w_post", w_post),
                 ("wgu", wgu), ("wd", wd), ("kcache", kcache), ("vcache", vcache), ("cos", cos), ("sin", sin),
                 ("workspace", workspace), ("out", out), ("h_out", h_out), ("o_out", o_out), ("k_new", k_new),
                 ("v_new", v_new)):
        if t is not None:
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{k} must be a contiguous CUDA tensor")
            setattr(p, k, t.data_ptr())
    p.workspace_bytes = workspace.numel() * workspace.element_size()
    s = stream if stream is not None else torch.cuda.current_stream(inp.device).cuda_stream
    _ok(lib().dsmem_decoder_layer_launch(ctypes.byref(p), ctypes.c_void_p(s or None)),
        f"dsmem_decoder_layer_launch(B={B}, hidden={hidden}, ffn={ffn}, S={seq_len}, cluster {cluster_size})")
    return out, h_out


def decoder_check(device=0):
    """Raise DsmemError(TIMEOUT/BOUNDS) if a decoder kernel's device-side check fired since the last call."""
    bits = ctypes.c_uint(0)
    _ok(lib().dsmem_decoder_check(int(device), ctypes.byref(bits)), "dsmem_decoder_check")
    if bits.value & 1:
        raise DsmemError(Status.TIMEOUT, "decoder")
    if bits.value & 2:
        raise DsmemError(Status.BOUNDS, "decoder")


def tp_emulate(xs, ys, w, eps=1e-6, cluster_size=8, residual=None, stream=None, oneshot=False):
    """The tensor-parallel AllReduce+RMSNorm kernel for len(xs) ranks emulated on one GPU: every
    ys[k] = RMSNorm(sum(xs) (+ residual)) * w. bf16 CUDA tensors [rows, hidden]. oneshot=False: the two-shot
    kernel in one launch; True: the one-shot kernel, every rank's push launched before every rank's reduction."""
    import torch

    tp = len(xs)
    if len(ys) != tp or tp == 0:
        raise ValueError("xs and ys must have one tensor per rank")
    rows, hidden = xs[0].shape
    for t in list(xs) + list(ys) + [w] + ([residual] if residual is not None else []):
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("bf16 contiguous CUDA tensors expected")
    xa = (ctypes.c_void_p * tp)(*[x.data_ptr() for x in xs])
    ya = (ctypes.c_void_p * tp)(*[y.data_ptr() for y in ys])
    s = stream if stream is not None else torch.cuda.current_stream(xs[0].device).cuda_stream
    fn = lib().dsmem_tp_emulate_oneshot if oneshot else lib().dsmem_tp_emulate
    _ok(fn(tp, xa, ya, int(Dtype.BF16), residual.data_ptr() if residual is not None else None,
           w.data_ptr(), float(eps), rows, hidden, int(cluster_size), ctypes.c_void_p(s or None)),
        f"{fn.__name__}(tp={tp}, {rows}x{hidden}, cluster {cluster_size})")


def tp_emulate_check():
    """Raise DsmemError(TIMEOUT/BOUNDS) if a device-side wait or check of tp_emulate fired (synchronous)."""
    bits, detail = ctypes.c_uint(0), ctypes.c_uint(0)
    st = lib().dsmem_tp_emulate_check(ctypes.byref(bits), ctypes.byref(detail))
    _ok(st, f"dsmem_tp_emulate_check (detail {detail.value:#x})")


def dsmem_bandwidth_point(mode, cluster_size, passes, reps=5, ctas_per_sm=1):
    """(median ms, payload bytes, clusters) of one DSMEM ceiling launch configuration (mode 0 pull, 1 ring
    push, 2 all-peers push; ctas_per_sm 1 = 96 KiB tiles, 4 = 24 KiB tiles)."""
    ms, nbytes, cl = ctypes.c_double(0), ctypes.c_longlong(0), ctypes.c_int(0)
    _ok(lib().dsmem_ceiling_dsmem_bw(int(mode), int(cluster_size), int(ctas_per_sm), int(passes), int(reps),
                                     ctypes.byref(ms), ctypes.byref(nbytes), ctypes.byref(cl)), "dsmem_ceiling_dsmem_bw")
    return ms.value, nbytes.value, cl.value


def dsmem_bandwidth_peak(mode, cluster_size, passes=(4, 8, 16, 32), reps=5, ctas_per_sm=1):
    """GPU-wide SM-to-SM bandwidth in GB/s = 1 / slope of launch time over payload bytes (least squares),
    the method of the reference's roofline/harness/ceilings/src/dsmem_bw.cu. Returns (GB/s, points)."""
    pts = [dsmem_bandwidth_point(mode, cluster_size, p, reps, ctas_per_sm) for p in passes]
    xs = [b for (_, b, _) in pts]
    ys = [ms * 1e-3 for (ms, _, _) in pts]
    mx, my = sum(xs) / len(xs), sum(ys) / len(ys)
    slope = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / sum((x - mx) ** 2 for x in xs)
    return (1.0 / slope / 1e9 if slope > 0 else float("nan")), pts


def _slope_rate(points):
    """1 / slope of time (s) over work, least squares over (work, ms) points."""
    xs = [w for (w, _) in points]
    ys = [ms * 1e-3 for (_, ms) in points]
    mx, my = sum(xs) / len(xs), sum(ys) / len(ys)
    slope = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / sum((x - mx) ** 2 for x in xs)
    return 1.0 / slope if slope > 0 else float("nan")


def sm100_ceilings(reps=5):
    """Ceilings beyond DSMEM and HBM (1 / slope): tcgen05 bf16 MMA TFLOP/s (M 128, N 256), L2 read GB/s
    (64 MiB buffer) and shared-memory read GB/s, GPU-wide."""
    out = {}
    ms, work, ctas = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
    pts = []
    for iters in (256, 1024):
        _ok(lib().dsmem_ceiling_tcgen05(256, iters, reps, ctypes.byref(ms), ctypes.byref(work), ctypes.byref(ctas)),
            "dsmem_ceiling_tcgen05")
        pts.append((work.value, ms.value))
    out["tcgen05_bf16_m128n256_TFLOPs"] = round(_slope_rate(pts) / 1e12, 1)
    pts = []
    for passes in (4, 16):
        _ok(lib().dsmem_ceiling_l2_bw(64 << 20, passes, reps, ctypes.byref(ms), ctypes.byref(work)), "dsmem_ceiling_l2_bw")
        pts.append((work.value, ms.value))
    out["l2_read_GBps"] = round(_slope_rate(pts) / 1e9, 1)
    pts = []
    for passes in (64, 256):
        _ok(lib().dsmem_ceiling_smem_bw(passes, reps, ctypes.byref(ms), ctypes.byref(work)), "dsmem_ceiling_smem_bw")
        pts.append((work.value, ms.value))
    out["smem_read_GBps"] = round(_slope_rate(pts) / 1e9, 1)
    return out


def version():
    return lib().dsmem_version().decode()


# ----------------------------------------------------------------------------------- torch helpers
def dtype_of(tensor):
    import torch

    return {torch.float32: Dtype.F32, torch.bfloat16: Dtype.BF16, torch.int32: Dtype.I32}[tensor.dtype]


def collective_host(op, alg, inp, out, cluster_size, bytes_per_cta, num_clusters=None, chunk_clusters=0):
    """The batched collective on HOST tensors (torch CPU, contiguous; page-locked for overlapped copies), synchronous
    (dsmem_collective_host): copies in, the batch and copies out overlap in chunks on three streams."""
    dt = dtype_of(inp)
    if out.dtype != inp.dtype or inp.is_cuda or out.is_cuda:
        raise ValueError("inp/out must be host (CPU) tensors of the same dtype")
    if not (inp.is_contiguous() and out.is_contiguous()):
        raise ValueError("inp/out must be contiguous")
    m = msg_elems(op, cluster_size, bytes_per_cta, dt)
    per_in = cluster_size * in_elems_per_rank(op, cluster_size, m)
    per_out = cluster_size * out_elems_per_rank(op, cluster_size, m)
    if num_clusters is None:
        num_clusters = inp.numel() // per_in
    if inp.numel() < num_clusters * per_in or out.numel() < num_clusters * per_out:
        raise ValueError(f"tensors too small for {num_clusters} cluster problems")
    _ok(lib().dsmem_collective_host(int(op), int(alg), int(dt), int(cluster_size), int(bytes_per_cta), inp.data_ptr(),
                                    out.data_ptr(), int(num_clusters), int(chunk_clusters)),
        f"dsmem_collective_host({Op(op).name}, {Alg(alg).name}, N={cluster_size}, P={bytes_per_cta})")
    return out


def collective(op, alg, inp, out, cluster_size, bytes_per_cta, num_clusters=None, stamps=None, smid=None,
               max_resident_clusters=0, stream=None):
    """Run one batched collective on torch CUDA tensors (contiguous, cluster-major layout of
    include/dsmem_b200.h). num_clusters defaults to what `inp` holds."""
    import torch

    dt = dtype_of(inp)
    if out.dtype != inp.dtype or not (inp.is_cuda and out.is_cuda):
        raise ValueError("inp/out must be CUDA tensors of the same dtype")
    if not (inp.is_contiguous() and out.is_contiguous()):
        raise ValueError("inp/out must be contiguous")
    m = msg_elems(op, cluster_size, bytes_per_cta, dt)
    per_in = cluster_size * in_elems_per_rank(op, cluster_size, m)
    per_out = cluster_size * out_elems_per_rank(op, cluster_size, m)
    if num_clusters is None:
        num_clusters = inp.numel() // per_in
    if inp.numel() < num_clusters * per_in or out.numel() < num_clusters * per_out:
        raise ValueError(f"tensors too small for {num_clusters} cluster problems")
    if stamps is not None and (stamps.dtype != torch.int64 or stamps.numel() < num_clusters * cluster_size * STAMPS_PER_RANK):
        raise ValueError("stamps must be int64 with num_clusters*N*32 entries")
    if smid is not None and (smid.dtype != torch.int32 or smid.numel() < num_clusters * cluster_size):
        raise ValueError("smid must be int32 with num_clusters*N entries")
    s = stream if stream is not None else torch.cuda.current_stream(inp.device).cuda_stream
    launch(op, alg, dt, cluster_size, bytes_per_cta, inp.data_ptr(), out.data_ptr(), num_clusters,
           stamps.data_ptr() if stamps is not None else 0, smid.data_ptr() if smid is not None else 0,
           max_resident_clusters, s)
    return out
