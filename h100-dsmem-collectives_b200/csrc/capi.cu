// capi.cu -- implementation of include/dsmem_b200.h: registry lookup, legality, persistent launch.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "registry.h"

namespace {

using dsb::KernelEntry;
using dsb::Registry;

constexpr int kThreads = 256;

const char* const kOpNames[] = {"allreduce", "allgather", "reducescatter", "alltoall", "broadcast",
                                "reduce",    "gather",    "scatter"};
constexpr int kNumOps = 8;
const char* const kAlgNames[DSMEM_ALG_COUNT] = {"auto",
                                                "ring",
                                                "recursive_doubling",
                                                "shift_accumulate_bulk",
                                                "shift_accumulate_atomic",
                                                "direct_replicated_push",
                                                "pull_reduce_scatter_push_allgather",
                                                "rabenseifner",
                                                "one_shot_pull",
                                                "two_shot_push",
                                                "reduce_bcast_binomial",
                                                "atomic_all_push",
                                                "2d_mesh",
                                                "direct_shift",
                                                "bruck",
                                                "direct_pull",
                                                "gather_bcast_binomial",
                                                "recursive_halving",
                                                "direct_push",
                                                "pairwise_exchange",
                                                "pairwise_xor",
                                                "shift",
                                                "rs_push_global_ag",
                                                "ring_credit",
                                                "recursive_doubling_credit",
                                                "binomial",
                                                "bruck_credit",
                                                "recursive_halving_credit",
                                                "rabenseifner_credit",
                                                "pairwise_xor_credit",
                                                "binomial_credit",
                                                "shift_accumulate_bulk_credit"};
const char* const kDtypeNames[] = {"f32", "bf16", "i32"};

// (op, alg) -> reference file stem collectives/<op>__<alg>__<src>.cu
struct Stem {
    int op, alg;
    const char* stem;
};
const Stem kStems[] = {
    {0, DSMEM_ALG_RECURSIVE_DOUBLING, "allreduce__recursive_doubling__clusterfusion"},
    {0, DSMEM_ALG_SHIFT_ACCUMULATE_BULK, "allreduce__shift_accumulate_bulk__clusterfusion"},
    {0, DSMEM_ALG_SHIFT_ACCUMULATE_ATOMIC, "allreduce__shift_accumulate_atomic__clusterfusion"},
    {0, DSMEM_ALG_DIRECT_REPLICATED_PUSH, "allreduce__direct_replicated_push__credit"},
    {0, DSMEM_ALG_PULL_REDUCE_SCATTER_PUSH_ALLGATHER, "allreduce__pull_reduce_scatter_push_allgather__hpcops"},
    {0, DSMEM_ALG_RING, "allreduce__ring__nccl"},
    {0, DSMEM_ALG_RABENSEIFNER, "allreduce__rabenseifner__mpich"},
    {0, DSMEM_ALG_ONE_SHOT_PULL, "allreduce__one_shot_pull__trtllm"},
    {0, DSMEM_ALG_TWO_SHOT_PUSH, "allreduce__two_shot_push__trtllm"},
    {0, DSMEM_ALG_REDUCE_BCAST_BINOMIAL, "allreduce__reduce_bcast_binomial__mpich"},
    {0, DSMEM_ALG_ATOMIC_ALL_PUSH, "allreduce__atomic_all_push__generic"},
    {0, DSMEM_ALG_2D_MESH, "allreduce__2d_mesh__generic"},
    {1, DSMEM_ALG_RECURSIVE_DOUBLING, "allgather__recursive_doubling__clusterfusion"},
    {1, DSMEM_ALG_DIRECT_SHIFT, "allgather__direct_shift__clusterfusion"},
    {1, DSMEM_ALG_DIRECT_REPLICATED_PUSH, "allgather__direct_replicated_push__credit"},
    {1, DSMEM_ALG_RING, "allgather__ring__nccl"},
    {1, DSMEM_ALG_BRUCK, "allgather__bruck__mpich"},
    {1, DSMEM_ALG_DIRECT_PULL, "allgather__direct_pull__generic"},
    {1, DSMEM_ALG_GATHER_BCAST_BINOMIAL, "allgather__gather_bcast_binomial__mpich"},
    {2, DSMEM_ALG_RING, "reducescatter__ring__nccl"},
    {2, DSMEM_ALG_RECURSIVE_HALVING, "reducescatter__recursive_halving__mpich"},
    {2, DSMEM_ALG_DIRECT_PUSH, "reducescatter__direct_push__generic"},
    {2, DSMEM_ALG_DIRECT_PULL, "reducescatter__direct_pull__generic"},
    {3, DSMEM_ALG_PAIRWISE_EXCHANGE, "alltoall__pairwise_exchange__fa4"},
    {3, DSMEM_ALG_DIRECT_PUSH, "alltoall__direct_push__generic"},
    {3, DSMEM_ALG_PAIRWISE_XOR, "alltoall__pairwise_xor__mpich"},
    {3, DSMEM_ALG_SHIFT, "alltoall__shift__generic"},
    {3, DSMEM_ALG_BRUCK, "alltoall__bruck__mpich"},
    {3, DSMEM_ALG_DIRECT_PULL, "alltoall__direct_pull__generic"},
};

// Built-in AUTO order per op when no measured table entry applies: first legal candidate wins.
const std::vector<int> kDefaultOrder[kNumOps] = {
    {DSMEM_ALG_TWO_SHOT_PUSH, DSMEM_ALG_ONE_SHOT_PULL, DSMEM_ALG_RABENSEIFNER, DSMEM_ALG_RING,
     DSMEM_ALG_RECURSIVE_DOUBLING, DSMEM_ALG_PULL_REDUCE_SCATTER_PUSH_ALLGATHER},
    {DSMEM_ALG_DIRECT_PULL, DSMEM_ALG_DIRECT_REPLICATED_PUSH, DSMEM_ALG_BRUCK, DSMEM_ALG_RING},
    {DSMEM_ALG_DIRECT_PUSH, DSMEM_ALG_DIRECT_PULL, DSMEM_ALG_RECURSIVE_HALVING, DSMEM_ALG_RING},
    {DSMEM_ALG_DIRECT_PUSH, DSMEM_ALG_DIRECT_PULL, DSMEM_ALG_SHIFT, DSMEM_ALG_PAIRWISE_XOR},
    {DSMEM_ALG_DIRECT_PUSH, DSMEM_ALG_BINOMIAL, DSMEM_ALG_DIRECT_PULL},
    {DSMEM_ALG_DIRECT_PULL, DSMEM_ALG_BINOMIAL, DSMEM_ALG_DIRECT_PUSH},   // reduce: the root's loads feed its sum
    {DSMEM_ALG_DIRECT_PUSH, DSMEM_ALG_DIRECT_PULL, DSMEM_ALG_BINOMIAL},   // gather
    {DSMEM_ALG_DIRECT_PULL, DSMEM_ALG_DIRECT_PUSH, DSMEM_ALG_BINOMIAL},   // scatter
};

constexpr size_t kErrWords = 4;

struct DeviceState {
    unsigned* err = nullptr;                       // device error words (kErrWords)
    std::map<const void*, int> smem_attr;          // largest MaxDynamicSharedMemorySize set per kernel
    std::map<std::pair<const void*, uint64_t>, int> occupancy;
    int optin = 0;
    int sms = 0;
};

// AUTO table key. regime 0 = one cluster per launch (picked by latency), 1 = batches (by throughput).
struct TuneKey {
    int op, n, dtype, regime;
    bool operator<(const TuneKey& o) const {
        return std::tie(op, n, dtype, regime) < std::tie(o.op, o.n, o.dtype, o.regime);
    }
};

struct State {
    std::once_flag once;
    Registry reg;
    std::mutex mu;
    std::map<int, DeviceState> dev;
    std::map<TuneKey, std::map<uint64_t, int>> tune;   // (op, N, dtype, regime) -> {bytes -> alg}
    std::once_flag default_table_once;                  // the measured table shipped beside the library
    unsigned long long wait_limit_ns = 1000000000ull;
    bool pipelined = true;        // batches use a pipelined driver where one exists
    uint64_t unit_bytes = 16384;  // pipelined drivers: largest sub-vector per CTA
    // Streamed drivers (measured on B200 at 64 KiB per CTA, 2 GiB batches): 16 KiB units, one slot stage (one
    // unit of reduce-scatter in flight), input stages by cluster size (kStreamDepth).
    uint64_t stream_unit_bytes = 16384;  // largest sub-vector per CTA
    int stream_depth = 0;                // input stages; 0: kStreamDepth
    int stream_lag = 1;                  // slot stages: units of reduce-scatter in flight
    bool stream_set = false;             // dsmem_set_stream_pipeline was called: no launch-size defaults
};

State& st() {
    static State* s = new State();   // never destroyed: kernels may be launched from exit handlers
    return *s;
}

const Registry& registry() {
    State& s = st();
    std::call_once(s.once, [&] {
        dsb::register_op0_dt0(s.reg);
        dsb::register_op0_dt1(s.reg);
        dsb::register_op0_dt2(s.reg);
        dsb::register_op1_dt0(s.reg);
        dsb::register_op1_dt1(s.reg);
        dsb::register_op1_dt2(s.reg);
        dsb::register_op2_dt0(s.reg);
        dsb::register_op2_dt1(s.reg);
        dsb::register_op2_dt2(s.reg);
        dsb::register_op3_dt0(s.reg);
        dsb::register_op3_dt1(s.reg);
        dsb::register_op3_dt2(s.reg);
        dsb::register_op4_dt0(s.reg);
        dsb::register_op4_dt1(s.reg);
        dsb::register_op4_dt2(s.reg);
        dsb::register_op5_dt0(s.reg);
        dsb::register_op5_dt1(s.reg);
        dsb::register_op5_dt2(s.reg);
        dsb::register_op6_dt0(s.reg);
        dsb::register_op6_dt1(s.reg);
        dsb::register_op6_dt2(s.reg);
        dsb::register_op7_dt0(s.reg);
        dsb::register_op7_dt1(s.reg);
        dsb::register_op7_dt2(s.reg);
    });
    return s.reg;
}

const KernelEntry* find(int op, int alg, int dtype, int n) {
    for (const KernelEntry& e : registry())
        if (e.op == op && e.alg == alg && e.dtype == dtype && e.n == n) return &e;
    return nullptr;
}

int elem_bytes(int dtype) { return dtype == DSMEM_BF16 ? 2 : 4; }

// Elements per rank block from the payload convention; 0 if P does not divide.
uint32_t msg_elems(int op, int dtype, int n, size_t bytes) {
    const size_t unit = (size_t)elem_bytes(dtype) *
                        (op == DSMEM_OP_ALLREDUCE || op == DSMEM_OP_BROADCAST || op == DSMEM_OP_REDUCE ? 1 : (size_t)n);
    if (bytes == 0 || bytes % unit != 0) return 0;
    const size_t m = bytes / unit;
    return m > 0xffffffffull ? 0u : (uint32_t)m;
}

bool valid_enums(int op, int alg, int dtype, int n) {
    return op >= 0 && op < kNumOps && alg >= 0 && alg < DSMEM_ALG_COUNT && dtype >= 0 && dtype <= 2 &&
           (n == 2 || n == 4 || n == 8 || n == 16);
}

// Legality of a concrete algorithm: 0 ok, else a dsmem_status.
dsmem_status classify(const KernelEntry* e, uint32_t m, uint64_t* smem) {
    if (e == nullptr || m == 0 || !e->legal(m)) return DSMEM_ERR_ILLEGAL_CONFIG;
    const uint64_t s = e->smem_bytes(m);
    if (smem) *smem = s;
    if (s > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    return DSMEM_OK;
}

// One line per entry: "op cluster_size bytes_per_cta dtype alg [single|batch]" ('#' comments).
dsmem_status parse_table(const char* path, std::map<TuneKey, std::map<uint64_t, int>>& table) {
    std::ifstream f(path);
    if (!f) return DSMEM_ERR_INVALID_ARGUMENT;
    std::string line;
    while (std::getline(f, line)) {
        if (line.empty() || line[0] == '#') continue;
        std::istringstream is(line);
        std::string ops, dts, algs, regs;
        int n = 0;
        unsigned long long bytes = 0;
        if (!(is >> ops >> n >> bytes >> dts >> algs)) return DSMEM_ERR_INVALID_ARGUMENT;
        int regime = 0;
        if (is >> regs) {
            if (regs == "batch") regime = 1;
            else if (regs != "single") return DSMEM_ERR_INVALID_ARGUMENT;
        }
        int op = -1, dt = -1, alg = -1;
        for (int i = 0; i < kNumOps; ++i)
            if (ops == kOpNames[i]) op = i;
        for (int i = 0; i < 3; ++i)
            if (dts == kDtypeNames[i]) dt = i;
        for (int i = 1; i < DSMEM_ALG_COUNT; ++i)
            if (algs == kAlgNames[i]) alg = i;
        if (op < 0 || dt < 0 || alg < 0 || !valid_enums(op, alg, dt, n)) return DSMEM_ERR_INVALID_ARGUMENT;
        if (find(op, alg, dt, n) == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
        table[TuneKey{op, n, dt, regime}][bytes] = alg;
    }
    return DSMEM_OK;
}

// The measured table shipped with the library (<package>/autotune_b200.tsv, found next to lib/), loaded
// once on the first AUTO resolution; the environment variable DSMEM_AUTOTUNE_TABLE names another file
// (empty: none). A missing or malformed file leaves the built-in order.
void load_default_table() {
    std::call_once(st().default_table_once, [] {
        std::string path;
        if (const char* env = std::getenv("DSMEM_AUTOTUNE_TABLE")) {
            path = env;
        } else {
            Dl_info info{};
            if (dladdr(reinterpret_cast<void*>(&dsmem_version), &info) == 0 || info.dli_fname == nullptr) return;
            std::string lib = info.dli_fname;
            const size_t a = lib.rfind('/');
            if (a == std::string::npos) return;
            const std::string libdir = lib.substr(0, a);
            const size_t b = libdir.rfind('/');
            path = (b == std::string::npos ? std::string(".") : libdir.substr(0, b)) + "/autotune_b200.tsv";
        }
        if (path.empty()) return;
        std::map<TuneKey, std::map<uint64_t, int>> table;
        if (parse_table(path.c_str(), table) != DSMEM_OK) return;
        std::lock_guard<std::mutex> lock(st().mu);
        st().tune.swap(table);
    });
}

uint32_t pipeline_units(const KernelEntry* e, uint32_t m, uint64_t unit_bytes = 0);

// classify() OK, or a payload above the one-piece limit that the pipelined driver runs in fitting units.
// Caller holds st().mu.
bool launchable(const KernelEntry* e, uint32_t m) {
    const dsmem_status s = classify(e, m, nullptr);
    if (s == DSMEM_OK) return true;
    if (s != DSMEM_ERR_SMEM_LIMIT || e->fn_pipe == nullptr || !st().pipelined) return false;
    const uint32_t sub = pipeline_units(e, m);
    return sub != 0 && e->smem_pipe(m / sub) <= dsb::kSmemLimit;
}

int resolve_auto(int op, int dtype, int n, size_t bytes, int regime = 0) {
    load_default_table();
    State& s = st();
    const uint32_t m = msg_elems(op, dtype, n, bytes);
    {
        std::lock_guard<std::mutex> g(s.mu);
        // the measured table of this regime, then of the other one: the entry of the largest measured
        // payload <= bytes whose algorithm is legal here
        for (int r : {regime, 1 - regime}) {
            auto it = s.tune.find(TuneKey{op, n, dtype, r});
            if (it == s.tune.end() || it->second.empty()) continue;
            auto jt = it->second.upper_bound((uint64_t)bytes);
            if (jt != it->second.begin()) {
                --jt;
                const KernelEntry* e = find(op, jt->second, dtype, n);
                if (e != nullptr && launchable(e, m)) return jt->second;
            }
        }
    }
    for (int alg : kDefaultOrder[op]) {
        const KernelEntry* e = find(op, alg, dtype, n);
        if (classify(e, m, nullptr) == DSMEM_OK) return alg;
    }
    for (const KernelEntry& e : registry())
        if (e.op == op && e.dtype == dtype && e.n == n && classify(&e, m, nullptr) == DSMEM_OK) return e.alg;
    return DSMEM_ALG_AUTO;
}

DeviceState& device_state(int dev) {
    // caller holds st().mu
    DeviceState& d = st().dev[dev];
    if (d.optin == 0) cudaDeviceGetAttribute(&d.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (d.sms == 0) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    return d;
}

cudaError_t ensure_attrs(DeviceState& d, const void* fn, int n, uint64_t smem) {
    auto it = d.smem_attr.find(fn);
    if (it == d.smem_attr.end() || (uint64_t)it->second < smem) {
        cudaError_t r;
        if (n > 8) {
            r = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (r != cudaSuccess) return r;
        }
        const int want = (int)std::max<uint64_t>(smem, it == d.smem_attr.end() ? 0 : (uint64_t)it->second);
        r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
        if (r != cudaSuccess) return r;
        // the whole unified L1/shared array as shared memory, so several CTAs fit per SM
        r = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (r != cudaSuccess) return r;
        d.smem_attr[fn] = want;
    }
    return cudaSuccess;
}

void fill_cfg(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, int n, long long clusters, uint64_t smem,
              cudaStream_t stream, int threads = kThreads) {
    cfg = cudaLaunchConfig_t{};
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
}

cudaError_t occupancy(DeviceState& d, const void* fn, int n_cta, uint64_t smem, int* out, int threads = kThreads) {
    auto key = std::make_pair(fn, smem);
    auto it = d.occupancy.find(key);
    if (it != d.occupancy.end()) {
        *out = it->second;
        return cudaSuccess;
    }
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    fill_cfg(cfg, attr, n_cta, 1, smem, nullptr, threads);
    int n = 0;
    cudaError_t r = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
    if (r != cudaSuccess) return r;
    d.occupancy[key] = n;
    *out = n;
    return cudaSuccess;
}

cudaError_t error_word(DeviceState& d, unsigned** out) {
    if (d.err == nullptr) {   // [error bits, first timeout detail, its cluster id, spare] + a snapshot of them
        cudaError_t r = cudaMalloc(reinterpret_cast<void**>(&d.err), 2 * kErrWords * sizeof(unsigned));
        if (r != cudaSuccess) return r;
        r = cudaMemset(d.err, 0, 2 * kErrWords * sizeof(unsigned));
        if (r != cudaSuccess) return r;
    }
    *out = d.err;
    return cudaSuccess;
}

// Input stages of the streamed drivers' ring by op and cluster size (batch launches with one slot stage),
// measured on B200 at 16-192 KiB per CTA, 1-2 GiB batches. AllReduce: 3 at N = 8 (f32 0.733 ms against 0.758
// with 2), else 2 (N = 16: 0.970 ms against 1.088 with 3; the smaller window fits more clusters). The other
// ops (their slot stages are N - 1 whole pieces): 3 at N = 4, and for AlltoAll at N = 8 too; else 2.
uint32_t kStreamDepth(int op, int n) {
    if (op == DSMEM_OP_ALLREDUCE) return n == 8 ? 3u : 2u;
    if (n <= 4 || (op == DSMEM_OP_ALLTOALL && n == 8)) return 3u;
    return 2u;
}

// Units per problem for a pipelined driver: the smallest split into legal sub-vectors of at most
// unit_bytes per CTA (default 16 KiB: three unit buffers in 48 KiB, four CTAs per SM) whose smallest window
// fits the shared-memory limit; 0 if none.
// Caller holds st().mu.
uint32_t pipeline_units(const KernelEntry* e, uint32_t m, uint64_t unit_bytes) {
    const uint64_t unit = unit_bytes != 0 ? unit_bytes : e->stage_pipe != nullptr ? st().stream_unit_bytes : st().unit_bytes;
    // the input of one unit: m elements of the rank block (N pieces of them for the streamed ReduceScatter and
    // AlltoAll)
    const uint64_t bytes = e->in_stage_pipe != nullptr ? e->in_stage_pipe(m) : (uint64_t)m * e->elem_bytes;
    const uint32_t s0 = (uint32_t)std::max<uint64_t>(1, (bytes + unit - 1) / unit);
    for (uint32_t s = s0; s <= m && s < s0 + 4096; ++s)
        if (m % s == 0 && e->legal(m / s) && e->smem_pipe(m / s) <= dsb::kSmemLimit) return s;
    return 0;
}

// Legality of a launch. A payload whose one-piece buffers exceed the shared-memory limit (the reference's
// SKIP:smem) still runs when the algorithm has a pipelined driver whose sub-vector units fit: *pipe_only is
// then set and the launch must take that driver (dsmem_query keeps the reference's classification).
dsmem_status prepare(int op, int alg, int dtype, int n, size_t bytes, const KernelEntry** entry, uint32_t* m_out,
                     uint64_t* smem_out, int regime = 0, bool* pipe_only = nullptr) {
    if (!valid_enums(op, alg, dtype, n)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (alg == DSMEM_ALG_AUTO) alg = resolve_auto(op, dtype, n, bytes, regime);
    if (alg == DSMEM_ALG_AUTO) return DSMEM_ERR_ILLEGAL_CONFIG;
    const KernelEntry* e = find(op, alg, dtype, n);
    const uint32_t m = msg_elems(op, dtype, n, bytes);
    uint64_t smem = 0;
    dsmem_status s = classify(e, m, &smem);
    if (pipe_only) *pipe_only = false;
    if (s == DSMEM_ERR_SMEM_LIMIT && pipe_only != nullptr && e->fn_pipe != nullptr) {
        std::lock_guard<std::mutex> lock(st().mu);
        const uint32_t sub = st().pipelined ? pipeline_units(e, m) : 0u;
        if (sub && e->smem_pipe(m / sub) <= dsb::kSmemLimit) {
            *pipe_only = true;
            s = DSMEM_OK;
        }
    }
    if (s != DSMEM_OK) return s;
    *entry = e;
    *m_out = m;
    *smem_out = smem;
    return DSMEM_OK;
}

// A 2-CTA cluster whose single mbarrier expects 16 bytes nobody sends: the bounded waits give up after
// `limit` ns and set the timeout bit; the cluster-barrier sequence stays uniform, so the kernel ends.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64) selftest_timeout_kernel(unsigned* err,
                                                                                          unsigned long long limit) {
    __shared__ __align__(8) unsigned long long bar;
    dsb::Ctx c;
    dsb::ctx_init(c, 0, err, limit);
    c.sa = dsmem::smem_u32(&bar);
    if (threadIdx.x == 0) {
        dsmem::mbar_init(c.sa, 1);
        dsmem::fence_mbar_init();
    }
    dsmem::cluster_sync();
    c.deadline = dsmem::globaltimer() + limit;
    if (threadIdx.x == 0) dsmem::mbar_arrive_expect_tx(c.sa, 16);
    dsb::wait(c, 0);
    dsmem::cluster_sync();
}

// Read and clear the error words in one atomic step each: a bit a kernel sets while the check runs is either in
// this snapshot or stays in the word for the next check, never lost between a read and a clear.
__global__ void take_error_words(unsigned* err) {
    if (threadIdx.x < kErrWords) err[kErrWords + threadIdx.x] = atomicExch(err + threadIdx.x, 0u);
}

}  // namespace

extern "C" {

dsmem_status dsmem_selftest_timeout(unsigned long long limit_ns, dsmem_stream_t stream) {
    if (limit_ns == 0 || limit_ns > 10000000000ull) return DSMEM_ERR_INVALID_ARGUMENT;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DSMEM_ERR_CUDA;
    unsigned* err = nullptr;
    {
        std::lock_guard<std::mutex> lock(st().mu);
        if (error_word(device_state(dev), &err) != cudaSuccess) return DSMEM_ERR_CUDA;
    }
    selftest_timeout_kernel<<<2, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(err, limit_ns);
    return cudaGetLastError() == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

dsmem_status dsmem_collective_launch_ex(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                        size_t bytes_per_cta, const void* in, void* out, long long num_clusters,
                                        unsigned long long* stamps, unsigned* smid, int max_resident_clusters,
                                        dsmem_stream_t stream) {
    const KernelEntry* e = nullptr;
    uint32_t m = 0;
    uint64_t smem = 0;
    bool pipe_only = false;
    dsmem_status s = prepare(op, alg, dtype, cluster_size, bytes_per_cta, &e, &m, &smem, num_clusters > 1 ? 1 : 0,
                             &pipe_only);
    if (s != DSMEM_OK) return s;
    if (num_clusters < 0 || in == nullptr || out == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) return DSMEM_ERR_INVALID_ARGUMENT;
    if (num_clusters == 0) return DSMEM_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DSMEM_ERR_CUDA;
    dsb::BatchArgs a{};
    int resident = 0;
    int threads = kThreads;
    const void* fn = e->fn;
    {
        State& g = st();
        std::lock_guard<std::mutex> lock(g.mu);
        DeviceState& d = device_state(dev);
        if (!pipe_only && smem > (uint64_t)d.optin) return DSMEM_ERR_SMEM_LIMIT;
        // batches use the pipelined driver when the algorithm has one and its shared memory fits (and so
        // does any payload too large for the one-piece kernel)
        a.sub = 1;
        // Streamed driver, launches of at most one wave (one CTA per SM covers them): 32 KiB units, four input
        // stages and three units of reduce-scatter in flight about halve a lone problem's time against the batch
        // defaults (measured at 128 and 192 KiB per CTA, N = 8 and 16).
        const bool small = e->stage_pipe != nullptr && !g.stream_set && num_clusters * e->n <= d.sms;
        if (g.pipelined && (num_clusters > 1 || pipe_only) && e->fn_pipe != nullptr) {
            const uint32_t sub = pipeline_units(e, m, small ? 32768 : 0);
            uint64_t sp = sub ? e->smem_pipe(m / sub) : 0;
            if (sub && sp <= dsb::kSmemLimit && sp <= (uint64_t)d.optin) {
                fn = e->fn_pipe;
                a.sub = sub;
                if (e->stage_pipe != nullptr) {
                    // streamed: an input ring of `depth` stages and a slot ring of `lag` stages (units in the
                    // reduce-scatter), as many as asked for and fit; depth > lag >= 1
                    const uint32_t u = m / sub;
                    const uint64_t in = e->in_stage_pipe(u), slot = e->stage_pipe(u) - in;
                    const uint64_t lim = std::min<uint64_t>(dsb::kSmemLimit, d.optin);
                    uint32_t dr = small ? 3u : (uint32_t)std::max(1, g.stream_lag);
                    uint32_t dx = g.stream_depth > 0 ? (uint32_t)g.stream_depth : (small ? 4u : kStreamDepth(e->op, e->n));
                    dx = std::max(dx, dr + 1);
                    auto window = [&] { return dsb::kD0 + dx * in + dr * slot; };
                    while (window() > lim && dx > dr + 1) --dx;
                    while (window() > lim && dr > 1) dx = std::max(--dr + 1, dx - 1);
                    sp = window();
                    a.depth = dx;
                    a.lag = dr;
                    threads = e->threads_pipe;
                }
                smem = sp;
            }
        }
        if (fn == e->fn && pipe_only) return DSMEM_ERR_SMEM_LIMIT;
        if (ensure_attrs(d, fn, e->n, smem) != cudaSuccess) return DSMEM_ERR_CUDA;
        if (occupancy(d, fn, e->n, smem, &resident, threads) != cudaSuccess) return DSMEM_ERR_CUDA;
        if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;   // the cluster cannot be placed (main.cu:221)
        if (error_word(d, &a.err) != cudaSuccess) return DSMEM_ERR_CUDA;
        a.wait_limit_ns = g.wait_limit_ns;
    }
    long long clusters = std::min<long long>(num_clusters, resident);
    if (max_resident_clusters > 0) clusters = std::min<long long>(clusters, max_resident_clusters);
    a.in = in;
    a.out = out;
    a.num_problems = num_clusters;
    a.stamps = stamps;
    a.smid = smid;
    a.M = m;
    a.smem_bytes = (uint32_t)smem;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    fill_cfg(cfg, attr, e->n, clusters, smem, reinterpret_cast<cudaStream_t>(stream), threads);
    void* args[] = {&a};
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return DSMEM_ERR_CUDA;
    return DSMEM_OK;
}

dsmem_status dsmem_collective_launch(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                     size_t bytes_per_cta, const void* in, void* out, int num_clusters,
                                     unsigned long long* stamps, dsmem_stream_t stream) {
    return dsmem_collective_launch_ex(op, alg, dtype, cluster_size, bytes_per_cta, in, out, num_clusters, stamps,
                                      nullptr, 0, stream);
}

dsmem_status dsmem_query(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta,
                         size_t* smem_bytes, int* legal) {
    if (!valid_enums(op, alg, dtype, cluster_size)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (alg == DSMEM_ALG_AUTO) alg = (dsmem_alg)resolve_auto(op, dtype, cluster_size, bytes_per_cta);
    const KernelEntry* e = alg == DSMEM_ALG_AUTO ? nullptr : find(op, alg, dtype, cluster_size);
    const uint32_t m = msg_elems(op, dtype, cluster_size, bytes_per_cta);
    uint64_t smem = 0;
    if (e != nullptr && m != 0 && e->legal(m)) smem = e->smem_bytes(m);
    const dsmem_status s = classify(e, m, nullptr);
    if (smem_bytes) *smem_bytes = (size_t)smem;
    if (legal) *legal = s == DSMEM_OK;
    return s;
}

dsmem_status dsmem_max_active_clusters(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                       size_t bytes_per_cta, int* clusters) {
    const KernelEntry* e = nullptr;
    uint32_t m = 0;
    uint64_t smem = 0;
    dsmem_status s = prepare(op, alg, dtype, cluster_size, bytes_per_cta, &e, &m, &smem);
    if (s != DSMEM_OK) return s;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DSMEM_ERR_CUDA;
    std::lock_guard<std::mutex> lock(st().mu);
    DeviceState& d = device_state(dev);
    if (smem > (uint64_t)d.optin) return DSMEM_ERR_SMEM_LIMIT;
    if (ensure_attrs(d, e->fn, e->n, smem) != cudaSuccess) return DSMEM_ERR_CUDA;
    int n = 0;
    if (occupancy(d, e->fn, e->n, smem, &n) != cudaSuccess) return DSMEM_ERR_CUDA;
    if (clusters) *clusters = n;
    return DSMEM_OK;
}

dsmem_status dsmem_autotune_table_load(const char* path) {
    if (path == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    std::call_once(st().default_table_once, [] {});   // an explicit table replaces the default one for good
    std::map<TuneKey, std::map<uint64_t, int>> table;
    const dsmem_status s = parse_table(path, table);
    if (s != DSMEM_OK) return s;
    std::lock_guard<std::mutex> lock(st().mu);
    st().tune.swap(table);
    return DSMEM_OK;
}

dsmem_alg dsmem_autotune_pick(dsmem_op op, dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta) {
    if (!valid_enums(op, 0, dtype, cluster_size)) return DSMEM_ALG_AUTO;
    return (dsmem_alg)resolve_auto(op, dtype, cluster_size, bytes_per_cta);
}

dsmem_alg dsmem_autotune_pick_ex(dsmem_op op, dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta,
                                 long long num_clusters) {
    if (!valid_enums(op, 0, dtype, cluster_size)) return DSMEM_ALG_AUTO;
    return (dsmem_alg)resolve_auto(op, dtype, cluster_size, bytes_per_cta, num_clusters > 1 ? 1 : 0);
}

dsmem_status dsmem_last_error_detail(int device, unsigned* error_bits, unsigned* detail, unsigned* cluster) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return DSMEM_ERR_CUDA;
    unsigned* w = nullptr;
    {
        std::lock_guard<std::mutex> lock(st().mu);
        auto it = st().dev.find(device);
        if (it != st().dev.end()) w = it->second.err;
    }
    unsigned v[kErrWords] = {};
    if (w != nullptr) {
        if (device != prev && cudaSetDevice(device) != cudaSuccess) return DSMEM_ERR_CUDA;
        cudaError_t r = cudaDeviceSynchronize();
        if (r == cudaSuccess) {
            take_error_words<<<1, 32>>>(w);
            r = cudaGetLastError();
        }
        if (r == cudaSuccess) r = cudaMemcpy(v, w + kErrWords, sizeof v, cudaMemcpyDeviceToHost);
        if (device != prev) cudaSetDevice(prev);
        if (r != cudaSuccess) return DSMEM_ERR_CUDA;
    }
    if (error_bits) *error_bits = v[0];
    if (detail) *detail = v[1];
    if (cluster) *cluster = v[2];
    return DSMEM_OK;
}

dsmem_status dsmem_last_error(int device, unsigned* error_bits) {
    return dsmem_last_error_detail(device, error_bits, nullptr, nullptr);
}

dsmem_status dsmem_check(dsmem_stream_t stream) {
    if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return DSMEM_ERR_CUDA;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DSMEM_ERR_CUDA;
    unsigned bits = 0;
    const dsmem_status s = dsmem_last_error(dev, &bits);
    if (s != DSMEM_OK) return s;
    if (bits & DSMEM_ERRBIT_TIMEOUT) return DSMEM_ERR_TIMEOUT;
    if (bits & DSMEM_ERRBIT_BOUNDS) return DSMEM_ERR_BOUNDS;
    return DSMEM_OK;
}

const char* dsmem_op_name(dsmem_op op) { return (op >= 0 && op < kNumOps) ? kOpNames[op] : "?"; }
const char* dsmem_alg_name(dsmem_alg alg) { return (alg >= 0 && alg < DSMEM_ALG_COUNT) ? kAlgNames[alg] : "?"; }
const char* dsmem_dtype_name(dsmem_dtype dt) { return (dt >= 0 && dt <= 2) ? kDtypeNames[dt] : "?"; }

const char* dsmem_status_string(dsmem_status s) {
    switch (s) {
        case DSMEM_OK: return "ok";
        case DSMEM_ERR_ILLEGAL_CONFIG: return "illegal configuration (reference SKIP:static_assert)";
        case DSMEM_ERR_SMEM_LIMIT: return "shared memory above the per-CTA limit (reference SKIP:smem)";
        case DSMEM_ERR_TIMEOUT: return "device-side mbarrier wait timed out";
        case DSMEM_ERR_CUDA: return "CUDA error";
        case DSMEM_ERR_INVALID_ARGUMENT: return "invalid argument";
        case DSMEM_ERR_BOUNDS: return "device-side bounds check failed";
        case DSMEM_ERR_NCCL: return "NCCL error";
        case DSMEM_ERR_SCRATCH_LIMIT: return "batch larger than the static scratch of the no-alloc entry point";
    }
    return "?";
}

const char* dsmem_file_stem(dsmem_op op, dsmem_alg alg) {
    for (const Stem& s : kStems)
        if (s.op == (int)op && s.alg == (int)alg) return s.stem;
    return nullptr;
}

dsmem_status dsmem_lookup(const char* file_stem, dsmem_op* op, dsmem_alg* alg) {
    if (file_stem == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    std::string f(file_stem);
    const size_t slash = f.find_last_of('/');
    if (slash != std::string::npos) f = f.substr(slash + 1);
    if (f.size() > 3 && f.compare(f.size() - 3, 3, ".cu") == 0) f.resize(f.size() - 3);
    for (const Stem& s : kStems)
        if (f == s.stem) {
            if (op) *op = (dsmem_op)s.op;
            if (alg) *alg = (dsmem_alg)s.alg;
            return DSMEM_OK;
        }
    return DSMEM_ERR_INVALID_ARGUMENT;
}

dsmem_status dsmem_set_wait_limit_ns(unsigned long long ns) {
    if (ns == 0) return DSMEM_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(st().mu);
    st().wait_limit_ns = ns;
    return DSMEM_OK;
}

dsmem_status dsmem_set_pipelined(int enable) {
    std::lock_guard<std::mutex> lock(st().mu);
    st().pipelined = enable != 0;
    return DSMEM_OK;
}

dsmem_status dsmem_set_pipeline_unit_bytes(size_t bytes) {
    if (bytes < 256 || bytes > 65536 || (bytes & 15u)) return DSMEM_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(st().mu);
    st().unit_bytes = bytes;
    return DSMEM_OK;
}

dsmem_status dsmem_set_stream_pipeline(size_t unit_bytes, int depth, int lag) {
    if (unit_bytes == 0 && depth == 0 && lag == 0) {   // back to the measured defaults
        std::lock_guard<std::mutex> lock(st().mu);
        st().stream_unit_bytes = 16384;
        st().stream_depth = 0;
        st().stream_lag = 1;
        st().stream_set = false;
        return DSMEM_OK;
    }
    if (unit_bytes < 256 || unit_bytes > 65536 || (unit_bytes & 15u) || (depth != 0 && (depth < 2 || depth > 8)) ||
        lag < 1 || lag >= (depth == 0 ? 2 : depth))
        return DSMEM_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(st().mu);
    st().stream_unit_bytes = unit_bytes;
    st().stream_depth = depth;
    st().stream_lag = lag;
    st().stream_set = true;
    return DSMEM_OK;
}

const char* dsmem_version(void) { return "dsmem_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
