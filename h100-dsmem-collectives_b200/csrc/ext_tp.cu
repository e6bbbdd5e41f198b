// ext_tp.cu -- tensor-parallel AllReduce + RMSNorm across the GPUs of one node, sm_100a.
//
// y = RMSNorm(sum over TP ranks of x_rank (+ residual)) * w on every rank, bf16 in/out, fp32 sum and
// statistics. Reference: kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197 (AllReduce
// then the cluster RMSNorm of the sum, h = x + residual) and the configs[4] pipeline (cross-GPU
// AllReduce feeding the cluster RMSNorm).
//
// B200 design: ONE kernel per rank over NVLink peer memory (one process per GPU, buffers exchanged by
// CUDA IPC). It fuses the collective with the normalisation:
//   * reduce-scatter by rows: rank r owns rows [r*T/TP, (r+1)*T/TP); its CTAs read the row slices of
//     every rank's x buffer with 16-byte peer loads (plain loads, no TMA and no multicast), sum them in
//     fp32 in rank order 0..TP-1 (so the result does not depend on which rank computes it), add the
//     residual, and round h to bf16;
//   * cluster RMSNorm of the owned rows: CTA b of a cluster of N owns column slice b; the per-row
//     partial sums of squares meet by the replicated st.async push of the single-GPU kernel
//     (rmsnorm_lamport...hpcops.cu:153-169), no cluster barrier per group;
//   * all-gather: the normalised rows are stored into the y buffer of every rank (peer stores), so each
//     row crosses NVLink once per destination, as in a ring-optimal AllReduce (2(TP-1)/TP of the tensor
//     per rank), with the RMSNorm fused between the two halves.
// Cross-GPU ordering: at entry CTA 0 writes the call's epoch (a per-rank device counter of completed
// calls, plus one; no host state, so the call can be captured in a CUDA graph) into every peer's start
// flag (release, system scope) and every CTA waits for all peers' start flags (their x is complete: it
// was written before their launch); at exit the last CTA of the grid (an atomic counter) publishes the epoch into
// every peer's end flag after all CTAs' peer stores, then waits for all peers' end flags, so when the
// kernel ends this rank's y is complete and no peer still reads its x. Every wait is bounded.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "f32x2.cuh"
#include "smem_attr.cuh"

namespace {

using namespace dsmem;
using namespace dsb2;

constexpr int kMaxTp = 8;
constexpr int kWarps = 8;
constexpr int kThreadsTp = kWarps * 32;
constexpr int kRowsPerWarp = 2;                 // one st.async.v2 of partials per warp and group
constexpr int kR = kWarps * kRowsPerWarp;       // rows per group
constexpr int kSets = 4;                        // partial-sum slot sets (2 are needed, see exec loop)
constexpr uint32_t kSlots = 128;                // slot sets start after the barrier area
constexpr size_t kSignalBytes = 4096;           // per-rank signal region at the start of its buffer
// signal words (u32): start flag per source rank at 0, end flag per source rank at 32, the grid's
// arrival counter at 64, the epoch of the last completed call at 65, error words at 96..99
constexpr int kSigStart = 0, kSigEnd = 32, kSigCounter = 64, kSigEpoch = 65, kSigErr = 96;

struct TpArgs {
    const uint4* x[kMaxTp];   // x buffer of every rank (this rank's own at [rank])
    uint4* y[kMaxTp];         // y buffer of every rank
    unsigned* sig[kMaxTp];    // signal region of every rank
    const uint4* res;         // this rank's residual (nullable)
    const uint4* w;
    unsigned* err;            // this rank's error words
    unsigned long long wait_limit_ns;
    long long rows;
    int hidden;
    float eps;
    uint32_t slice_bytes;
    uint32_t smem_bytes;
    int rank;
    int emulate;              // 1: one launch computes every row for TP local buffers, no flags
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Bounded wait for `*flag == epoch` (flag written by a peer GPU). Records a timeout with barrier id
// `id` and returns false when the deadline passes.
__device__ __forceinline__ bool wait_flag(dsb::Ctx& c, const unsigned* flag, unsigned epoch, int id) {
    const unsigned long long until = globaltimer() + c.wait_limit;
    while (ld_acquire_sys(flag) != epoch) {
        if (globaltimer() > until) {
            c.dead = true;
            dsb::report_timeout(c, id);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

template <int N, int TP, int UPL>
__global__ void __launch_bounds__(kThreadsTp, (UPL >= 4 ? 1 : 2)) tp_allreduce_rmsnorm_kernel(const TpArgs a) {
    constexpr int P = RmsElem<__nv_bfloat16>::kPairs;
    using E = RmsElem<__nv_bfloat16>;
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t units = a.slice_bytes >> 4;             // 16-B units of a row slice (<= 32 * UPL)
    const long long row_u4 = a.hidden / 8;                 // 16-B units per row
    const long long col_u4 = (long long)c.rank * units;    // first unit of my column slice
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSets; ++s) mbar_init(c.bar(s), 1);
        fence_mbar_init();
    }
    // ---- cross-GPU entry: every peer has launched, so its x (written before its launch) is complete.
    // The call's epoch is one past the last completed call's, kept in device memory (the last CTA of a
    // call stores it), so the kernel can sit in a CUDA graph: every rank makes the same sequence of calls.
    unsigned epoch = 0;
    if (!a.emulate) {
        epoch = ld_acquire_sys(a.sig[a.rank] + kSigEpoch) + 1u;
        if (blockIdx.x == 0 && threadIdx.x < TP && (int)threadIdx.x != a.rank) {
            fence_sys();
            st_release_sys(a.sig[threadIdx.x] + kSigStart + a.rank, epoch);
        }
        if (threadIdx.x < TP && (int)threadIdx.x != a.rank)
            wait_flag(c, a.sig[a.rank] + kSigStart + threadIdx.x, epoch, 0x70 + (int)threadIdx.x);
    }
    __syncthreads();
    cluster_sync();   // every CTA's slot barriers initialised before any remote store completes on them

    // rows of this rank (all rows when emulating), split evenly over the clusters
    const long long own_lo = a.emulate ? 0 : a.rank * a.rows / TP;
    const long long own_hi = a.emulate ? a.rows : (a.rank + 1) * a.rows / TP;
    const long long nclu = (long long)num_clusters(), cq = (long long)cluster_id();
    const long long lo = own_lo + cq * (own_hi - own_lo) / nclu, hi = own_lo + (cq + 1) * (own_hi - own_lo) / nclu;
    const long long iters = (hi - lo + kR - 1) / kR;
    const float inv_hidden = 1.0f / (float)a.hidden;

    constexpr bool kWReg = UPL <= 2;   // weight units as fp32 pairs in registers (8 per unit)
    f2x wr[kWReg ? UPL : 1][P];
    if constexpr (kWReg) {
#pragma unroll
        for (int q = 0; q < UPL; ++q) {
            const uint32_t u = lane + 32u * q;
            if (u < units) E::unpack(__ldg(a.w + col_u4 + u), wr[q]);
        }
    }

    for (long long i = 0; i < iters; ++i) {
        c.deadline = globaltimer() + c.wait_limit;
        const long long row0 = lo + i * kR + (long long)warp * kRowsPerWarp;
        uint4 h[kRowsPerWarp][UPL];
        float ss[kRowsPerWarp];
        bool ok[kRowsPerWarp][UPL];
        long long idx[kRowsPerWarp][UPL];
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
            for (int q = 0; q < UPL; ++q) {
                const uint32_t u = lane + 32u * q;
                ok[k][q] = row0 + k < hi && u < units;
                idx[k][q] = (row0 + k) * row_u4 + col_u4 + u;
            }
        // Sum over the ranks in rank order. The group's loads from PB ranks at a time are all issued before
        // any is used, so a lane keeps PB * 2 * UPL 16-byte peer loads in flight.
        constexpr int PB_MAX = UPL >= 4 ? 1 : (UPL == 2 ? 2 : 4);
        constexpr int PB = TP < PB_MAX ? TP : PB_MAX;   // a divisor of TP: ranks p0 + pp stay below TP
        static_assert(TP % PB == 0, "rank batches must tile the TP ranks");
        f2x acc[kRowsPerWarp][UPL][P];
#pragma unroll
        for (int p0 = 0; p0 < TP; p0 += PB) {
            uint4 v[PB][kRowsPerWarp][UPL];
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q)
                        v[pp][k][q] = ok[k][q] ? a.x[p0 + pp][idx[k][q]] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q) {
                        if (p0 + pp == 0) {
                            E::unpack(v[pp][k][q], acc[k][q]);
                        } else {
                            f2x t[P];
                            E::unpack(v[pp][k][q], t);
#pragma unroll
                            for (int e = 0; e < P; ++e) acc[k][q][e] = f2_add(acc[k][q][e], t[e]);
                        }
                    }
        }
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            f2x sacc = 0ull;
#pragma unroll
            for (int q = 0; q < UPL; ++q) {
                if (a.res != nullptr && ok[k][q]) {
                    f2x t[P];
                    E::unpack(a.res[idx[k][q]], t);
#pragma unroll
                    for (int e = 0; e < P; ++e) acc[k][q][e] = f2_add(acc[k][q][e], t[e]);
                }
                h[k][q] = E::pack(acc[k][q]);   // h rounded to bf16, as the unfused AllReduce would give it
                f2x hf[P];
                E::unpack(h[k][q], hf);
#pragma unroll
                for (int e = 0; e < P; ++e) sacc = f2_fma(hf[e], hf[e], sacc);   // zero where !ok
            }
            const float2 s2 = f2_split(sacc);
            ss[k] = s2.x + s2.y;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], off);
        }
        // replicated push of the warp's two partials into slot set i of every CTA of the cluster. The set
        // of group i is rewritten for group i+kSets; a writer sends group g only after it normalised g-1,
        // which needed the owner's partials of g-1, sent after the owner finished reading set g-2.
        const int set = (int)(i & (kSets - 1));
        if (threadIdx.x == 0) dsb::arm(c, set, (uint32_t)N * kR * 4u);
        if (lane < (uint32_t)N) {
            const uint32_t dst = kSlots + (((uint32_t)set * N + c.rank) * kR + warp * kRowsPerWarp) * 4u;
            const uint32_t rd = mapa(c.sa + dst, lane), rbar = mapa(c.bar(set), lane);
            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1,%2}, [%3];" ::"r"(rd),
                         "f"(ss[0]), "f"(ss[1]), "r"(rbar)
                         : "memory");
        }
        dsb::wait(c, set);
        float2 part = make_float2(0.f, 0.f);
        if (lane < (uint32_t)N)
            part = *c.ptr<const float2>(kSlots + (((uint32_t)set * N + lane) * kR + warp * kRowsPerWarp) * 4u);
#pragma unroll
        for (int off = N / 2; off > 0; off >>= 1) {
            part.x += __shfl_xor_sync(0xffffffffu, part.x, off);
            part.y += __shfl_xor_sync(0xffffffffu, part.y, off);
        }
        const float tot[kRowsPerWarp] = {__shfl_sync(0xffffffffu, part.x, 0), __shfl_sync(0xffffffffu, part.y, 0)};
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            const long long row = row0 + k;
            const float scale = rsqrtf(fmaf(tot[k], inv_hidden, a.eps));
            const f2x scale2 = f2_make(scale, scale);
            if (row >= hi) continue;
#pragma unroll
            for (int q = 0; q < UPL; ++q) {
                const uint32_t u = lane + 32u * q;
                if (u < units) {
                    f2x f[P];
                    E::unpack(h[k][q], f);
                    if constexpr (kWReg) {
#pragma unroll
                        for (int e = 0; e < P; ++e) f[e] = f2_mul(f2_mul(f[e], scale2), wr[q][e]);
                    } else {
                        f2x wv[P];
                        E::unpack(__ldg(a.w + col_u4 + u), wv);
#pragma unroll
                        for (int e = 0; e < P; ++e) f[e] = f2_mul(f2_mul(f[e], scale2), wv[e]);
                    }
                    const uint4 yv = E::pack(f);
#pragma unroll
                    for (int p = 0; p < TP; ++p) a.y[p][idx[k][q]] = yv;   // all-gather: every rank's y
                }
            }
        }
    }
    // ---- cross-GPU exit: the last CTA publishes after every CTA's peer stores, then waits for all peers
    if (!a.emulate) {
        __syncthreads();
        if (threadIdx.x == 0) {
            fence_sys();
            unsigned* counter = a.sig[a.rank] + kSigCounter;
            const unsigned prev = atomicAdd(counter, 1u);
            if (prev == gridDim.x - 1) {
                fence_sys();
                *counter = 0u;   // for the next call (stream-ordered after this kernel)
                for (int t = 0; t < TP; ++t)
                    if (t != a.rank) st_release_sys(a.sig[t] + kSigEnd + a.rank, epoch);
                for (int t = 0; t < TP; ++t)
                    if (t != a.rank) wait_flag(c, a.sig[a.rank] + kSigEnd + t, epoch, 0x78 + t);
                a.sig[a.rank][kSigEpoch] = epoch;   // read by the next call's CTAs (stream-ordered)
            }
        }
    }
    dsb::finish(c);
}

template <int N, int TP>
const void* tp_fn_upl(int upl) {
    switch (upl) {
        case 1: return reinterpret_cast<const void*>(&tp_allreduce_rmsnorm_kernel<N, TP, 1>);
        case 2: return reinterpret_cast<const void*>(&tp_allreduce_rmsnorm_kernel<N, TP, 2>);
        case 4: return reinterpret_cast<const void*>(&tp_allreduce_rmsnorm_kernel<N, TP, 4>);
    }
    return nullptr;
}
template <int N>
const void* tp_fn_tp(int tp, int upl) {
    switch (tp) {
        case 1: return tp_fn_upl<N, 1>(upl);
        case 2: return tp_fn_upl<N, 2>(upl);
        case 4: return tp_fn_upl<N, 4>(upl);
        case 8: return tp_fn_upl<N, 8>(upl);
    }
    return nullptr;
}
const void* tp_fn(int n, int tp, int upl) {
    switch (n) {
        case 2: return tp_fn_tp<2>(tp, upl);
        case 4: return tp_fn_tp<4>(tp, upl);
        case 8: return tp_fn_tp<8>(tp, upl);
        case 16: return tp_fn_tp<16>(tp, upl);
    }
    return nullptr;
}

uint32_t tp_smem() { return kSlots + (uint32_t)kSets * 16u * kR * 4u; }   // slots sized for N <= 16

std::mutex g_tp_mu;

// Shape checks and launch of the kernel for `tp` ranks (emulate: all buffers local, one launch).
dsmem_status tp_launch(const void* const* xs, void* const* ys, unsigned* const* sigs, unsigned* err, int tp,
                       int rank, int emulate, dsmem_dtype dtype, const void* residual,
                       const void* w, float eps, long long rows, int hidden, int cluster_size,
                       cudaStream_t stream, unsigned long long wait_limit_ns = 2000000000ull) {
    if (dtype != DSMEM_BF16) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (!(tp == 1 || tp == 2 || tp == 4 || tp == 8) || rank < 0 || rank >= tp) return DSMEM_ERR_INVALID_ARGUMENT;
    const int n = cluster_size;
    if (!(n == 2 || n == 4 || n == 8 || n == 16)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (w == nullptr || rows < 0 || hidden <= 0 || !(eps >= 0.f)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (hidden % (8 * n) != 0) return DSMEM_ERR_ILLEGAL_CONFIG;   // whole 16-B units per CTA slice
    const uint32_t slice = (uint32_t)(hidden / n) * 2u, units = slice / 16u;
    if (units > 128u) return DSMEM_ERR_ILLEGAL_CONFIG;            // <= 4 units per lane
    const int upl = units <= 32 ? 1 : units <= 64 ? 2 : 4;
    uintptr_t al = reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(residual);
    for (int p = 0; p < tp; ++p) {
        if (xs[p] == nullptr || ys[p] == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
        al |= reinterpret_cast<uintptr_t>(xs[p]) | reinterpret_cast<uintptr_t>(ys[p]);
    }
    if (al & 15u) return DSMEM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DSMEM_OK;
    const void* fn = tp_fn(n, tp, upl);
    if (fn == nullptr) return DSMEM_ERR_ILLEGAL_CONFIG;
    const uint32_t smem = tp_smem();
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreadsTp, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int resident = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DSMEM_ERR_CUDA;
    {
        // kernel attributes and the occupancy query once per (kernel, device): they cost more than a launch
        static std::map<std::tuple<const void*, int, uint32_t>, int> occupancy;
        std::lock_guard<std::mutex> lock(g_tp_mu);
        if (dsb_attr::ensure_smem(fn, dev, (uint32_t)smem, n > 8, false) != cudaSuccess) return DSMEM_ERR_CUDA;
        auto it = occupancy.find({fn, dev, (uint32_t)smem});
        if (it != occupancy.end()) {
            resident = it->second;
        } else {
            cfg.gridDim = dim3((unsigned)n, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&resident, fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
            occupancy[{fn, dev, (uint32_t)smem}] = resident;
        }
    }
    if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;
    // every CTA must be resident (the exit counter is passed by all of them); at least one cluster even
    // for a rank that owns no rows, so it still takes part in the flags
    const long long own = emulate ? rows : (rank + 1) * rows / tp - rank * rows / tp;
    const long long clusters = std::max<long long>(1, std::min<long long>((own + kR - 1) / kR, resident));
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    TpArgs a{};
    for (int p = 0; p < tp; ++p) {
        a.x[p] = static_cast<const uint4*>(xs[p]);
        a.y[p] = static_cast<uint4*>(ys[p]);
        a.sig[p] = sigs != nullptr ? sigs[p] : nullptr;
    }
    a.res = static_cast<const uint4*>(residual);
    a.w = static_cast<const uint4*>(w);
    a.err = err;
    a.wait_limit_ns = wait_limit_ns;
    a.rows = rows;
    a.hidden = hidden;
    a.eps = eps;
    a.slice_bytes = slice;
    a.smem_bytes = smem;
    a.rank = rank;
    a.emulate = emulate;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

}  // namespace

// ------------------------------------------------------------------------------------------ TP context
struct dsmem_tp_ctx {
    int device = 0;
    int rank = -1;
    int tp = 0;
    size_t capacity = 0;             // bytes of each of the x and y regions
    unsigned char* base = nullptr;   // this rank's buffer: [signals 4 KiB][x][y]
    unsigned char* peer[kMaxTp] = {};
    unsigned long long wait_limit_ns = 2000000000ull;   // each cross-GPU flag wait of a call
};

extern "C" {

dsmem_status dsmem_tp_alloc(size_t capacity_bytes, dsmem_tp_t* ctx, void* ipc_handle) {
    if (ctx == nullptr || ipc_handle == nullptr || capacity_bytes == 0) return DSMEM_ERR_INVALID_ARGUMENT;
    *ctx = nullptr;
    auto* c = new dsmem_tp_ctx();
    c->capacity = (capacity_bytes + 255) & ~(size_t)255;
    if (cudaGetDevice(&c->device) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&c->base), kSignalBytes + 2 * c->capacity) != cudaSuccess) {
        delete c;
        return DSMEM_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaMemset(c->base, 0, kSignalBytes) != cudaSuccess || cudaIpcGetMemHandle(&h, c->base) != cudaSuccess) {
        cudaFree(c->base);
        delete c;
        return DSMEM_ERR_CUDA;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == DSMEM_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle, &h, sizeof h);
    *ctx = c;
    return DSMEM_OK;
}

dsmem_status dsmem_tp_open(dsmem_tp_t c, int rank, int tp, const void* handles) {
    if (c == nullptr || handles == nullptr || !(tp == 1 || tp == 2 || tp == 4 || tp == 8) || rank < 0 || rank >= tp ||
        c->tp != 0)
        return DSMEM_ERR_INVALID_ARGUMENT;
    const auto* hs = static_cast<const unsigned char*>(handles);
    for (int p = 0; p < tp; ++p) {
        if (p == rank) {
            c->peer[p] = c->base;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + (size_t)p * DSMEM_TP_HANDLE_BYTES, sizeof h);
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            for (int q = 0; q < p; ++q)
                if (q != rank && c->peer[q] != nullptr) cudaIpcCloseMemHandle(c->peer[q]);
            return DSMEM_ERR_CUDA;
        }
        c->peer[p] = static_cast<unsigned char*>(ptr);
    }
    c->rank = rank;
    c->tp = tp;
    return DSMEM_OK;
}

dsmem_status dsmem_tp_buffers(dsmem_tp_t c, void** x, void** y, size_t* capacity_bytes) {
    if (c == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    if (x) *x = c->base + kSignalBytes;
    if (y) *y = c->base + kSignalBytes + c->capacity;
    if (capacity_bytes) *capacity_bytes = c->capacity;
    return DSMEM_OK;
}

dsmem_status dsmem_tp_allreduce_rmsnorm(dsmem_tp_t c, dsmem_dtype dtype, const void* x, const void* residual,
                                        const void* w, float eps, long long rows, int hidden, int cluster_size,
                                        void* y, dsmem_stream_t stream) {
    if (c == nullptr || c->tp == 0) return DSMEM_ERR_INVALID_ARGUMENT;
    const size_t bytes = (size_t)std::max<long long>(rows, 0) * (size_t)std::max(hidden, 0) * 2u;
    if (bytes > c->capacity) return DSMEM_ERR_SCRATCH_LIMIT;
    auto s = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* xb = c->base + kSignalBytes;
    unsigned char* yb = xb + c->capacity;
    if (x != nullptr && x != xb && bytes && cudaMemcpyAsync(xb, x, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    const void* xs[kMaxTp];
    void* ys[kMaxTp];
    unsigned* sigs[kMaxTp];
    for (int p = 0; p < c->tp; ++p) {
        xs[p] = c->peer[p] + kSignalBytes;
        ys[p] = c->peer[p] + kSignalBytes + c->capacity;
        sigs[p] = reinterpret_cast<unsigned*>(c->peer[p]);
    }
    const dsmem_status st = tp_launch(xs, ys, sigs, reinterpret_cast<unsigned*>(c->base) + kSigErr, c->tp, c->rank,
                                      0, dtype, residual, w, eps, rows, hidden, cluster_size, s, c->wait_limit_ns);
    if (st != DSMEM_OK) return st;
    if (y != nullptr && y != yb && bytes && cudaMemcpyAsync(y, yb, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    return DSMEM_OK;
}

dsmem_status dsmem_tp_emulate(int tp, const void* const* xs, void* const* ys, dsmem_dtype dtype, const void* residual,
                              const void* w, float eps, long long rows, int hidden, int cluster_size,
                              dsmem_stream_t stream) {
    if (xs == nullptr || ys == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    static unsigned* err[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    {
        std::lock_guard<std::mutex> lock(g_tp_mu);
        if (err[dev] == nullptr) {
            if (cudaMalloc(&err[dev], 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(err[dev], 0, 4 * sizeof(unsigned));
        }
    }
    return tp_launch(xs, ys, nullptr, err[dev], tp, 0, 1, dtype, residual, w, eps, rows, hidden, cluster_size,
                     reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_tp_check(dsmem_tp_t c, unsigned* error_bits, unsigned* detail) {
    if (c == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    unsigned v[4] = {};
    unsigned* w = reinterpret_cast<unsigned*>(c->base) + kSigErr;
    if (cudaMemcpy(v, w, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemset(w, 0, sizeof v) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    if (error_bits) *error_bits = v[0];
    if (detail) *detail = v[1];
    return (v[0] & DSMEM_ERRBIT_TIMEOUT) ? DSMEM_ERR_TIMEOUT : (v[0] & DSMEM_ERRBIT_BOUNDS) ? DSMEM_ERR_BOUNDS : DSMEM_OK;
}

dsmem_status dsmem_tp_set_wait_limit_ns(dsmem_tp_t c, unsigned long long ns) {
    if (c == nullptr || ns == 0 || ns > 60000000000ull) return DSMEM_ERR_INVALID_ARGUMENT;
    c->wait_limit_ns = ns;
    return DSMEM_OK;
}

dsmem_status dsmem_tp_close(dsmem_tp_t c) {
    if (c == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    dsmem_status st = DSMEM_OK;
    for (int p = 0; p < c->tp; ++p)
        if (p != c->rank && c->peer[p] != nullptr && cudaIpcCloseMemHandle(c->peer[p]) != cudaSuccess) st = DSMEM_ERR_CUDA;
    if (c->base != nullptr && cudaFree(c->base) != cudaSuccess) st = DSMEM_ERR_CUDA;
    delete c;
    return st;
}

// ------------------------------------------------------------------ NCCL composition (the baseline)
// ncclAllReduce(bf16, sum) of x into `sum`, then the cluster RMSNorm of sum (+ residual). NCCL is
// resolved at run time from the process (libnccl.so.2, normally already loaded by the framework).
namespace {
using nccl_fn_allreduce = int (*)(const void*, void*, size_t, int, int, void*, cudaStream_t);
using nccl_fn_uid = int (*)(void*);
using nccl_fn_init = int (*)(void**, int, const void*, int);   // (comm*, nranks, uid by value, rank)
using nccl_fn_destroy = int (*)(void*);
void* nccl_sym(const char* name) {
    static void* h = [] {
        void* p = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        return p != nullptr ? p : dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }();
    return h != nullptr ? dlsym(h, name) : nullptr;
}
constexpr int kNcclBf16 = 9, kNcclSum = 0, kNcclUidBytes = 128;
struct NcclUid {
    char internal[kNcclUidBytes];
};
}  // namespace

dsmem_status dsmem_nccl_unique_id(void* uid) {
    auto f = reinterpret_cast<nccl_fn_uid>(nccl_sym("ncclGetUniqueId"));
    if (uid == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    if (f == nullptr) return DSMEM_ERR_NCCL;
    return f(uid) == 0 ? DSMEM_OK : DSMEM_ERR_NCCL;
}

dsmem_status dsmem_nccl_comm_init(int world, int rank, const void* uid, dsmem_nccl_comm_t* comm) {
    if (uid == nullptr || comm == nullptr || world < 1 || rank < 0 || rank >= world) return DSMEM_ERR_INVALID_ARGUMENT;
    // ncclCommInitRank takes the 128-byte ncclUniqueId by value
    using init_by_value = int (*)(void**, int, NcclUid, int);
    auto f = reinterpret_cast<init_by_value>(nccl_sym("ncclCommInitRank"));
    if (f == nullptr) return DSMEM_ERR_NCCL;
    NcclUid id;
    std::memcpy(id.internal, uid, kNcclUidBytes);
    return f(comm, world, id, rank) == 0 ? DSMEM_OK : DSMEM_ERR_NCCL;
}

dsmem_status dsmem_nccl_comm_destroy(dsmem_nccl_comm_t comm) {
    auto f = reinterpret_cast<nccl_fn_destroy>(nccl_sym("ncclCommDestroy"));
    if (comm == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    if (f == nullptr) return DSMEM_ERR_NCCL;
    return f(comm) == 0 ? DSMEM_OK : DSMEM_ERR_NCCL;
}

dsmem_status dsmem_tp_allreduce_rmsnorm_nccl(dsmem_nccl_comm_t comm, dsmem_dtype dtype, const void* x,
                                             const void* residual, const void* w, float eps, long long rows,
                                             int hidden, int cluster_size, void* sum, void* y, dsmem_stream_t stream) {
    if (dtype != DSMEM_BF16) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (comm == nullptr || x == nullptr || sum == nullptr || y == nullptr || rows < 0 || hidden <= 0)
        return DSMEM_ERR_INVALID_ARGUMENT;
    auto f = reinterpret_cast<nccl_fn_allreduce>(nccl_sym("ncclAllReduce"));
    if (f == nullptr) return DSMEM_ERR_NCCL;
    if (f(x, sum, (size_t)rows * (size_t)hidden, kNcclBf16, kNcclSum, comm, reinterpret_cast<cudaStream_t>(stream)) != 0)
        return DSMEM_ERR_NCCL;
    if (residual == nullptr)
        return dsmem_rmsnorm_launch(dtype, sum, w, eps, rows, hidden, cluster_size, y, stream);
    return dsmem_rmsnorm_residual_launch(dtype, sum, residual, w, eps, rows, hidden, cluster_size, nullptr, y, stream);
}

}  // extern "C"
