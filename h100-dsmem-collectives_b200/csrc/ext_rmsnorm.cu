// ext_rmsnorm.cu -- cluster-fused RMSNorm for sm_100a.
//
// Computes, per row, y = h * rsqrt(mean(h^2) + eps) * w with h = x (+ residual, written back as the
// pre-norm row when requested), bf16 or f32 in/out, fp32 statistics. Reference kernels:
//   kernels/rmsnorm__llama__clusterfusion.cu:35-108   row per cluster, CTA b owns columns
//     [b*H/N, (b+1)*H/N), partial sum of squares by warp shuffles, cluster AllReduce of one float;
//   kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197   h = x + residual written back,
//     replicated-push scalar AllReduce (one store into slot[b] of every CTA) (:153-169).
// B200 design (one launch, persistent clusters of N CTAs; per CTA 8 consumer warps + 1 producer warp):
//   * rows are taken in groups of R = 16 (two per consumer warp); cluster q handles groups q,
//     q + nclusters, ...; CTA b owns the column slice b of every row;
//   * the producer warp streams each group's R row slices (and residual slices) with one-CTA bulk copies
//     (cp.async.bulk, no multicast) into a ring of 4 shared-memory stages (full/empty mbarriers); a stage
//     is released only after its rows are normalised, so x is read from shared memory twice and never
//     held in registers;
//   * the per-row partial sums of squares meet in the hpc-ops replicated push: lane 0 of each consumer
//     warp writes its 2 partials into slot[set][b][warp*2..] of every CTA with one st.async, whose bytes
//     complete on that CTA's mbarrier of the set (armed for N*R*4 bytes), so there is no release fence and
//     no cluster barrier per group;
//   * the exchange runs one group ahead: a warp sends group i+1's partials before it waits for group
//     i's sums. A CTA can then write a peer's slot set for group i+2 while that peer still reads set i,
//     so slot sets rotate over 4 groups: the set of group j is rewritten for j+4 only after the writer
//     received the owner's partials of j+2, which the owner sends after reading set j;
//   * outputs leave with 16-byte streaming stores.
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"

namespace {

using namespace dsmem;

constexpr int kConsumers = 8;                       // consumer warps
constexpr int kThreadsRms = (kConsumers + 1) * 32;  // + one producer warp
constexpr int kRowsPerWarp = 2;
constexpr int kR = kConsumers * kRowsPerWarp;       // rows per group
constexpr int kStages = 4;                          // most stages (barrier ids); a launch uses 2..4
constexpr int kSets = 4;                            // partial-sum slot sets (see the header comment)
constexpr int kMaxUnitsPerLane = 4;                 // 16-byte units of a row slice per lane (<= 2 KiB)
// barrier ids: full[s] 0..3, empty[s] 4..7, sum[set] 8..11
constexpr int kFull = 0, kEmpty = kStages, kSum = 2 * kStages;

struct RmsArgs {
    const void* x;
    const void* res;     // nullable
    const void* w;
    void* y;
    void* pre;           // nullable: h = x + res
    unsigned* err;
    unsigned long long wait_limit_ns;
    long long rows;
    int hidden;
    float eps;
    uint32_t slice_bytes;   // bytes of one row slice of one CTA
    uint32_t smem_bytes;
    int stages;             // shared-memory stages of the row ring (2..kStages)
};

template <typename T>
struct RmsElem;
template <>
struct RmsElem<__nv_bfloat16> {
    static constexpr int kPer16 = 8;
    static __device__ __forceinline__ void unpack(uint4 p, float* f) {
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
            f[2 * k] = v.x;
            f[2 * k + 1] = v.y;
        }
    }
    static __device__ __forceinline__ uint4 pack(const float* f) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
            w[k] = *reinterpret_cast<const uint32_t*>(&h);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};
template <>
struct RmsElem<float> {
    static constexpr int kPer16 = 4;
    static __device__ __forceinline__ void unpack(uint4 p, float* f) {
        f[0] = __uint_as_float(p.x);
        f[1] = __uint_as_float(p.y);
        f[2] = __uint_as_float(p.z);
        f[3] = __uint_as_float(p.w);
    }
    static __device__ __forceinline__ uint4 pack(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
};

// Shared-memory layout: [0,128) barriers | slots kSets x N x R floats | w slice | stages x R x slice (x2 with residual)
__host__ __device__ constexpr uint32_t rms_slots_off() { return 128u; }
__host__ __device__ constexpr uint32_t rms_w_off(int n) { return 128u + (uint32_t)kSets * n * kR * 4u; }
__host__ __device__ constexpr uint32_t rms_stage_off(int n, uint32_t slice) { return rms_w_off(n) + slice; }
__host__ __device__ constexpr uint32_t rms_smem(int n, uint32_t slice, bool residual, int stages) {
    return rms_stage_off(n, slice) + (uint32_t)stages * kR * slice * (residual ? 2u : 1u);
}

// Bounded wait on barrier i by one thread (its own phase bookkeeping in c.phase).
__device__ __forceinline__ void wait_one(dsb::Ctx& c, int i) { dsb::wait(c, i); }

template <int N, typename T, bool RES, int UPL>
__global__ void __launch_bounds__(kThreadsRms, 3) rmsnorm_cluster_kernel(const RmsArgs a) {
    using E = RmsElem<T>;
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t slice = a.slice_bytes, units = slice >> 4;   // 16-B units per row slice (<= 32 * UPL)
    const uint32_t slots = rms_slots_off(), woff = rms_w_off(N), stage0 = rms_stage_off(N, slice);
    const uint32_t stage_bytes = (uint32_t)kR * slice * (RES ? 2u : 1u);
    const long long nst = a.stages;
    const long long groups = (a.rows + kR - 1) / kR;
    const long long step = (long long)num_clusters();
    const long long first = (long long)cluster_id();
    const long long iters = first < groups ? (groups - 1 - first) / step + 1 : 0;
    const size_t row_bytes = (size_t)a.hidden * sizeof(T);
    const size_t col_off = (size_t)c.rank * slice;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(c.bar(kFull + s), 1);
            mbar_init(c.bar(kEmpty + s), kConsumers);
        }
        for (int s = 0; s < kSets; ++s) mbar_init(c.bar(kSum + s), 1);
        fence_mbar_init();
    }
    {   // weight slice -> shared
        const uint4* wsrc = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(a.w) + col_off);
        uint4* wdst = c.ptr<uint4>(woff);
        for (uint32_t i = threadIdx.x; i < units; i += blockDim.x) wdst[i] = __ldg(wsrc + i);
    }
    __syncthreads();
    cluster_sync();   // barriers of every CTA initialised before any remote store completes on them
    c.deadline = globaltimer() + c.wait_limit;

    if (warp == kConsumers) {
        // ---------------------------------------------------------------- producer warp (lane 0)
        if (lane == 0) {
            const unsigned char* xb = static_cast<const unsigned char*>(a.x);
            const unsigned char* rb = static_cast<const unsigned char*>(a.res);
            for (long long i = 0; i < iters; ++i) {
                const int s = (int)(i % nst);
                if (i >= nst) {   // the stage's previous group is normalised by every consumer warp
                    c.deadline = globaltimer() + c.wait_limit;
                    wait_one(c, kEmpty + s);
                }
                const long long r0 = (first + i * step) * kR;
                const int nr = (int)min((long long)kR, a.rows - r0);
                const uint32_t dst = stage0 + (uint32_t)s * stage_bytes;
                dsb::arm(c, kFull + s, (uint32_t)nr * slice * (RES ? 2u : 1u));
                for (int r = 0; r < nr; ++r) {
                    const size_t src = (size_t)(r0 + r) * row_bytes + col_off;
                    bulk_load_g2s(c.sa + dst + (uint32_t)r * slice, xb + src, slice, c.bar(kFull + s));
                    if (RES)
                        bulk_load_g2s(c.sa + dst + ((uint32_t)kR + r) * slice, rb + src, slice, c.bar(kFull + s));
                }
            }
        }
        __syncwarp();   // reconverge before the aligned cluster barrier
    } else {
        // ---------------------------------------------------------------- consumer warps
        const uint4* wp = c.ptr<const uint4>(woff);
        // h of row k of group i (slot of the stage), unit u, as floats
        auto load_h = [&](long long i, int k, uint32_t u, float* f) {
            const uint4* xs = c.ptr<const uint4>(stage0 + (uint32_t)(i % nst) * stage_bytes);
            const uint32_t idx = (warp * kRowsPerWarp + k) * units + u;
            E::unpack(xs[idx], f);
            if (RES) {
                float r[E::kPer16];
                E::unpack(xs[(size_t)kR * units + idx], r);
#pragma unroll
                for (int e = 0; e < E::kPer16; ++e) f[e] += r[e];
                E::unpack(E::pack(f), f);   // h rounded to the element type (the pre-norm output)
            }
        };
        // wait for group j's rows, reduce my rows' sums of squares and push them to every CTA
        auto send = [&](long long j) {
            wait_one(c, kFull + (int)(j % nst));
            const long long row0 = (first + j * step) * kR + (long long)warp * kRowsPerWarp;
            float ss[kRowsPerWarp];
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) {
                ss[k] = 0.f;
                if (row0 + k < a.rows) {
#pragma unroll
                    for (int q = 0; q < UPL; ++q) {
                        const uint32_t u = lane + 32u * q;
                        if (u < units) {
                            float f[E::kPer16];
                            load_h(j, k, u, f);
#pragma unroll
                            for (int e = 0; e < E::kPer16; ++e) ss[k] = fmaf(f[e], f[e], ss[k]);
                        }
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], off);
            }
            const int set = (int)(j % kSets);
            if (threadIdx.x == 0) dsb::arm(c, kSum + set, (uint32_t)N * kR * 4u);
            if (lane == 0) {
                const uint32_t dst = slots + (((uint32_t)set * N + c.rank) * kR + warp * kRowsPerWarp) * 4u;
                const uint32_t bar = c.bar(kSum + set);
                for (uint32_t q = 0; q < (uint32_t)N; ++q) {
                    const uint32_t rd = mapa(c.sa + dst, q), rbar = mapa(bar, q);
                    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1,%2}, [%3];" ::
                                     "r"(rd),
                                 "f"(ss[0]), "f"(ss[1]), "r"(rbar)
                                 : "memory");
                }
            }
        };
        if (iters > 0) send(0);
        for (long long i = 0; i < iters; ++i) {
            c.deadline = globaltimer() + c.wait_limit;
            if (i + 1 < iters) send(i + 1);   // one group ahead
            const int set = (int)(i % kSets);
            wait_one(c, kSum + set);
            const long long row0 = (first + i * step) * kR + (long long)warp * kRowsPerWarp;
            const float* sl = c.ptr<const float>(slots + (uint32_t)set * N * kR * 4u);
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) {
                const long long row = row0 + k;
                float tot = 0.f;
#pragma unroll
                for (int q = 0; q < N; ++q) tot += sl[q * kR + warp * kRowsPerWarp + k];
                const float scale = rsqrtf(tot / (float)a.hidden + a.eps);
                if (row >= a.rows) continue;
                uint4* yo = reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.y) + (size_t)row * row_bytes + col_off);
                uint4* po = RES && a.pre != nullptr
                                ? reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.pre) + (size_t)row * row_bytes +
                                                           col_off)
                                : nullptr;
#pragma unroll
                for (int q = 0; q < UPL; ++q) {
                    const uint32_t u = lane + 32u * q;
                    if (u < units) {
                        float f[E::kPer16], w[E::kPer16];
                        load_h(i, k, u, f);
                        if (RES && po != nullptr) __stcs(po + u, E::pack(f));
                        E::unpack(wp[u], w);
#pragma unroll
                        for (int e = 0; e < E::kPer16; ++e) f[e] = f[e] * scale * w[e];
                        __stcs(yo + u, E::pack(f));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(c.bar(kEmpty + (int)(i % nst)));   // stage free for the producer
        }
    }
    dsb::finish(c);   // no CTA leaves while a peer may still store into its slots
}

struct RmsKey {
    const void* fn;
    int dev;
    uint32_t smem;
    bool operator<(const RmsKey& o) const {
        return fn < o.fn || (fn == o.fn && (dev < o.dev || (dev == o.dev && smem < o.smem)));
    }
};
std::mutex g_mu;
std::map<RmsKey, int> g_occ;
unsigned* g_err[64] = {};

template <int N, typename T, bool RES>
const void* rms_fn(int upl) {
    switch (upl) {
        case 1: return reinterpret_cast<const void*>(&rmsnorm_cluster_kernel<N, T, RES, 1>);
        case 2: return reinterpret_cast<const void*>(&rmsnorm_cluster_kernel<N, T, RES, 2>);
        case 4: return reinterpret_cast<const void*>(&rmsnorm_cluster_kernel<N, T, RES, 4>);
    }
    return nullptr;
}

template <typename T, bool RES>
const void* pick(int n, int upl) {
    switch (n) {
        case 1: return rms_fn<1, T, RES>(upl);
        case 2: return rms_fn<2, T, RES>(upl);
        case 4: return rms_fn<4, T, RES>(upl);
        case 8: return rms_fn<8, T, RES>(upl);
        case 16: return rms_fn<16, T, RES>(upl);
    }
    return nullptr;
}

dsmem_status rms_launch(int dtype, const void* x, const void* res, const void* w, void* y, void* pre, float eps,
                        long long rows, int hidden, int cluster_size, int max_clusters, cudaStream_t stream) {
    if (x == nullptr || w == nullptr || y == nullptr || rows < 0 || hidden <= 0 || !(eps >= 0.f))
        return DSMEM_ERR_INVALID_ARGUMENT;
    if (dtype != DSMEM_BF16 && dtype != DSMEM_F32) return DSMEM_ERR_ILLEGAL_CONFIG;
    const int n = cluster_size;
    if (!(n == 1 || n == 2 || n == 4 || n == 8 || n == 16)) return DSMEM_ERR_INVALID_ARGUMENT;
    const size_t eb = dtype == DSMEM_BF16 ? 2 : 4;
    if ((size_t)hidden % n) return DSMEM_ERR_ILLEGAL_CONFIG;
    const size_t slice = (size_t)hidden / n * eb;
    if (slice % 16 || slice / 16 > (size_t)kMaxUnitsPerLane * 32) return DSMEM_ERR_ILLEGAL_CONFIG;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(res) | reinterpret_cast<uintptr_t>(pre);
    if (al & 15u) return DSMEM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DSMEM_OK;
    const bool has_res = res != nullptr;
    const uint32_t units = (uint32_t)(slice / 16);
    const int upl = units <= 32 ? 1 : units <= 64 ? 2 : 4;
    // the deepest ring (at most kStages, at least 2) that fits the per-CTA shared-memory limit
    int stages = kStages;
    while (stages > 2 && rms_smem(n, (uint32_t)slice, has_res, stages) > dsb::kSmemLimit) --stages;
    const uint32_t smem = rms_smem(n, (uint32_t)slice, has_res, stages);
    if (smem > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    const void* fn = dtype == DSMEM_BF16
                         ? (has_res ? pick<__nv_bfloat16, true>(n, upl) : pick<__nv_bfloat16, false>(n, upl))
                         : (has_res ? pick<float, true>(n, upl) : pick<float, false>(n, upl));
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreadsRms, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int resident = 0;
    RmsArgs a{};
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_err[dev] == nullptr) {   // error bits, timeout detail, cluster id, spare
            if (cudaMalloc(&g_err[dev], 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(g_err[dev], 0, 4 * sizeof(unsigned));
        }
        const RmsKey key{fn, dev, smem};
        auto it = g_occ.find(key);
        if (it == g_occ.end()) {
            if (n > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                return DSMEM_ERR_CUDA;
            if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return DSMEM_ERR_CUDA;
            if (cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared) != cudaSuccess)
                return DSMEM_ERR_CUDA;
            cfg.gridDim = dim3((unsigned)n, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&resident, fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
            g_occ[key] = resident;
        } else {
            resident = it->second;
        }
        a.err = g_err[dev];
    }
    if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;
    const long long groups = (rows + kR - 1) / kR;
    long long clusters = std::min<long long>(groups, resident);
    if (max_clusters > 0) clusters = std::min<long long>(clusters, max_clusters);
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    a.x = x;
    a.res = res;
    a.w = w;
    a.y = y;
    a.pre = pre;
    a.wait_limit_ns = 1000000000ull;
    a.rows = rows;
    a.hidden = hidden;
    a.eps = eps;
    a.slice_bytes = (uint32_t)slice;
    a.smem_bytes = smem;
    a.stages = stages;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

}  // namespace

extern "C" {

dsmem_status dsmem_rmsnorm_launch(dsmem_dtype dtype, const void* x, const void* w, float eps, long long rows,
                                  int hidden, int cluster_size, void* y, dsmem_stream_t stream) {
    return rms_launch(dtype, x, nullptr, w, y, nullptr, eps, rows, hidden, cluster_size, 0,
                      reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_rmsnorm_residual_launch(dsmem_dtype dtype, const void* x, const void* residual, const void* w,
                                           float eps, long long rows, int hidden, int cluster_size, void* pre_norm,
                                           void* y, dsmem_stream_t stream) {
    if (residual == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    return rms_launch(dtype, x, residual, w, y, pre_norm, eps, rows, hidden, cluster_size, 0,
                      reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_rmsnorm_check(int device, unsigned* error_bits) {
    unsigned v = 0;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (device < 0 || device >= 64) return DSMEM_ERR_INVALID_ARGUMENT;
        if (g_err[device] != nullptr) {
            if (cudaMemcpy(&v, g_err[device], sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(g_err[device], 0, 4 * sizeof(unsigned));
        }
    }
    if (error_bits) *error_bits = v;
    return DSMEM_OK;
}

}  // extern "C"
