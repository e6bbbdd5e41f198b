// ext_rmsnorm.cu -- cluster-fused RMSNorm for sm_100a.
//
// Computes, per row, y = h * rsqrt(mean(h^2) + eps) * w with h = x (+ residual, written back as the
// pre-norm row when requested), bf16 or f32 in/out, fp32 statistics. Reference kernels:
//   kernels/rmsnorm__llama__clusterfusion.cu:35-108   row per cluster, CTA b owns columns
//     [b*H/N, (b+1)*H/N), partial sum of squares by warp shuffles, cluster AllReduce of one float;
//   kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197   h = x + residual written back,
//     replicated-push scalar AllReduce (one store into slot[b] of every CTA) (:153-169).
// B200 design (one launch, persistent clusters of N CTAs; per CTA 8 consumer warps + 1 producer warp):
//   * cluster q of C owns the contiguous rows [q*rows/C, (q+1)*rows/C), taken in groups of R = 16 (two per
//     consumer warp; the last group partial); CTA b owns the column slice b of every row;
//   * the producer warp streams the weight slice and each group's R row slices (and residual slices) with
//     one-CTA bulk copies (cp.async.bulk, no multicast) into a ring of 2..4 shared-memory stages (as many
//     as fit; full/empty mbarriers); a stage is released only after its rows are normalised, so x is read
//     from shared memory twice and never held in registers. The producer starts loading before the
//     cluster rendezvous (split arrive/wait), which only the remote stores need;
//   * the per-row partial sums of squares meet in the hpc-ops replicated push: lane q < N of each consumer
//     warp writes the warp's 2 partials into slot[set][b][warp*2..] of CTA q with one st.async, whose
//     bytes complete on that CTA's mbarrier of the set (armed for N*R*4 bytes), so there is no release
//     fence and no cluster barrier per group;
//   * the exchange runs up to L = 1 group ahead (rms_lookahead): before it waits for group i's sums a
//     warp sends group i+1's partials if its rows have landed, else right after normalising i. A writer sends group g after it received everyone's
//     partials of g-L-1, so an owner may still be reading any set of groups g-L-1 .. g+L-1 when g's
//     partials arrive: slot sets rotate over kSets >= 2L+2 groups, so g's set is none of those;
//   * outputs leave with 16-byte streaming stores; the weight slice sits in registers when it fits.
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "f32x2.cuh"

namespace {

using namespace dsmem;
using namespace dsb2;

constexpr int kConsumers = 8;                       // consumer warps
constexpr int kThreadsRms = (kConsumers + 1) * 32;  // + one producer warp
constexpr int kRowsPerWarp = 2;                     // one st.async.v2 / float2 of partials per warp
static_assert(kRowsPerWarp == 2, "the partial exchange moves float2 pairs");
constexpr int kR = kConsumers * kRowsPerWarp;       // rows per group
constexpr int kStages = 4;                          // most stages (barrier ids); a launch uses 2..4
constexpr int kSets = 8;                            // partial-sum slot sets (see the header comment)
constexpr int kMaxUnitsPerLane = 4;                 // 16-byte units of a row slice per lane (<= 2 KiB)
constexpr int kCtasPerSm = 3;                       // occupancy target (registers capped to fit it)
constexpr uint32_t kSmemPerSm = 233472;             // 228 KiB of shared memory per SM
// barrier ids: full[s] 0..3, empty[s] 4..7, weight 8, sum[set] 16..23 (id 15 would overlap the
// end-of-kernel flag word at byte 120)
constexpr int kFull = 0, kEmpty = kStages, kWBar = 2 * kStages, kSum = 16;
static_assert(8 * kWBar < (int)dsb::kFlagOff && kSum * 8 > (int)dsb::kFlagOff, "barriers overlap the flag word");
// partial sums are sent at most `lookahead` groups ahead of the group being normalised (only for groups
// whose rows have landed, so the first group never waits for later loads). Measured: 1 is best; 3 delays
// every group's stores by the partials of the groups ahead (config 3: 21.9 us against 18.5 us).
__host__ __device__ constexpr int rms_lookahead(int) { return 1; }
static_assert(kSets >= 2 * rms_lookahead(kStages) + 2, "slot sets must cover 2 * lookahead + 2 groups");

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

// Shared-memory layout: [0,256) barriers | slots kSets x N x R floats | w slice | stages x R x slice (x2 with residual)
__host__ __device__ constexpr uint32_t rms_slots_off() { return 256u; }
__host__ __device__ constexpr uint32_t rms_w_off(int n) { return rms_slots_off() + (uint32_t)kSets * n * kR * 4u; }
__host__ __device__ constexpr uint32_t rms_stage_off(int n, uint32_t slice) { return rms_w_off(n) + slice; }
__host__ __device__ constexpr uint32_t rms_smem(int n, uint32_t slice, bool residual, int stages) {
    return rms_stage_off(n, slice) + (uint32_t)stages * kR * slice * (residual ? 2u : 1u);
}

// Bounded wait on barrier i by one thread (its own phase bookkeeping in c.phase).
__device__ __forceinline__ void wait_one(dsb::Ctx& c, int i) { dsb::wait(c, i); }

template <int N, typename T, bool RES, int UPL>
__global__ void __launch_bounds__(kThreadsRms, kCtasPerSm) rmsnorm_cluster_kernel(const RmsArgs a) {
    using E = RmsElem<T>;
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t slice = a.slice_bytes, units = slice >> 4;   // 16-B units per row slice (<= 32 * UPL)
    const uint32_t slots = rms_slots_off(), woff = rms_w_off(N), stage0 = rms_stage_off(N, slice);
    const uint32_t stage_bytes = (uint32_t)kR * slice * (RES ? 2u : 1u);
    const uint32_t nst = (uint32_t)a.stages;
    // cluster q owns the contiguous rows [lo, hi) = [q*rows/C, (q+1)*rows/C): every cluster moves the same
    // bytes (within one row), in groups of kR rows (the last one partial)
    const long long nclu = (long long)num_clusters(), cq = (long long)cluster_id();
    const long long lo = cq * a.rows / nclu, hi = (cq + 1) * a.rows / nclu;
    const long long iters = (hi - lo + kR - 1) / kR;
    const size_t row_bytes = (size_t)a.hidden * sizeof(T);
    const size_t col_off = (size_t)c.rank * slice;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(c.bar(kFull + s), 1);
            mbar_init(c.bar(kEmpty + s), kConsumers);
        }
        mbar_init(c.bar(kWBar), 1);
        for (int s = 0; s < kSets; ++s) mbar_init(c.bar(kSum + s), 1);
        fence_mbar_init();
    }
    __syncthreads();   // local barriers initialised: the producer may load at once
    // Split cluster barrier: every thread arrives now (releasing its barrier inits cluster-wide); consumers
    // wait before their first remote store, the producer only after it has issued its loads, so the first
    // HBM reads overlap the cluster rendezvous.
    cluster_arrive();
    c.deadline = globaltimer() + c.wait_limit;

    if (warp == kConsumers) {
        // ---------------------------------------------------------------- producer warp (lane 0)
        if (lane == 0) {
            dsb::arm(c, kWBar, slice);   // weight slice -> shared, on its own barrier
            bulk_load_g2s(c.sa + woff, static_cast<const unsigned char*>(a.w) + col_off, slice, c.bar(kWBar));
            const unsigned char* xb = static_cast<const unsigned char*>(a.x);
            const unsigned char* rb = static_cast<const unsigned char*>(a.res);
            uint32_t s = 0;   // stage of group i
            for (long long i = 0; i < iters; ++i, s = (s + 1 == nst) ? 0u : s + 1) {
                if (i >= (long long)nst) {   // the stage's previous group is normalised by every consumer warp
                    c.deadline = globaltimer() + c.wait_limit;
                    wait_one(c, kEmpty + (int)s);
                }
                const long long r0 = lo + i * kR;
                const int nr = (int)min((long long)kR, hi - r0);
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
        cluster_wait();
    } else {
        // ---------------------------------------------------------------- consumer warps
        cluster_wait();   // every CTA's barriers initialised before any remote store completes on them
        wait_one(c, kWBar);
        const uint4* wp = c.ptr<const uint4>(woff);
        const float inv_hidden = 1.0f / (float)a.hidden;
        constexpr int P = E::kPairs;
        // this lane's weight units as fp32 pairs, held in registers when they fit in 16 of them
        constexpr bool kWReg = UPL * P * 2 <= 16;
        f2x wr[kWReg ? UPL : 1][P];
        if constexpr (kWReg) {
#pragma unroll
            for (int q = 0; q < UPL; ++q) {
                const uint32_t u = lane + 32u * q;
                if (u < units) E::unpack(wp[u], wr[q]);
            }
        }
        // h of row k of the group held in stage s, unit u, as fp32 pairs
        auto load_h = [&](uint32_t s, int k, uint32_t u, f2x* f) {
            const uint4* xs = c.ptr<const uint4>(stage0 + s * stage_bytes);
            const uint32_t idx = (warp * kRowsPerWarp + k) * units + u;
            E::unpack(xs[idx], f);
            if (RES) {
                f2x r[P];
                E::unpack(xs[(size_t)kR * units + idx], r);
#pragma unroll
                for (int e = 0; e < P; ++e) f[e] = f2_add(f[e], r[e]);
                E::unpack(E::pack(f), f);   // h rounded to the element type (the pre-norm output)
            }
        };
        // wait for group j's rows (stage s), reduce my rows' sums of squares and push them to every CTA
        auto send = [&](long long j, uint32_t s) {
            wait_one(c, kFull + (int)s);
            const long long row0 = lo + j * kR + (long long)warp * kRowsPerWarp;
            float ss[kRowsPerWarp];
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) {
                f2x acc = 0ull;   // (+0.0f, +0.0f)
                if (row0 + k < hi) {
#pragma unroll
                    for (int q = 0; q < UPL; ++q) {
                        const uint32_t u = lane + 32u * q;
                        if (u < units) {
                            f2x f[P];
                            load_h(s, k, u, f);
#pragma unroll
                            for (int e = 0; e < P; ++e) acc = f2_fma(f[e], f[e], acc);
                        }
                    }
                }
                const float2 a2 = f2_split(acc);
                ss[k] = a2.x + a2.y;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], off);
            }
            const int set = (int)(j & (kSets - 1));
            if (threadIdx.x == 0) dsb::arm(c, kSum + set, (uint32_t)N * kR * 4u);
            if (lane < (uint32_t)N) {   // lane q stores the pair into CTA q (the butterfly left it in every lane)
                const uint32_t dst = slots + (((uint32_t)set * N + c.rank) * kR + warp * kRowsPerWarp) * 4u;
                const uint32_t rd = mapa(c.sa + dst, lane), rbar = mapa(c.bar(kSum + set), lane);
                asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1,%2}, [%3];" ::"r"(rd),
                             "f"(ss[0]), "f"(ss[1]), "r"(rbar)
                             : "memory");
            }
        };
        constexpr long long kLook = rms_lookahead(kStages);
        uint32_t s = 0, s_send = 0;   // stages of group i and of the next group to send
        long long sent = 0;            // groups whose partials this warp has sent
        auto send_next = [&]() {
            send(sent++, s_send);
            s_send = (s_send + 1 == nst) ? 0u : s_send + 1;
        };
        if (iters > 0) send_next();
        for (long long i = 0; i < iters; ++i) {
            c.deadline = globaltimer() + c.wait_limit;
            // The partials of groups i+1 .. i+L (L = rms_lookahead) whose rows have already landed go out
            // before group i is normalised, so their exchanges overlap this group's work; group i+1's goes
            // out right after it at the latest. No group waits for a later group's load.
            while (sent < iters && sent <= i + kLook) {
                const int fb = kFull + (int)s_send;
                const bool ready = __shfl_sync(0xffffffffu, mbar_try_wait_parity(c.bar(fb), (c.phase >> fb) & 1u), 0);
                if (!ready) break;
                send_next();
            }
            const int set = (int)(i & (kSets - 1));
            wait_one(c, kSum + set);
            const long long row0 = lo + i * kR + (long long)warp * kRowsPerWarp;
            // the N partials of my two rows: lane q < N loads CTA q's pair, a butterfly over N lanes sums them
            float2 part = make_float2(0.f, 0.f);
            if (lane < (uint32_t)N)
                part = *c.ptr<const float2>(slots + (((uint32_t)set * N + lane) * kR + warp * kRowsPerWarp) * 4u);
#pragma unroll
            for (int off = N / 2; off > 0; off >>= 1) {
                part.x += __shfl_xor_sync(0xffffffffu, part.x, off);
                part.y += __shfl_xor_sync(0xffffffffu, part.y, off);
            }
            const float tot2[kRowsPerWarp] = {__shfl_sync(0xffffffffu, part.x, 0), __shfl_sync(0xffffffffu, part.y, 0)};
#pragma unroll
            for (int k = 0; k < kRowsPerWarp; ++k) {
                const long long row = row0 + k;
                const float scale = rsqrtf(fmaf(tot2[k], inv_hidden, a.eps));
                const f2x scale2 = f2_make(scale, scale);
                if (row >= hi) continue;
                uint4* yo = reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.y) + (size_t)row * row_bytes + col_off);
                uint4* po = RES && a.pre != nullptr
                                ? reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.pre) + (size_t)row * row_bytes +
                                                           col_off)
                                : nullptr;
#pragma unroll
                for (int q = 0; q < UPL; ++q) {
                    const uint32_t u = lane + 32u * q;
                    if (u < units) {
                        f2x f[P];
                        load_h(s, k, u, f);
                        if (RES && po != nullptr) __stcs(po + u, E::pack(f));
                        if constexpr (kWReg) {
#pragma unroll
                            for (int e = 0; e < P; ++e) f[e] = f2_mul(f2_mul(f[e], scale2), wr[q][e]);
                        } else {
                            f2x w[P];
                            E::unpack(wp[u], w);
#pragma unroll
                            for (int e = 0; e < P; ++e) f[e] = f2_mul(f2_mul(f[e], scale2), w[e]);
                        }
                        __stcs(yo + u, E::pack(f));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(c.bar(kEmpty + (int)s));   // stage free for the producer
            s = (s + 1 == nst) ? 0u : s + 1;
            if (sent == i + 1 && sent < iters) send_next();
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
    // Ring depth: the deepest (<= kStages) that still lets kCtasPerSm CTAs share an SM (228 KiB of shared
    // memory, 1 KiB reserved per CTA), else the deepest that fits one CTA; at least 2.
    auto per_sm = [&](int st) { return (int)(kSmemPerSm / (rms_smem(n, (uint32_t)slice, has_res, st) + 1024u)); };
    int stages = kStages;
    while (stages > 2 && per_sm(stages) < kCtasPerSm) --stages;
    if (per_sm(stages) < kCtasPerSm) {
        stages = kStages;
        while (stages > 2 && rms_smem(n, (uint32_t)slice, has_res, stages) > dsb::kSmemLimit) --stages;
    }
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

