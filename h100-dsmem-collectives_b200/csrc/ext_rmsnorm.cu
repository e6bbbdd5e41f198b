// ext_rmsnorm.cu -- cluster-fused RMSNorm for sm_100a.
//
// Computes, per row, y = h * rsqrt(mean(h^2) + eps) * w with h = x (+ residual, written back as the
// pre-norm row when requested), bf16 or f32 in/out, fp32 statistics. Reference kernels:
//   kernels/rmsnorm__llama__clusterfusion.cu:35-108   row per cluster, CTA b owns columns
//     [b*H/N, (b+1)*H/N), partial sum of squares by warp shuffles, cluster AllReduce of one float;
//   kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197   h = x + residual written back,
//     replicated-push scalar AllReduce (one store into slot[b] of every CTA) (:153-169).
// B200 design (one launch, persistent clusters of N CTAs; per CTA 1 producer warp, 4 sum warps and 8
// normalising warps):
//   * rows go in groups of R = 16 (only the tensor's last group is partial); cluster q of C takes groups
//     q, q + C, q + 2C, ..; CTA b owns the column slice b of every row;
//   * the producer warp streams the weight slice (one bulk copy) and each group's R row slices (and residual
//     slices) as ONE tiled TMA load per operand: a 3-D tensor map {chunk, chunks per row, rows} whose box
//     is the CTA's slice of 16 rows (no multicast; rows past the tensor read as zeros). Loads go into a
//     ring of 2..12 shared-memory stages (as many as fit two CTAs per SM; full/empty mbarriers), at most
//     kAhead groups beyond the last one landed; a stage is released only after its rows are normalised, so
//     x is read from HBM once and from shared memory twice, never held in registers. The cluster
//     rendezvous (split arrive/wait) starts before the first load and completes under the loads;
//   * sum warp v computes the partial sums of squares of rows 4v..4v+3 of a group as soon as its stage has
//     landed and meets the peers' partials in the hpc-ops replicated push: lane q < N writes the 4 partials
//     into slot[set][b][4v..] of CTA q with one st.async, whose bytes complete on that CTA's mbarrier of the
//     set (armed for N*R*4 bytes), so there is no release fence and no cluster barrier per group;
//   * normalising warp w waits for the set's barrier, sums the N partials of rows 2w, 2w+1 (lane-parallel
//     loads, butterfly), scales, multiplies by the weight and writes the rows. The sum warps run up to the
//     ring depth ahead, so the exchange of later groups overlaps this group's stores; slot sets rotate over
//     a power of two >= 2 * stages of sets (the reuse argument is at kMaxSets);
//   * outputs leave with 16-byte streaming stores; the weight slice sits in registers when it fits.
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "f32x2.cuh"
#include "smem_attr.cuh"
#include "tmap.cuh"

namespace {

using namespace dsmem;
using namespace dsb2;

// Warp roles: kNormWarps normalise (2 rows of a 16-row group each), kSsWarps compute the rows' sums of
// squares and push them to the cluster (4 rows each), one producer warp streams the rows in. The sum
// warps run ahead of the normalising warps, so a group's exchange overlaps the previous group's stores.
constexpr int kNormWarps = 8;
constexpr int kSsWarps = 4;
constexpr int kConsumers = kNormWarps;              // arrivals that free a stage
constexpr int kProducerWarp = kNormWarps + kSsWarps;
constexpr int kThreadsRms = (kProducerWarp + 1) * 32;
constexpr int kRowsPerWarp = 2;                     // rows a normalising warp owns in a group
constexpr int kRowsPerSs = 4;                       // rows a sum warp owns in a group (one st.async.v4)
constexpr int kR = kNormWarps * kRowsPerWarp;       // rows per group
static_assert(kR == kSsWarps * kRowsPerSs, "both roles cover the group");
constexpr int kMaxStages = 12;                      // most ring stages (barrier ids); a launch uses 2..12
constexpr int kAhead = 2;                           // groups in flight beyond the last one landed (<= 2 stages)
constexpr int kMaxSets = 32;                        // most partial-sum slot sets (a power of two >= 2 * stages)
constexpr int kMaxUnitsPerLane = 4;                 // 16-byte units of a row slice per lane (<= 2 KiB)
constexpr int kCtasPerSm = 2;                       // occupancy target (registers capped to fit it)
constexpr uint32_t kSmemPerSm = 233472;             // 228 KiB of shared memory per SM
// barrier ids (8 bytes each, [0, 512) of shared memory): full[s] 0..11, weight 12, empty[s] 16..27,
// sum[set] 32..63; id 15 holds the end-of-kernel flag word (byte 120)
constexpr int kFull = 0, kWBar = kMaxStages, kEmpty = 16, kSum = 32;
constexpr uint32_t kBarBytes = 8u * (kSum + kMaxSets);
static_assert(8 * kWBar < (int)dsb::kFlagOff && kEmpty * 8 > (int)dsb::kFlagOff && kEmpty + kMaxStages <= kSum,
              "barrier ids overlap");
// Slot-set reuse: CTA b's sum warps send group g only after b's stage for g was loaded, i.e. after b's
// normalising warps finished group g - stages, which needed every peer's partials of g - stages. A peer q's
// sum warps sent g - stages only after q's stage for it was loaded, i.e. after q's normalising warps finished
// g - 2 stages (and q's sum barrier of that group completed). So when g's partials reach q, q may still read
// the sets of groups g - 2 stages + 1 .. g - 1 only, and 2 * stages sets keep g's set out of them.
static_assert(kMaxSets >= 2 * kMaxStages, "slot sets must cover 2 * stages groups");

struct RmsArgs {
    // 3-D views of x and of the residual: {chunk elements, chunks per row, rows}; one box = 16 rows of one
    // CTA's column slice, so a group's rows arrive with one TMA load per operand
    alignas(64) CUtensorMap tmx;
    alignas(64) CUtensorMap tmr;
    int chunks_per_slice;   // box extent along the chunk dimension
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
    int stages;             // shared-memory stages of the row ring (2..kMaxStages)
    int sets;               // partial-sum slot sets: a power of two >= 2 * stages
};

// Shared-memory layout: [0,512) barriers | slots sets x N x R floats | w slice | stages x R x slice (x2 with residual)
__host__ __device__ constexpr uint32_t rms_slots_off() { return kBarBytes; }
__host__ __device__ constexpr uint32_t rms_w_off(int n, int sets) { return rms_slots_off() + (uint32_t)sets * n * kR * 4u; }
__host__ __device__ constexpr uint32_t rms_stage_off(int n, int sets, uint32_t slice) {
    return rms_w_off(n, sets) + ((slice + 127u) & ~127u);   // stages start 128-byte aligned (TMA destination)
}
__host__ __device__ constexpr uint32_t rms_smem(int n, uint32_t slice, bool residual, int stages, int sets) {
    return rms_stage_off(n, sets, slice) + (uint32_t)stages * kR * slice * (residual ? 2u : 1u);
}
__host__ __device__ constexpr int rms_sets(int stages) {
    int s = 2;
    while (s < 2 * stages) s *= 2;
    return s;
}

// Bounded wait by one thread for barrier i to finish the phase of parity `par` (the phases follow from the
// group index, so the kernel keeps no per-barrier phase word).
__device__ __forceinline__ void wait_par(dsb::Ctx& c, int i, uint32_t par) {
    if (c.dead) return;
    if (mbar_try_wait_parity(c.bar(i), par)) return;
    if (!mbar_wait_parity_until(c.bar(i), par, c.deadline)) {
        c.dead = true;
        if ((threadIdx.x & 31) == 0) dsb::report_timeout(c, i);
    }
}

template <int N, typename T, bool RES, int UPL>
__global__ void __launch_bounds__(kThreadsRms, kCtasPerSm) rmsnorm_cluster_kernel(const __grid_constant__ RmsArgs a) {
    using E = RmsElem<T>;
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t slice = a.slice_bytes, units = slice >> 4;   // 16-B units per row slice (<= 32 * UPL)
    const uint32_t nsets = (uint32_t)a.sets;
    const uint32_t slots = rms_slots_off(), woff = rms_w_off(N, a.sets), stage0 = rms_stage_off(N, a.sets, slice);
    const uint32_t stage_bytes = (uint32_t)kR * slice * (RES ? 2u : 1u);
    const uint32_t nst = (uint32_t)a.stages;
    // Groups of kR rows (G = ceil(rows / kR); only the tensor's last group is partial, its rows past the end
    // arrive as zeros). Cluster q takes groups q, q + C, q + 2C, ..: the clusters stream neighbouring groups
    // at the same time (measured 4% faster than contiguous blocks per cluster at 16384 x 4096 bf16).
    const long long nclu = (long long)num_clusters(), cq = (long long)cluster_id();
    const long long groups = (a.rows + kR - 1) / kR;
    const long long iters = groups > cq ? (groups - cq + nclu - 1) / nclu : 0;
    const long long hi = a.rows;
    auto group_of = [&](long long i) { return cq + i * nclu; };   // the cluster's i-th group
    const size_t row_bytes = (size_t)a.hidden * sizeof(T);
    const size_t col_off = (size_t)c.rank * slice;

    const int cy = (int)c.rank * a.chunks_per_slice;   // this CTA's first chunk of a row
    // Issue the loads of the cluster's i-th group into stage s: whole boxes (rows past the tensor included)
    // on full[s].
    auto load_group = [&](long long i, uint32_t s) {
        const int r0 = (int)(group_of(i) * kR);
        const uint32_t dst = stage0 + s * stage_bytes;
        dsb::arm(c, kFull + (int)s, stage_bytes);
        tma_load_3d(c.sa + dst, &a.tmx, 0, cy, r0, c.bar(kFull + (int)s));
        if (RES) tma_load_3d(c.sa + dst + (uint32_t)kR * slice, &a.tmr, 0, cy, r0, c.bar(kFull + (int)s));
    };
    if (threadIdx.x == kProducerWarp * 32) {   // the barriers the loads complete on
        for (uint32_t s = 0; s < nst; ++s) mbar_init(c.bar(kFull + (int)s), 1);
        mbar_init(c.bar(kWBar), 1);
        fence_mbar_init();
        prefetch_tmap(&a.tmx);
        if (RES) prefetch_tmap(&a.tmr);
    } else if (warp == 0) {   // lane l initialises empty[l] and sum[l] (in parallel)
        if (lane < nst) mbar_init(c.bar(kEmpty + (int)lane), kConsumers);
        if (lane < nsets) mbar_init(c.bar(kSum + (int)lane), 1);
        fence_mbar_init();
    }
    __syncthreads();   // every local barrier initialised
    // Split cluster barrier: every thread arrives now (releasing its barrier inits cluster-wide); consumers
    // wait before their first remote store, the producer only after its loop, so the HBM reads overlap the
    // cluster rendezvous. The arrivals go out before the first bulk load: arriving after the loads were
    // issued held the cluster's rendezvous back until most of the loaded bytes had come in (about 5 us at
    // 4096 x 4096 bf16 on B200).
    cluster_arrive();
    c.deadline = globaltimer() + c.wait_limit;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------------- producer warp (lane 0)
        if (lane == 0) {
            dsb::arm(c, kWBar, slice);   // weight slice -> shared, on its own barrier
            bulk_load_g2s(c.sa + woff, static_cast<const unsigned char*>(a.w) + col_off, slice, c.bar(kWBar));
            // Group i goes out once group i - kAhead has landed (fewer bytes queued per CTA: the first groups
            // of every CTA arrive sooner and closer together) and its stage's previous group is normalised.
            uint32_t s = 0, round = 0;   // group i = round * nst + s
            uint32_t sa = 0, pa = 0;     // stage and full-phase parity of group i - kAhead
            for (long long i = 0; i < iters; ++i) {
                c.deadline = globaltimer() + c.wait_limit;
                if (i >= kAhead) {
                    wait_par(c, kFull + (int)sa, pa);
                    if (++sa == nst) sa = 0, pa ^= 1u;
                }
                if (round > 0) wait_par(c, kEmpty + (int)s, (round - 1u) & 1u);
                load_group(i, s);
                if (++s == nst) s = 0, ++round;
            }
        }
        __syncwarp();   // reconverge before the aligned cluster barrier
        cluster_wait();
    } else {
        cluster_wait();   // every CTA's barriers initialised before any remote store completes on them
        constexpr int P = E::kPairs;
        // h of row `row` (within the group) held in stage s, unit u, as fp32 pairs
        auto load_h = [&](uint32_t s, int row, uint32_t u, f2x* f) {
            const uint4* xs = c.ptr<const uint4>(stage0 + s * stage_bytes);
            const uint32_t idx = (uint32_t)row * units + u;
            E::unpack(xs[idx], f);
            if (RES) {
                f2x r[P];
                E::unpack(xs[(size_t)kR * units + idx], r);
#pragma unroll
                for (int e = 0; e < P; ++e) f[e] = f2_add(f[e], r[e]);
                E::unpack(E::pack(f), f);   // h rounded to the element type (the pre-norm output)
            }
        };
        if (warp >= kNormWarps) {
            // ------------------------------------------------------------ sum warps: rows 4v..4v+3
            const uint32_t v = warp - kNormWarps;
            uint32_t s = 0, ph = 0, set = 0;   // stage, its full parity, slot set of group j
            for (long long j = 0; j < iters; ++j) {
                c.deadline = globaltimer() + c.wait_limit;
                wait_par(c, kFull + (int)s, ph);
                const long long row0 = group_of(j) * kR + (long long)v * kRowsPerSs;
                float ss[kRowsPerSs];
#pragma unroll
                for (int k = 0; k < kRowsPerSs; ++k) {
                    f2x acc = 0ull;
                    if (row0 + k < hi) {
#pragma unroll
                        for (int q = 0; q < UPL; ++q) {
                            const uint32_t u = lane + 32u * q;
                            if (u < units) {
                                f2x f[P];
                                load_h(s, (int)(v * kRowsPerSs) + k, u, f);
#pragma unroll
                                for (int e = 0; e < P; ++e) acc = f2_fma(f[e], f[e], acc);
                            }
                        }
                    }
                    const float2 a2 = f2_split(acc);
                    ss[k] = a2.x + a2.y;
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int k = 0; k < kRowsPerSs; ++k) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], off);
                if (v == 0 && lane == 0) dsb::arm(c, kSum + (int)set, (uint32_t)N * kR * 4u);
                if (lane < (uint32_t)N) {   // lane q stores the 4 partials into CTA q
                    const uint32_t dst = slots + ((set * N + c.rank) * kR + v * kRowsPerSs) * 4u;
                    const uint32_t rd = mapa(c.sa + dst, lane), rbar = mapa(c.bar(kSum + (int)set), lane);
                    asm volatile(
                        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1,%2,%3,%4}, [%5];" ::"r"(rd),
                        "f"(ss[0]), "f"(ss[1]), "f"(ss[2]), "f"(ss[3]), "r"(rbar)
                        : "memory");
                }
                if (++s == nst) s = 0, ph ^= 1u;
                if (++set == nsets) set = 0;
            }
        } else {
            // ------------------------------------------------------------ normalising warps: rows 2w, 2w+1
            wait_par(c, kWBar, 0);
            const uint4* wp = c.ptr<const uint4>(woff);
            const float inv_hidden = 1.0f / (float)a.hidden;
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
            uint32_t s = 0, ph = 0, set = 0, sph = 0;   // stage and its full parity, slot set and its parity
            for (long long i = 0; i < iters; ++i) {
                c.deadline = globaltimer() + c.wait_limit;
                wait_par(c, kSum + (int)set, sph);
                wait_par(c, kFull + (int)s, ph);   // completed already (the own sum warps waited on it); makes
                                                   // the bulk-copied rows visible to this warp
                const long long row0 = group_of(i) * kR + (long long)warp * kRowsPerWarp;
                // the N partials of my two rows: lane q < N loads CTA q's pair, a butterfly over N lanes sums them
                float2 part = make_float2(0.f, 0.f);
                if (lane < (uint32_t)N)
                    part = *c.ptr<const float2>(slots + ((set * N + lane) * kR + warp * kRowsPerWarp) * 4u);
#pragma unroll
                for (int off = N / 2; off > 0; off >>= 1) {
                    part.x += __shfl_xor_sync(0xffffffffu, part.x, off);
                    part.y += __shfl_xor_sync(0xffffffffu, part.y, off);
                }
                const float tot2[kRowsPerWarp] = {__shfl_sync(0xffffffffu, part.x, 0),
                                                  __shfl_sync(0xffffffffu, part.y, 0)};
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k) {
                    const long long row = row0 + k;
                    const float scale = rsqrtf(fmaf(tot2[k], inv_hidden, a.eps));
                    const f2x scale2 = f2_make(scale, scale);
                    if (row >= hi) continue;
                    uint4* yo = reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.y) + (size_t)row * row_bytes + col_off);
                    uint4* po = RES && a.pre != nullptr
                                    ? reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.pre) +
                                                               (size_t)row * row_bytes + col_off)
                                    : nullptr;
#pragma unroll
                    for (int q = 0; q < UPL; ++q) {
                        const uint32_t u = lane + 32u * q;
                        if (u < units) {
                            f2x f[P];
                            load_h(s, (int)(warp * kRowsPerWarp) + k, u, f);
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
                if (++s == nst) s = 0, ph ^= 1u;
                if (++set == nsets) set = 0, sph ^= 1u;
            }
        }
    }
    // No cluster barrier at the end: every remote store into this CTA (the partial sums of each group) completed
    // on a sum barrier its normalising warps waited for. A CTA whose wait gave up lingers instead, so partials
    // still in flight to it land before it exits.
    if (__syncthreads_or(c.dead ? 1 : 0)) {
        const unsigned long long until = globaltimer() + dsb::kSettleNs;
        while (globaltimer() < until) {
        }
    }
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

// 3-D tiled view of a [rows x hidden] row-major tensor: {ce, hidden/ce, rows}, box {ce, cps, kR}.
bool encode_rows(CUtensorMap* m, const void* base, bool bf16, long long rows, int hidden, int ce, int cps) {
    const cuuint64_t eb = bf16 ? 2 : 4;
    const cuuint64_t dims[3] = {(cuuint64_t)ce, (cuuint64_t)(hidden / ce), (cuuint64_t)rows};
    const cuuint64_t strides[2] = {(cuuint64_t)ce * eb, (cuuint64_t)hidden * eb};
    const cuuint32_t box[3] = {(cuuint32_t)ce, (cuuint32_t)cps, (cuuint32_t)kR};
    return dsb_tmap::encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base,
                            dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

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
    if (rows > 0x7fffffffLL) return DSMEM_ERR_INVALID_ARGUMENT;   // TMA row coordinates are 32-bit
    const bool has_res = res != nullptr;
    // TMA chunk: the widest divisor of the slice's elements within the 256-element box limit whose bytes are
    // a multiple of 16 (16 bytes always qualifies: the slice is a multiple of 16 bytes)
    const int slice_elems = (int)(slice / eb);
    int ce = std::min(slice_elems, 256);
    while (slice_elems % ce != 0 || ((size_t)ce * eb) % 16 != 0) --ce;
    const int cps = slice_elems / ce;
    const uint32_t units = (uint32_t)(slice / 16);
    const int upl = units <= 32 ? 1 : units <= 64 ? 2 : 4;
    // Ring depth: the deepest (<= kMaxStages) that still lets kCtasPerSm CTAs share an SM (228 KiB of shared
    // memory, 1 KiB reserved per CTA), else the deepest that fits one CTA; at least 2.
    auto bytes = [&](int st) { return rms_smem(n, (uint32_t)slice, has_res, st, rms_sets(st)); };
    auto per_sm = [&](int st) { return (int)(kSmemPerSm / (bytes(st) + 1024u)); };
    int stages = kMaxStages;
    while (stages > 2 && per_sm(stages) < kCtasPerSm) --stages;
    if (per_sm(stages) < kCtasPerSm) {
        stages = kMaxStages;
        while (stages > 2 && bytes(stages) > dsb::kSmemLimit) --stages;
    }
    const int sets = rms_sets(stages);
    const uint32_t smem = bytes(stages);
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
        if (dsb_attr::ensure_smem(fn, dev, smem, n > 8) != cudaSuccess) return DSMEM_ERR_CUDA;
        const RmsKey key{fn, dev, smem};
        auto it = g_occ.find(key);
        if (it == g_occ.end()) {
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
    if (!encode_rows(&a.tmx, x, dtype == DSMEM_BF16, rows, hidden, ce, cps)) return DSMEM_ERR_CUDA;
    if (has_res && !encode_rows(&a.tmr, res, dtype == DSMEM_BF16, rows, hidden, ce, cps)) return DSMEM_ERR_CUDA;
    a.chunks_per_slice = cps;
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
    a.sets = sets;
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

