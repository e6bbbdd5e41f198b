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

// The epoch of a call: one past the last completed call's, never 0, so that no signal or LL word still at
// its initial zero matches a call (after 2^32 - 1 calls the epochs repeat). The word was stored by an
// earlier kernel of this rank's stream, so a relaxed load at GPU scope sees it.
__device__ __forceinline__ unsigned next_epoch(const unsigned* last) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(last) : "memory");
    const unsigned e = v + 1u;
    return e != 0u ? e : 1u;
}

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

// The indices of a warp's part of one group: rows row0 and row0 + 1, 16-byte units lane + 32 q of the CTA's
// column slice, as unit indices into the [rows x hidden] tensor.
template <int UPL>
struct GroupIdx {
    bool ok[kRowsPerWarp][UPL];
    long long idx[kRowsPerWarp][UPL];
    __device__ __forceinline__ GroupIdx(long long row0, long long hi, long long row_u4, long long col_u4,
                                        uint32_t units, uint32_t lane) {
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
            for (int q = 0; q < UPL; ++q) {
                const uint32_t u = lane + 32u * q;
                ok[k][q] = row0 + k < hi && u < units;
                idx[k][q] = (row0 + k) * row_u4 + col_u4 + u;
            }
    }
};

// Adds unit v (operand number `p` of the rank-order sum) into acc: operand 0 initialises it, so every
// kernel sums the ranks as ((x0 + x1) + x2) + ... in fp32.
__device__ __forceinline__ void accumulate(f2x* acc, uint4 v, int p) {
    using E = RmsElem<__nv_bfloat16>;
    if (p == 0) {
        E::unpack(v, acc);
    } else {
        f2x t[E::kPairs];
        E::unpack(v, t);
#pragma unroll
        for (int e = 0; e < E::kPairs; ++e) acc[e] = f2_add(acc[e], t[e]);
    }
}

// The normalisation half of a group, shared by both kernels (so their results are the same bits):
// residual add, h rounded to bf16 as the unfused AllReduce would give it, each row's sum of squares over
// the cluster (replicated st.async push of the warp's two partials into slot set `set` of every CTA;
// rmsnorm_lamport...hpcops.cu:153-169), the scale, the weight, and each output unit handed to
// store(unit index, value). The set of group i is rewritten for group i + kSets; a writer sends group g
// only after it normalised g - 1, which needed the owner's partials of g - 1, sent after the owner
// finished reading set g - 2.
template <int N, int UPL, bool kWReg, class Store>
__device__ __forceinline__ void normalise_group(dsb::Ctx& c, f2x (&acc)[kRowsPerWarp][UPL][4], const GroupIdx<UPL>& g,
                                                long long row0, long long hi, int set, const uint4* res,
                                                const uint4* w, const f2x (&wr)[kWReg ? UPL : 1][4],
                                                long long col_u4, uint32_t units, float eps, float inv_hidden,
                                                Store store) {
    using E = RmsElem<__nv_bfloat16>;
    constexpr int P = E::kPairs;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    uint4 h[kRowsPerWarp][UPL];
    float ss[kRowsPerWarp];
#pragma unroll
    for (int k = 0; k < kRowsPerWarp; ++k) {
        f2x sacc = 0ull;
#pragma unroll
        for (int q = 0; q < UPL; ++q) {
            if (res != nullptr && g.ok[k][q]) {
                f2x t[P];
                E::unpack(res[g.idx[k][q]], t);
#pragma unroll
                for (int e = 0; e < P; ++e) acc[k][q][e] = f2_add(acc[k][q][e], t[e]);
            }
            h[k][q] = E::pack(acc[k][q]);
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
        const float scale = rsqrtf(fmaf(tot[k], inv_hidden, eps));
        const f2x scale2 = f2_make(scale, scale);
        if (row0 + k >= hi) continue;
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
                    E::unpack(__ldg(w + col_u4 + u), wv);
#pragma unroll
                    for (int e = 0; e < P; ++e) f[e] = f2_mul(f2_mul(f[e], scale2), wv[e]);
                }
                store(g.idx[k][q], E::pack(f));
            }
        }
    }
}

// The weight units of the CTA's slice as fp32 pairs in registers, when a lane holds at most 2 of them.
template <int UPL, bool kWReg>
__device__ __forceinline__ void load_weights(f2x (&wr)[kWReg ? UPL : 1][4], const uint4* w, long long col_u4,
                                             uint32_t units, uint32_t lane) {
    if constexpr (kWReg) {
#pragma unroll
        for (int q = 0; q < UPL; ++q) {
            const uint32_t u = lane + 32u * q;
            if (u < units) RmsElem<__nv_bfloat16>::unpack(__ldg(w + col_u4 + u), wr[q]);
        }
    }
}

template <int N, int TP, int UPL>
__global__ void __launch_bounds__(kThreadsTp, (UPL >= 4 ? 1 : 2)) tp_allreduce_rmsnorm_kernel(const TpArgs a) {
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
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
        epoch = next_epoch(a.sig[a.rank] + kSigEpoch);
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
    f2x wr[kWReg ? UPL : 1][4];
    load_weights<UPL, kWReg>(wr, a.w, col_u4, units, lane);

    for (long long i = 0; i < iters; ++i) {
        c.deadline = globaltimer() + c.wait_limit;
        const long long row0 = lo + i * kR + (long long)warp * kRowsPerWarp;
        const GroupIdx<UPL> g(row0, hi, row_u4, col_u4, units, lane);
        // Sum over the ranks in rank order. The group's loads from PB ranks at a time are all issued before
        // any is used, so a lane keeps PB * 2 * UPL 16-byte peer loads in flight.
        constexpr int PB_MAX = UPL >= 4 ? 1 : (UPL == 2 ? 2 : 4);
        constexpr int PB = TP < PB_MAX ? TP : PB_MAX;   // a divisor of TP: ranks p0 + pp stay below TP
        static_assert(TP % PB == 0, "rank batches must tile the TP ranks");
        f2x acc[kRowsPerWarp][UPL][4];
#pragma unroll
        for (int p0 = 0; p0 < TP; p0 += PB) {
            uint4 v[PB][kRowsPerWarp][UPL];
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q)
                        v[pp][k][q] = g.ok[k][q] ? a.x[p0 + pp][g.idx[k][q]] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q) accumulate(acc[k][q], v[pp][k][q], p0 + pp);
        }
        normalise_group<N, UPL, kWReg>(c, acc, g, row0, hi, (int)(i & (kSets - 1)), a.res, a.w, wr, col_u4, units,
                                       a.eps, inv_hidden, [&](long long u, uint4 yv) {
#pragma unroll
                                           for (int p = 0; p < TP; ++p) a.y[p][u] = yv;   // all-gather: every rank's y
                                       });
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

// ------------------------------------------------------------------------------- one-shot (small T)
// Every rank pushes its whole x into every peer's LL region and then reduces and normalises ALL rows
// itself from what it received, writing only its own y: one trip over NVLink instead of the two-shot's
// reduce-scatter, all-gather and the flag round trips around them; (TP - 1) * rows * hidden * 4 bytes
// leave each rank (the LL words double the data).
//
// LL words (the low-latency protocol of NCCL's small collectives): each 8-byte word carries 4 bytes of x
// in its low half and the call's epoch in its high half, stored and loaded as 64-bit elements, which are
// single-copy atomic; a receiver polls its own memory until every word's epoch is the call's, with no
// flag, fence or round trip. The region of each rank holds two buffers (epoch & 1) of kMaxTp sender slots:
// a rank writes buffer b for call e + 2 only after its call e + 1 received this peer's data of e + 1,
// which the peer sent after its call e (the last reader of buffer b) had ended.
constexpr int kLLBufs = 2;
constexpr size_t kLLSlotMax = size_t(4) << 20;   // bytes of one sender's slot: rows * hidden * 4 at most
constexpr int kPushUnroll = 4;

struct OsArgs {
    const uint4* x;             // this rank's x [rows x hidden]
    uint4* y;                   // this rank's y
    unsigned char* ll[kMaxTp];  // LL region of every rank (buffer 0, slot 0)
    unsigned* sig;              // this rank's signal words; nullptr when emulating (epoch below)
    const uint4* res;           // residual (nullable): the same tensor on every rank
    const uint4* w;
    unsigned* err;
    unsigned long long wait_limit_ns;
    unsigned long long ll_slot; // bytes of one sender slot
    long long rows;
    int hidden;
    float eps;
    uint32_t slice_bytes;
    uint32_t smem_bytes;
    int rank;
    int phases;                 // bit 0: push x to the peers; bit 1: reduce, normalise and store y
    unsigned epoch;             // emulation only: the call's epoch
};

__device__ __forceinline__ void st_ll(unsigned char* p, unsigned long long lo, unsigned long long hi) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(lo), "l"(hi) : "memory");
}
__device__ __forceinline__ void ld_ll(const unsigned char* p, unsigned long long& lo, unsigned long long& hi) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "l"(p) : "memory");
}
__device__ __forceinline__ bool ll_ready(unsigned long long w0, unsigned long long w1, unsigned long long w2,
                                         unsigned long long w3, unsigned epoch) {
    return (unsigned)(w0 >> 32) == epoch && (unsigned)(w1 >> 32) == epoch && (unsigned)(w2 >> 32) == epoch &&
           (unsigned)(w3 >> 32) == epoch;
}
// One CTA per SM at every width (the one-shot serves small tensors; the registers go to the unit batch).
template <int N, int TP, int UPL>
__global__ void __launch_bounds__(kThreadsTp, 1) tp_oneshot_kernel(const OsArgs a) {
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t units = a.slice_bytes >> 4;
    const long long row_u4 = a.hidden / 8;
    const long long col_u4 = (long long)c.rank * units;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSets; ++s) mbar_init(c.bar(s), 1);
        fence_mbar_init();
    }
    // the cluster barrier that orders the slot barriers' initialisation before any remote st.async: arrived
    // here, waited for just before this CTA's first push of partials (it overlaps the push and the poll)
    if (a.phases & 2) cluster_arrive_relaxed();

    // ---- push: this rank's x into slot [rank] of buffer `buf` of every peer, flat over the whole grid, 8 bytes
    // of x (two LL words, one 16-byte store) per thread and step, so that a warp's store instruction covers 512
    // contiguous bytes of the peer's slot (LL bytes [16 h, 16 h + 16) carry x bytes [8 h, 8 h + 8)). The first x
    // load is issued before the epoch load, so the two latencies overlap; every thread reads the epoch itself
    // (one past the last completed call's: the last CTA of each call stores it; stream-ordered).
    const long long total = a.rows * row_u4 * 2;   // 8-byte halves of 16-byte units
    const long long stride = (long long)gridDim.x * kThreadsTp;
    const long long g0 = (long long)blockIdx.x * kThreadsTp + threadIdx.x;
    const uint2* xh = reinterpret_cast<const uint2*>(a.x);
    uint2 v0 = make_uint2(0u, 0u);   // the thread's first half (the grid gives most threads at most a few)
    if ((a.phases & 1) && g0 < total) v0 = __ldg(xh + g0);
    const unsigned epoch = a.sig != nullptr ? next_epoch(a.sig + kSigEpoch) : a.epoch;
    const size_t buf = epoch & 1u;
    if (a.phases & 1) {
        const unsigned long long f = (unsigned long long)epoch << 32;
        const size_t soff = (buf * kMaxTp + (size_t)a.rank) * a.ll_slot;
        for (long long gb = g0; gb < total; gb += kPushUnroll * stride) {
            uint2 v[kPushUnroll];
#pragma unroll
            for (int j = 0; j < kPushUnroll; ++j) {
                if (gb == g0 && j == 0) {
                    v[j] = v0;
                } else if (gb + j * stride < total) {
                    v[j] = __ldg(xh + gb + j * stride);
                }
            }
#pragma unroll
            for (int j = 0; j < kPushUnroll; ++j) {
                const long long gi = gb + j * stride;
                if (gi >= total) break;
#pragma unroll
                for (int p = 0; p < TP; ++p) {
                    if (p == a.rank) continue;
                    st_ll(a.ll[p] + soff + (size_t)gi * 16u, f | v[j].x, f | v[j].y);
                }
            }
        }
    }
    if (!(a.phases & 2)) return;   // emulation's push launch: no cluster barrier, no exchange

    // ---- every row, split evenly over the clusters
    const long long nclu = (long long)num_clusters(), cq = (long long)cluster_id();
    const long long lo = cq * a.rows / nclu, hi = (cq + 1) * a.rows / nclu;
    const long long iters = (hi - lo + kR - 1) / kR;
    const float inv_hidden = 1.0f / (float)a.hidden;
    constexpr bool kWReg = UPL <= 2;
    f2x wr[kWReg ? UPL : 1][4];
    load_weights<UPL, kWReg>(wr, a.w, col_u4, units, lane);
    const unsigned char* mine = a.ll[a.rank] + buf * kMaxTp * a.ll_slot;

    for (long long i = 0; i < iters; ++i) {
        c.deadline = globaltimer() + c.wait_limit;
        const long long row0 = lo + i * kR + (long long)warp * kRowsPerWarp;
        const GroupIdx<UPL> g(row0, hi, row_u4, col_u4, units, lane);
        f2x acc[kRowsPerWarp][UPL][4];
        // PB ranks' units at a time (at most 64 registers of units per lane, and fewer ranks than TP: a batch of
        // every rank let the compiler index the batch by this rank at run time, through local memory): every load
        // of the batch is issued before any is checked; the units not yet ready are read again together, one
        // round trip per pass for all of them, until they are or until the group's deadline; then they join the
        // sum in rank order
        constexpr int PB0 = UPL >= 4 ? 2 : (UPL == 2 ? 4 : 8);
        constexpr int PB = TP / 2 < 1 ? 1 : (TP / 2 < PB0 ? TP / 2 : PB0);   // a divisor of TP
        static_assert(TP % PB == 0, "rank batches must tile the TP ranks");
#pragma unroll
        for (int p0 = 0; p0 < TP; p0 += PB) {
            uint4 v[PB][kRowsPerWarp][UPL];
            bool ready[PB][kRowsPerWarp][UPL];
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q) {
                        const int p = p0 + pp;
                        ready[pp][k][q] = true;
                        if (!g.ok[k][q]) {
                            v[pp][k][q] = make_uint4(0u, 0u, 0u, 0u);
                        } else if (p == a.rank) {
                            v[pp][k][q] = __ldg(a.x + g.idx[k][q]);
                        } else {
                            const unsigned char* src = mine + (size_t)p * a.ll_slot + (size_t)g.idx[k][q] * 32u;
                            unsigned long long w0, w1, w2, w3;
                            ld_ll(src, w0, w1);
                            ld_ll(src + 16, w2, w3);
                            v[pp][k][q] = make_uint4((unsigned)w0, (unsigned)w1, (unsigned)w2, (unsigned)w3);
                            ready[pp][k][q] = ll_ready(w0, w1, w2, w3, epoch);
                        }
                    }
            bool all = true;
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q) all = all && ready[pp][k][q];
            while (!all && !c.dead) {
                if (globaltimer() > c.deadline) {
                    c.dead = true;
                    int first = p0;   // the lowest rank of the batch whose data did not arrive
#pragma unroll
                    for (int pp = PB - 1; pp >= 0; --pp)
#pragma unroll
                        for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                            for (int q = 0; q < UPL; ++q)
                                if (!ready[pp][k][q]) first = p0 + pp;
                    dsb::report_timeout(c, 0x70 + first);   // that rank's data did not arrive
                    break;
                }
                all = true;
#pragma unroll
                for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                    for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                        for (int q = 0; q < UPL; ++q)
                            if (!ready[pp][k][q]) {
                                const unsigned char* src =
                                    mine + (size_t)(p0 + pp) * a.ll_slot + (size_t)g.idx[k][q] * 32u;
                                unsigned long long w0, w1, w2, w3;
                                ld_ll(src, w0, w1);
                                ld_ll(src + 16, w2, w3);
                                v[pp][k][q] = make_uint4((unsigned)w0, (unsigned)w1, (unsigned)w2, (unsigned)w3);
                                ready[pp][k][q] = ll_ready(w0, w1, w2, w3, epoch);
                                all = all && ready[pp][k][q];
                            }
            }
#pragma unroll
            for (int pp = 0; pp < PB; ++pp)
#pragma unroll
                for (int k = 0; k < kRowsPerWarp; ++k)
#pragma unroll
                    for (int q = 0; q < UPL; ++q) accumulate(acc[k][q], v[pp][k][q], p0 + pp);
        }
        if (i == 0) cluster_wait();
        // The exchange may wait one more limit: a warp with no units in this group passes the poll at once and
        // waits here for partials that warps still polling send only after their poll ends (data, or its
        // deadline), so only a missing rank's poll reports the timeout.
        c.deadline += c.wait_limit;
        normalise_group<N, UPL, kWReg>(c, acc, g, row0, hi, (int)(i & (kSets - 1)), a.res, a.w, wr, col_u4, units,
                                       a.eps, inv_hidden, [&](long long u, uint4 yv) { a.y[u] = yv; });
    }
    if (iters == 0) cluster_wait();   // every arrive is matched (the same iters on every CTA of a cluster)
    // ---- exit: the last CTA stores the call's epoch for the next call (stream-ordered after this kernel)
    if (a.sig != nullptr) {
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned prev;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.sig + kSigCounter) : "memory");
            if (prev == gridDim.x - 1) {
                a.sig[kSigCounter] = 0u;
                a.sig[kSigEpoch] = epoch;
            }
        }
    }
    // No cluster barrier at the end: every remote write to this CTA (the partials of each group) completed on
    // a slot barrier this CTA waited for. A CTA whose wait gave up lingers instead, so partials still in flight
    // to it land before it exits.
    if (__syncthreads_or(c.dead ? 1 : 0)) {
        const unsigned long long until = globaltimer() + dsb::kSettleNs;
        while (globaltimer() < until) {
        }
    }
}

template <int N, int TP>
const void* tp_fn_upl(int upl, bool oneshot) {
    switch (upl) {
        case 1: return oneshot ? reinterpret_cast<const void*>(&tp_oneshot_kernel<N, TP, 1>)
                               : reinterpret_cast<const void*>(&tp_allreduce_rmsnorm_kernel<N, TP, 1>);
        case 2: return oneshot ? reinterpret_cast<const void*>(&tp_oneshot_kernel<N, TP, 2>)
                               : reinterpret_cast<const void*>(&tp_allreduce_rmsnorm_kernel<N, TP, 2>);
        case 4: return oneshot ? reinterpret_cast<const void*>(&tp_oneshot_kernel<N, TP, 4>)
                               : reinterpret_cast<const void*>(&tp_allreduce_rmsnorm_kernel<N, TP, 4>);
    }
    return nullptr;
}
template <int N>
const void* tp_fn_tp(int tp, int upl, bool oneshot) {
    switch (tp) {
        case 1: return tp_fn_upl<N, 1>(upl, oneshot);
        case 2: return tp_fn_upl<N, 2>(upl, oneshot);
        case 4: return tp_fn_upl<N, 4>(upl, oneshot);
        case 8: return tp_fn_upl<N, 8>(upl, oneshot);
    }
    return nullptr;
}
const void* tp_fn(int n, int tp, int upl, bool oneshot) {
    switch (n) {
        case 2: return tp_fn_tp<2>(tp, upl, oneshot);
        case 4: return tp_fn_tp<4>(tp, upl, oneshot);
        case 8: return tp_fn_tp<8>(tp, upl, oneshot);
        case 16: return tp_fn_tp<16>(tp, upl, oneshot);
    }
    return nullptr;
}

uint32_t tp_smem() { return kSlots + (uint32_t)kSets * 16u * kR * 4u; }   // slots sized for N <= 16

std::mutex g_tp_mu;

// The shape rules both kernels share: bf16, TP in {1,2,4,8}, cluster of 2-16 CTAs each owning a whole number
// of 16-byte units of a row (at most 4 per lane); returns the row slice in bytes and the units per lane.
dsmem_status tp_shape(dsmem_dtype dtype, int tp, int rank, int n, const void* w, long long rows, int hidden, float eps,
                      uint32_t* slice, int* upl) {
    if (dtype != DSMEM_BF16) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (!(tp == 1 || tp == 2 || tp == 4 || tp == 8) || rank < 0 || rank >= tp) return DSMEM_ERR_INVALID_ARGUMENT;
    if (!(n == 2 || n == 4 || n == 8 || n == 16)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (w == nullptr || rows < 0 || hidden <= 0 || !(eps >= 0.f)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (hidden % (8 * n) != 0) return DSMEM_ERR_ILLEGAL_CONFIG;   // whole 16-B units per CTA slice
    *slice = (uint32_t)(hidden / n) * 2u;
    const uint32_t units = *slice / 16u;
    if (units > 128u) return DSMEM_ERR_ILLEGAL_CONFIG;            // <= 4 units per lane
    *upl = units <= 32 ? 1 : units <= 64 ? 2 : 4;
    return DSMEM_OK;
}

// Launch configuration of kernel `fn` with cluster n; the resident clusters per GPU (cached per kernel and
// device: the attribute set-up and the occupancy query cost more than a launch).
dsmem_status tp_config(const void* fn, int n, cudaStream_t stream, cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr,
                       int* resident) {
    const uint32_t smem = tp_smem();
    cfg = {};
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreadsTp, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DSMEM_ERR_CUDA;
    static std::map<std::tuple<const void*, int, uint32_t>, int> occupancy;
    std::lock_guard<std::mutex> lock(g_tp_mu);
    if (dsb_attr::ensure_smem(fn, dev, (uint32_t)smem, n > 8, false) != cudaSuccess) return DSMEM_ERR_CUDA;
    auto it = occupancy.find({fn, dev, (uint32_t)smem});
    if (it != occupancy.end()) {
        *resident = it->second;
    } else {
        cfg.gridDim = dim3((unsigned)n, 1, 1);
        if (cudaOccupancyMaxActiveClusters(resident, fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
        occupancy[{fn, dev, (uint32_t)smem}] = *resident;
    }
    return *resident < 1 ? DSMEM_ERR_SMEM_LIMIT : DSMEM_OK;
}

// Shape checks and launch of the two-shot kernel for `tp` ranks (emulate: all buffers local, one launch).
dsmem_status tp_launch(const void* const* xs, void* const* ys, unsigned* const* sigs, unsigned* err, int tp,
                       int rank, int emulate, dsmem_dtype dtype, const void* residual,
                       const void* w, float eps, long long rows, int hidden, int cluster_size,
                       cudaStream_t stream, unsigned long long wait_limit_ns = 2000000000ull) {
    const int n = cluster_size;
    uint32_t slice = 0;
    int upl = 0;
    if (dsmem_status st = tp_shape(dtype, tp, rank, n, w, rows, hidden, eps, &slice, &upl); st != DSMEM_OK) return st;
    uintptr_t al = reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(residual);
    for (int p = 0; p < tp; ++p) {
        if (xs[p] == nullptr || ys[p] == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
        al |= reinterpret_cast<uintptr_t>(xs[p]) | reinterpret_cast<uintptr_t>(ys[p]);
    }
    if (al & 15u) return DSMEM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DSMEM_OK;
    const void* fn = tp_fn(n, tp, upl, false);
    if (fn == nullptr) return DSMEM_ERR_ILLEGAL_CONFIG;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    int resident = 0;
    if (dsmem_status st = tp_config(fn, n, stream, cfg, attr, &resident); st != DSMEM_OK) return st;
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
    a.smem_bytes = tp_smem();
    a.rank = rank;
    a.emulate = emulate;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

// Shape checks and launch of the one-shot kernel of rank `rank`: x and y are this rank's, lls[p] every rank's LL
// region; phases 3 on a real rank, 1 (push) or 2 (reduce) for the emulation's separate launches.
dsmem_status oneshot_launch(const void* x, void* y, unsigned char* const* lls, size_t ll_slot, unsigned* sig,
                            unsigned epoch, int phases, unsigned* err, int tp, int rank, dsmem_dtype dtype,
                            const void* residual, const void* w, float eps, long long rows, int hidden,
                            int cluster_size, cudaStream_t stream, unsigned long long wait_limit_ns) {
    const int n = cluster_size;
    uint32_t slice = 0;
    int upl = 0;
    if (dsmem_status st = tp_shape(dtype, tp, rank, n, w, rows, hidden, eps, &slice, &upl); st != DSMEM_OK) return st;
    if (x == nullptr || y == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    uintptr_t al = reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(residual) |
                   reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y);
    for (int p = 0; p < tp; ++p) {
        if (lls[p] == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
        al |= reinterpret_cast<uintptr_t>(lls[p]);
    }
    if ((al & 15u) || (ll_slot & 15u)) return DSMEM_ERR_INVALID_ARGUMENT;
    if ((size_t)rows * (size_t)hidden * 4u > ll_slot) return DSMEM_ERR_SCRATCH_LIMIT;
    if (rows == 0) return DSMEM_OK;
    const void* fn = tp_fn(n, tp, upl, true);
    if (fn == nullptr) return DSMEM_ERR_ILLEGAL_CONFIG;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    int resident = 0;
    if (dsmem_status st = tp_config(fn, n, stream, cfg, attr, &resident); st != DSMEM_OK) return st;
    // clusters for the row groups, or enough CTAs that each thread pushes one half unit (up to every resident
    // cluster: the push's remote stores go out at a limited rate per SM); every CTA resident (the exit
    // counter is passed by all of them)
    const long long total = rows * (long long)(hidden / 4);   // 8-byte halves pushed, one per thread
    const long long push_ctas = (total + kThreadsTp - 1) / kThreadsTp;
    const long long want = std::max<long long>((rows + kR - 1) / kR, (push_ctas + n - 1) / n);
    const long long clusters = std::max<long long>(1, std::min<long long>(want, resident));
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    OsArgs a{};
    a.x = static_cast<const uint4*>(x);
    a.y = static_cast<uint4*>(y);
    for (int p = 0; p < tp; ++p) a.ll[p] = lls[p];
    a.sig = sig;
    a.res = static_cast<const uint4*>(residual);
    a.w = static_cast<const uint4*>(w);
    a.err = err;
    a.wait_limit_ns = wait_limit_ns;
    a.ll_slot = ll_slot;
    a.rows = rows;
    a.hidden = hidden;
    a.eps = eps;
    a.slice_bytes = slice;
    a.smem_bytes = tp_smem();
    a.rank = rank;
    a.phases = phases;
    a.epoch = epoch;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

}  // namespace

// ------------------------------------------------------------------------------------------ TP context
namespace {
// Default one-shot limit on the LL bytes a rank sends, (tp - 1) * rows * hidden * 4: measured at hidden 8192,
// the one-shot is the faster form at 1 and 64 tokens on TP 2 (6 MiB at TP 4, where it still wins).
constexpr size_t kOneShotDefault = size_t(16) << 20;
size_t ll_offset(size_t capacity) { return kSignalBytes + 2 * capacity; }

// Error words of the one-GPU emulation entry points, one set per device (read by dsmem_tp_emulate_check).
dsmem_status emu_err(unsigned** out) {
    static unsigned* err[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_tp_mu);
    if (err[dev] == nullptr) {
        if (cudaMalloc(&err[dev], 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
        if (cudaMemset(err[dev], 0, 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
    }
    *out = err[dev];
    return DSMEM_OK;
}
}  // namespace

struct dsmem_tp_ctx {
    int device = 0;
    int rank = -1;
    int tp = 0;
    size_t capacity = 0;             // bytes of each of the x and y regions
    size_t ll_slot = 0;              // bytes of one sender slot of the LL region
    unsigned char* base = nullptr;   // this rank's buffer: [signals 4 KiB][x][y][LL: 2 buffers x kMaxTp slots]
    unsigned char* peer[kMaxTp] = {};
    unsigned long long wait_limit_ns = 2000000000ull;   // each cross-GPU flag wait of a call
    size_t oneshot_limit = kOneShotDefault;             // one-shot when (tp - 1) * rows * hidden * 4 <= this
};

extern "C" {

dsmem_status dsmem_tp_alloc(size_t capacity_bytes, dsmem_tp_t* ctx, void* ipc_handle) {
    if (ctx == nullptr || ipc_handle == nullptr || capacity_bytes == 0) return DSMEM_ERR_INVALID_ARGUMENT;
    *ctx = nullptr;
    auto* c = new dsmem_tp_ctx();
    c->capacity = (capacity_bytes + 255) & ~(size_t)255;
    c->ll_slot = std::min(2 * c->capacity, kLLSlotMax);   // rows * hidden * 4 of a tensor that fills x, or 4 MiB
    const size_t ll_bytes = (size_t)kLLBufs * kMaxTp * c->ll_slot;
    if (cudaGetDevice(&c->device) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&c->base), ll_offset(c->capacity) + ll_bytes) != cudaSuccess) {
        delete c;
        return DSMEM_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    // signal words and LL words start at 0: every call's epoch is at least 1
    if (cudaMemset(c->base, 0, kSignalBytes) != cudaSuccess ||
        cudaMemset(c->base + ll_offset(c->capacity), 0, ll_bytes) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, c->base) != cudaSuccess) {
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
    const size_t ll_bytes = bytes * 2;   // one sender slot: rows * hidden LL words of 8 bytes per 2 elements
    if (c->tp > 1 && ll_bytes <= c->ll_slot && (size_t)(c->tp - 1) * ll_bytes <= c->oneshot_limit) {
        // one-shot: reads x and writes y where they are (no copies), pushes x into the peers' LL regions
        unsigned char* lls[kMaxTp];
        for (int p = 0; p < c->tp; ++p) lls[p] = c->peer[p] + ll_offset(c->capacity);
        return oneshot_launch(x != nullptr ? x : xb, y != nullptr ? y : yb, lls, c->ll_slot,
                              reinterpret_cast<unsigned*>(c->base), 0u, 3, reinterpret_cast<unsigned*>(c->base) + kSigErr,
                              c->tp, c->rank, dtype, residual, w, eps, rows, hidden, cluster_size, s, c->wait_limit_ns);
    }
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
    unsigned* err = nullptr;
    if (dsmem_status st = emu_err(&err); st != DSMEM_OK) return st;
    return tp_launch(xs, ys, nullptr, err, tp, 0, 1, dtype, residual, w, eps, rows, hidden, cluster_size,
                     reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_tp_emulate_oneshot(int tp, const void* const* xs, void* const* ys, dsmem_dtype dtype,
                                      const void* residual, const void* w, float eps, long long rows, int hidden,
                                      int cluster_size, dsmem_stream_t stream) {
    if (xs == nullptr || ys == nullptr || !(tp == 1 || tp == 2 || tp == 4 || tp == 8) || rows < 0 || hidden <= 0)
        return DSMEM_ERR_INVALID_ARGUMENT;
    // Each virtual rank's LL region is one buffer of tp sender slots, all on this GPU; the pushes of every
    // rank are launched before any rank's reduction, so no launch waits for another one.
    static unsigned char* scratch[64] = {};
    static size_t scratch_bytes[64] = {};
    unsigned* err = nullptr;
    if (dsmem_status st = emu_err(&err); st != DSMEM_OK) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    const size_t slot = ((size_t)rows * (size_t)hidden * 4u + 255) & ~(size_t)255;
    const size_t need = std::max<size_t>(256, (size_t)tp * tp * slot);
    auto s = reinterpret_cast<cudaStream_t>(stream);
    {
        std::lock_guard<std::mutex> lock(g_tp_mu);
        if (scratch_bytes[dev] < need) {
            if (scratch[dev] != nullptr && cudaFree(scratch[dev]) != cudaSuccess) return DSMEM_ERR_CUDA;
            scratch[dev] = nullptr;
            scratch_bytes[dev] = 0;
            if (cudaMalloc(&scratch[dev], need) != cudaSuccess) return DSMEM_ERR_CUDA;
            scratch_bytes[dev] = need;
        }
    }
    // zeroed for every call, so no word of an earlier call carries this call's epoch (2: buffer 0)
    if (cudaMemsetAsync(scratch[dev], 0, need, s) != cudaSuccess) return DSMEM_ERR_CUDA;
    unsigned char* lls[kMaxTp] = {};
    for (int p = 0; p < tp; ++p) lls[p] = scratch[dev] + (size_t)p * tp * slot;
    for (int phase = 1; phase <= 2; ++phase)
        for (int r = 0; r < tp; ++r) {
            if (xs[r] == nullptr || ys[r] == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
            const dsmem_status st = oneshot_launch(xs[r], ys[r], lls, slot, nullptr, 2u, phase, err, tp, r, dtype,
                                                   residual, w, eps, rows, hidden, cluster_size, s, 2000000000ull);
            if (st != DSMEM_OK) return st;
        }
    return DSMEM_OK;
}

dsmem_status dsmem_tp_emulate_check(unsigned* error_bits, unsigned* detail) {
    unsigned* err = nullptr;
    if (dsmem_status st = emu_err(&err); st != DSMEM_OK) return st;
    unsigned v[4] = {};
    if (cudaMemcpy(v, err, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess || cudaMemset(err, 0, sizeof v) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    if (error_bits) *error_bits = v[0];
    if (detail) *detail = v[1];
    return (v[0] & DSMEM_ERRBIT_TIMEOUT) ? DSMEM_ERR_TIMEOUT : (v[0] & DSMEM_ERRBIT_BOUNDS) ? DSMEM_ERR_BOUNDS : DSMEM_OK;
}

dsmem_status dsmem_tp_set_oneshot_limit(dsmem_tp_t c, size_t bytes) {
    if (c == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    c->oneshot_limit = bytes;
    return DSMEM_OK;
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
