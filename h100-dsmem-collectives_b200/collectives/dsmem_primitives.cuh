// dsmem_primitives.cuh -- thread-block-cluster (DSMEM) primitive surface for B200 (sm_100a).
//
// Drop-in for the reference header collectives/dsmem_primitives.cuh: every name the reference's
// algorithm files and harness use (collectives/dsmem_primitives.cuh:40-245, defaults :250-258) exists
// here with the same signature and meaning, so collectives/harness/main.cu can include the
// <op>__<alg>__<src>.cu files of this directory unchanged. Differences, all deliberate:
//   * mbar_wait_parity() is bounded. The reference spins forever (:140-150); here a wait gives up
//     after DSMEM_WAIT_LIMIT_NS of %globaltimer time, records DSMEM_ERR_BIT_TIMEOUT in the
//     translation unit's `dsmem_wait_error` word and returns, so a mis-armed barrier shows up as a
//     wrong result instead of a hung GPU. barrier.cluster cannot time out; every kernel built on this
//     header therefore executes the same number of cluster barriers on every CTA, with no
//     data-dependent early exit.
//   * Extensions used by the B200 kernels: try-wait, deadline-bounded wait, mbarrier invalidate,
//     cp.reduce.async.bulk (element-wise add into a peer), one-CTA bulk global<->shared copies
//     (no cluster multicast anywhere: every bulk load names exactly one destination CTA),
//     %clusterid / %nclusterid for persistent multi-cluster kernels, and .acquire.cluster waits for
//     barriers that peers arrive on with plain remote arrivals.
//
// Vocabulary: rank b = %cluster_ctarank in [0, N); a "shared::cluster" address is a 32-bit address
// produced by mapa that names a byte in some CTA of the cluster; mbarrier phases complete when the
// pending-arrival count and the transaction-byte count both reach zero.
#pragma once
#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#ifndef DSMEM_WAIT_LIMIT_NS
#define DSMEM_WAIT_LIMIT_NS 1000000000ull   // 1 s of %globaltimer per mbarrier wait
#endif

namespace dsmem {

namespace cg = cooperative_groups;

// Error bits shared by device code and the C ABI (DSMEM_ERRBIT_* in include/dsmem_b200.h).
constexpr unsigned DSMEM_ERR_BIT_TIMEOUT = 1u;   // an mbarrier wait ran out of time
constexpr unsigned DSMEM_ERR_BIT_BOUNDS = 2u;    // a bulk copy / remote access failed its bounds check

// One word per translation unit; the harness-compatible kernels report timeouts here.
static __device__ unsigned dsmem_wait_error;

// ------------------------------------------------------------------ identity
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t v;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(v));
    return v;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t v;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(v));
    return v;
}
// Index of this cluster in the grid and number of clusters (x dimension; launches here are 1-D).
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t v;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(v));
    return v;
}
__device__ __forceinline__ uint32_t num_clusters() {
    uint32_t v;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(v));
    return v;
}
__device__ __forceinline__ uint32_t smid() {
    uint32_t v;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(v));
    return v;
}
// Nanosecond timer that all SMs share (clock64 is per SM).
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long v;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(v));
    return v;
}

// ---------------------------------------------------------------- addressing
template <typename T>
__device__ __forceinline__ uint32_t smem_u32(const T* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Same shared-memory offset, but inside CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t smem_addr, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr), "r"(rank));
    return out;
}
// Generic pointer into CTA `rank`'s copy of a shared variable (usable by plain loads, stores, atomics).
template <typename T>
__device__ __forceinline__ T* map_ptr(T* local, uint32_t rank) {
    return cg::this_cluster().map_shared_rank(local, rank);
}

// ------------------------------------------------------- remote loads/stores
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t caddr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(caddr) : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t caddr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(caddr), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t caddr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(caddr) : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t caddr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(caddr), "f"(v) : "memory");
}
__device__ __forceinline__ uint16_t ld_cluster_u16(uint32_t caddr) {
    uint16_t v;
    asm volatile("ld.shared::cluster.u16 %0, [%1];" : "=h"(v) : "r"(caddr) : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster_u16(uint32_t caddr, uint16_t v) {
    asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(caddr), "h"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_cluster_v4(uint32_t caddr) {
    uint4 v;
    asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(caddr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t caddr, uint4 v) {
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(caddr), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}
// Fire-and-forget remote reductions (the destination SM's shared-memory atomic unit does the add).
__device__ __forceinline__ void red_cluster_add_f32(uint32_t caddr, float v) {
    asm volatile("red.shared::cluster.add.f32 [%0], %1;" ::"r"(caddr), "f"(v) : "memory");
}
__device__ __forceinline__ void red_cluster_add_u32(uint32_t caddr, uint32_t v) {
    asm volatile("red.shared::cluster.add.u32 [%0], %1;" ::"r"(caddr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_cas_cluster_b32(uint32_t caddr, uint32_t expected, uint32_t desired) {
    uint32_t old;
    asm volatile("atom.shared::cluster.cas.b32 %0, [%1], %2, %3;"
                 : "=r"(old)
                 : "r"(caddr), "r"(expected), "r"(desired)
                 : "memory");
    return old;
}
// Order this thread's generic-proxy shared-memory accesses against the async proxy (bulk copies,
// st.async). Needed between writing a buffer with ordinary stores and handing it to a bulk copy.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
}

// ------------------------------------------------------------------ mbarrier
// `bar` is the 32-bit shared::cta address of an 8-byte aligned 64-bit mbarrier object.
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t arrival_count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(arrival_count) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint32_t bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// Publish mbarrier.init results to the whole cluster (before any peer arrives or completes bytes).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Arrive + expect `bytes` on the barrier at the same offset in CTA `rank`.
__device__ __forceinline__ void mbar_arrive_expect_tx_remote(uint32_t bar, uint32_t rank, uint32_t bytes) {
    const uint32_t remote = mapa(bar, rank);
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(remote),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar, uint32_t rank) {
    const uint32_t remote = mapa(bar, rank);
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// Arrives without release semantics (PTX .relaxed): they order nothing before them, so they do not wait for
// this thread's outstanding global stores. For a consumer that only signals "my reads of this buffer are done":
// those reads have returned their values before the arrive issues.
__device__ __forceinline__ void mbar_arrive_relaxed(uint32_t bar) {
    asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t bar, uint32_t rank) {
    const uint32_t remote = mapa(bar, rank);
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// One probe of the phase with parity `parity`; true once it has completed. Acquire at cluster
// scope, so plain remote stores released by a peer's arrive are visible after success.
__device__ __forceinline__ bool mbar_try_wait_parity(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
// As mbar_try_wait_parity, but the thread may be suspended in hardware for up to `suspend_ns` while the
// phase is incomplete (it resumes as soon as the phase completes), so a waiting warp stops competing for
// issue slots with the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_parity_suspend(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(suspend_ns)
        : "memory");
    return done != 0;
}
// Wait until the phase completes or %globaltimer passes `deadline_ns`; false on time-out. Each probe may
// suspend the thread for up to 100 us, so the limit is honoured to within that.
#ifndef DSMEM_WAIT_SUSPEND_NS
#define DSMEM_WAIT_SUSPEND_NS 100000u
#endif
constexpr uint32_t kWaitSuspendNs = DSMEM_WAIT_SUSPEND_NS;   // 0: probe without a suspend hint
__device__ __forceinline__ bool mbar_wait_parity_until(uint32_t bar, uint32_t parity, unsigned long long deadline_ns) {
    while (kWaitSuspendNs != 0u ? !mbar_try_wait_parity_suspend(bar, parity, kWaitSuspendNs)
                                : !mbar_try_wait_parity(bar, parity)) {
        if (globaltimer() > deadline_ns) return false;
    }
    return true;
}
// Reference-compatible wait (same signature). Bounded: see the header comment.
__device__ __forceinline__ void mbar_wait_parity(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait_parity(bar, parity)) return;
    if (!mbar_wait_parity_until(bar, parity, globaltimer() + DSMEM_WAIT_LIMIT_NS))
        atomicOr(&dsmem_wait_error, DSMEM_ERR_BIT_TIMEOUT);
}

// ------------------------------------------------------------ bulk transfers
// One thread: copy `bytes` (multiple of 16, both ends 16-B aligned) from local shared memory `src`
// into CTA `dst_rank`'s shared memory at the offset of local address `dst`, completing `bytes`
// transaction bytes on that CTA's mbarrier at the offset of local `dst_bar`.
__device__ __forceinline__ void bulk_push(uint32_t dst_rank, uint32_t dst, uint32_t src, uint32_t bytes,
                                          uint32_t dst_bar) {
    const uint32_t rdst = mapa(dst, dst_rank);
    const uint32_t rbar = mapa(dst_bar, dst_rank);
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(rdst),
        "r"(src), "r"(bytes), "r"(rbar)
        : "memory");
}
// As bulk_push, but the destination receives dst[i] += src[i]; the element type is in the function
// name. The add happens in the destination SM.
__device__ __forceinline__ void bulk_push_add_f32(uint32_t dst_rank, uint32_t dst, uint32_t src, uint32_t bytes,
                                                  uint32_t dst_bar) {
    const uint32_t rdst = mapa(dst, dst_rank);
    const uint32_t rbar = mapa(dst_bar, dst_rank);
    asm volatile(
        "cp.reduce.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes.add.f32 [%0], [%1], %2, [%3];" ::
            "r"(rdst),
        "r"(src), "r"(bytes), "r"(rbar)
        : "memory");
}
__device__ __forceinline__ void bulk_push_add_u32(uint32_t dst_rank, uint32_t dst, uint32_t src, uint32_t bytes,
                                                  uint32_t dst_bar) {
    const uint32_t rdst = mapa(dst, dst_rank);
    const uint32_t rbar = mapa(dst_bar, dst_rank);
    asm volatile(
        "cp.reduce.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes.add.u32 [%0], [%1], %2, [%3];" ::
            "r"(rdst),
        "r"(src), "r"(bytes), "r"(rbar)
        : "memory");
}
// 16-byte asynchronous remote store that completes 16 bytes on the destination mbarrier.
__device__ __forceinline__ void st_async_v4(uint32_t dst_rank, uint32_t dst, uint4 v, uint32_t dst_bar) {
    const uint32_t rdst = mapa(dst, dst_rank);
    const uint32_t rbar = mapa(dst_bar, dst_rank);
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1,%2,%3,%4}, [%5];" ::"r"(rdst),
        "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
        : "memory");
}
// Bulk copy global -> this CTA's shared memory (no multicast), completing on a local mbarrier.
__device__ __forceinline__ void bulk_load_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// Tiled TMA load of one box of a 3-D tensor map (global -> this CTA's shared memory, no multicast),
// completing on a local mbarrier. `tmap` is the generic address of a __grid_constant__ CUtensorMap;
// x * element size must be a multiple of 16 bytes. Box elements outside the tensor read as zero and
// still count toward the transaction bytes.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
// 4-D form of the tiled TMA load above (same rules).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int x, int y, int z, int w, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
        : "memory");
}
// 2-D form of the tiled TMA load above (same rules).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// Bulk copy this CTA's shared memory -> global, tracked by the issuing thread's bulk groups.
__device__ __forceinline__ void bulk_store_s2g(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most 0 committed groups still READ shared memory (the source may be reused).
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until every committed group has completed (global writes done).
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ------------------------------------------------------------ cluster barrier
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
    cluster_arrive();
    cluster_wait();
}

// ---------------------------------------------------------------- reductions
template <typename T>
__device__ __forceinline__ T lowest_value();
template <>
__device__ __forceinline__ float lowest_value<float>() {
    return __int_as_float(0xff800000);
}
template <>
__device__ __forceinline__ double lowest_value<double>() {
    return __longlong_as_double(0xfff0000000000000ll);
}
template <>
__device__ __forceinline__ int lowest_value<int>() {
    return (int)0x80000000;
}
template <>
__device__ __forceinline__ unsigned lowest_value<unsigned>() {
    return 0u;
}
template <>
__device__ __forceinline__ __half lowest_value<__half>() {
    return __ushort_as_half((unsigned short)0xfc00u);
}
template <>
__device__ __forceinline__ __nv_bfloat16 lowest_value<__nv_bfloat16>() {
    return __ushort_as_bfloat16((unsigned short)0xff80u);
}

struct Sum {
    template <typename T>
    __device__ __forceinline__ T operator()(T a, T b) const { return a + b; }
    template <typename T>
    static __device__ __forceinline__ T identity() { return T(0); }
};
struct Max {
    template <typename T>
    __device__ __forceinline__ T operator()(T a, T b) const { return a < b ? b : a; }
    template <typename T>
    static __device__ __forceinline__ T identity() { return lowest_value<T>(); }
};

// ---------------------------------------------------------- harness contract
// Kernel contract of every <op>__<alg>__<src>.cu (one cluster per launch, gridDim.x == CLUSTER_N):
//   __global__ void __cluster_dims__(CLUSTER_N,1,1)
//   collective_kernel(const ELEM_T* in, ELEM_T* out, unsigned long long* ts, unsigned* smid);
// Per-rank layouts (b = rank, M = MSG_ELEMS):
//   allreduce     in[b*M + i]            -> out[b*M + i]          = sum_r in[r*M + i]
//   allgather     in[b*M + i]            -> out[b*N*M + r*M + i]  = in[r*M + i]
//   reducescatter in[b*N*M + j*M + i]    -> out[b*M + i]          = sum_r in[r*N*M + b*M + i]
//   alltoall      in[b*N*M + j*M + i]    -> out[b*N*M + r*M + i]  = in[r*N*M + b*M + i]
// Stamps: ts[b*kStamps + 0] entry, +1 exit, +2+r end of round r (%globaltimer ns); smid[b] = SM.
// Shared memory: `struct CollectiveSmem` taken from the dynamic window; size passed at launch.
constexpr int kStamps = 32;

extern __shared__ __align__(128) unsigned char dyn_smem_raw[];
template <class S>
__device__ __forceinline__ S& dyn_smem() {
    return *reinterpret_cast<S*>(dyn_smem_raw);
}

struct Stamps {
    unsigned long long* base;   // &ts[rank * kStamps], or nullptr for no stamps
    __device__ __forceinline__ void mark(int i) const {
        if (base != nullptr && threadIdx.x == 0) base[i] = globaltimer();
    }
    __device__ __forceinline__ void round(int r) const {
        if (r + 2 < kStamps) mark(2 + r);
    }
};

template <typename T, int M>
__device__ __forceinline__ void load_block(T* smem, const T* g) {
    for (int i = threadIdx.x; i < M; i += blockDim.x) smem[i] = g[i];
    __syncthreads();
}
template <typename T, int M>
__device__ __forceinline__ void store_block(T* g, const T* smem) {
    __syncthreads();
    for (int i = threadIdx.x; i < M; i += blockDim.x) g[i] = smem[i];
}

}  // namespace dsmem

// Compile-time knobs of the harness build (override with -D).
#ifndef CLUSTER_N
#define CLUSTER_N 4
#endif
#ifndef MSG_ELEMS
#define MSG_ELEMS 1024
#endif
#ifndef ELEM_T
#define ELEM_T float
#endif
