// ext_ceilings.cu -- SM-to-SM (DSMEM) bandwidth ceiling of this GPU, the denominator of the shared::cluster
// roofline fractions.
//
// Method of the reference's roofline/harness/ceilings/src/dsmem_bw.cu:1-40 (written anew for sm_100a):
// every SM that can host a CTA of a cluster of size CS gets one CTA (max active clusters at ~200 KB of
// shared memory, 1024 threads), and every CTA streams a 96 KiB tile per pass to / from its ring neighbour
// (rank r -> (r+1) mod CS), in one of two directions of use (plus a fan-out mode, below):
//   pull  16-byte ld.shared::cluster.v4 from the neighbour's source tile by all threads;
//   push  one thread per CTA issues cp.async.bulk shared::cta -> shared::cluster copies of 16 KiB into the
//         neighbour's destination tile, completing on one mbarrier per pass in the neighbour, which waits.
// The host times launches with 4..32 passes; GPU-wide bandwidth = 1 / slope of time over bytes, which
// removes the fixed cost of a launch (tile init, cluster barriers, launch overhead).
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"

namespace {

constexpr int kMaxPasses = 32;
constexpr uint32_t kBars = 256;                     // 32 mbarriers
constexpr uint32_t kSrc = kBars;

// Two shapes: the reference's (96 KiB tiles, 1024 threads, ~196 KiB: one CTA per SM) and a small one
// (24 KiB tiles, 256 threads, ~52 KiB: four CTAs per SM), which lets clusters of 8 and 16 use the SMs
// that one-CTA-per-SM placement leaves idle in every GPC.
template <uint32_t TILE>
struct Shape {
    static constexpr uint32_t kTile = TILE;
    static constexpr uint32_t kChunk = TILE >= 96u * 1024u ? 16u * 1024u : 8u * 1024u;
    static constexpr uint32_t kDst = kSrc + TILE;
    static constexpr uint32_t kSmem = kDst + TILE + 4096;
    // all-peers mode: bytes per peer per pass (a multiple of 1 KiB, at most 8 KiB, all peers within the tile)
    static __host__ __device__ constexpr uint32_t fan_chunk(uint32_t cs) {
        return (TILE / (cs - 1) / 1024u) * 1024u < 8192u ? (TILE / (cs - 1) / 1024u) * 1024u : 8192u;
    }
};

template <int MODE, uint32_t TILE, int THREADS>
__global__ void __launch_bounds__(THREADS, 1) dsmem_bw_kernel(int passes, unsigned* err, unsigned* sink,
                                                              unsigned long long limit) {
    using namespace dsmem;
    using Sh = Shape<TILE>;
    constexpr uint32_t kTile = Sh::kTile, kChunk = Sh::kChunk, kDst = Sh::kDst;
    const uint32_t sa = smem_u32(dyn_smem_raw);
    const uint32_t rank = cluster_rank(), cs = cluster_size(), peer = (rank + 1) % cs;
    uint4* src = reinterpret_cast<uint4*>(dyn_smem_raw + kSrc);
    for (uint32_t i = threadIdx.x; i < kTile / 16; i += blockDim.x) src[i] = make_uint4(i, rank, i ^ 0x5a5a5a5au, ~i);
    // mode 2 (all peers): per pass every CTA sends one chunk of q bytes to each of its cs-1 peers
    const uint32_t q = Sh::fan_chunk(cs);
    const uint32_t per_pass = MODE == 1 ? kTile : (cs - 1) * q;
    if (MODE != 0 && threadIdx.x == 0) {
        for (int p = 0; p < passes; ++p) {
            mbar_init(sa + 8u * p, 1);
            mbar_arrive_expect_tx(sa + 8u * p, per_pass);   // armed up front: bytes of pass p
        }
        fence_mbar_init();
    }
    fence_proxy_async_smem();
    __syncthreads();
    cluster_sync();
    if (MODE == 0) {
        const uint32_t base = mapa(sa + kSrc, peer);
        uint32_t acc = 0;
        for (int p = 0; p < passes; ++p) {
#pragma unroll 4
            for (uint32_t i = threadIdx.x; i < kTile / 16; i += blockDim.x) {
                const uint4 v = ld_cluster_v4(base + 16u * i);
                acc ^= v.x ^ v.y ^ v.z ^ v.w;
            }
        }
        if (acc == 0x9e3779b9u) atomicAdd(sink, 1u);   // keeps every load live
    } else {
        if (threadIdx.x == 0) {
            for (int p = 0; p < passes; ++p) {
                if (MODE == 1) {
                    for (uint32_t c = 0; c < kTile; c += kChunk)
                        bulk_push(peer, sa + kDst + c, sa + kSrc + c, kChunk, sa + 8u * p);
                } else {
                    // chunk to rank+j lands in the receiver's slot j-1 (unique per sender)
                    for (uint32_t j = 1; j < cs; ++j)
                        bulk_push((rank + j) % cs, sa + kDst + (j - 1) * q, sa + kSrc + (j - 1) * q, q, sa + 8u * p);
                }
            }
        }
        if (threadIdx.x == 32) {   // one waiter: every pass's bytes landed in my destination tile
            const unsigned long long deadline = globaltimer() + limit;
            for (int p = 0; p < passes; ++p)
                if (!mbar_wait_parity_until(sa + 8u * p, 0, deadline)) {
                    atomicOr(err, DSMEM_ERR_BIT_TIMEOUT);
                    break;
                }
        }
        __syncthreads();
    }
    cluster_sync();   // no CTA leaves while a peer may still access its shared memory
}

}  // namespace

extern "C" {

// Time `reps` launches (after 2 warm-ups) of the DSMEM bandwidth kernel on the current device.
// mode 0 = pull (ld.shared::cluster.v4), 1 = push to the ring neighbour (cp.async.bulk), 2 = push to every
// peer (one chunk of 8 KiB, 4 KiB at CS 16, per peer per pass: the fan-out of the direct / two-shot
// algorithms). ctas_per_sm 1: 96 KiB tiles, 1024 threads (the reference's shape); 4: 24 KiB tiles, 256
// threads. Outputs: median ms per launch, payload bytes per launch and the resident clusters used.
dsmem_status dsmem_ceiling_dsmem_bw(int mode, int cluster_size, int ctas_per_sm, int passes, int reps,
                                    double* ms_median, long long* bytes_per_launch, int* clusters_out) {
    if (mode < 0 || mode > 2 || passes < 1 || passes > kMaxPasses || reps < 1 ||
        (ctas_per_sm != 1 && ctas_per_sm != 4) ||
        !(cluster_size == 2 || cluster_size == 4 || cluster_size == 8 || cluster_size == 16))
        return DSMEM_ERR_INVALID_ARGUMENT;
    const bool big = ctas_per_sm == 1;
    const void* const fns[2][3] = {
        {reinterpret_cast<const void*>(&dsmem_bw_kernel<0, 24u * 1024u, 256>),
         reinterpret_cast<const void*>(&dsmem_bw_kernel<1, 24u * 1024u, 256>),
         reinterpret_cast<const void*>(&dsmem_bw_kernel<2, 24u * 1024u, 256>)},
        {reinterpret_cast<const void*>(&dsmem_bw_kernel<0, 96u * 1024u, 1024>),
         reinterpret_cast<const void*>(&dsmem_bw_kernel<1, 96u * 1024u, 1024>),
         reinterpret_cast<const void*>(&dsmem_bw_kernel<2, 96u * 1024u, 1024>)}};
    const void* fn = fns[big ? 1 : 0][mode];
    const uint32_t kSmem = big ? Shape<96u * 1024u>::kSmem : Shape<24u * 1024u>::kSmem;
    const uint32_t kTile = big ? 96u * 1024u : 24u * 1024u;
    const uint32_t fan = big ? Shape<96u * 1024u>::fan_chunk((uint32_t)cluster_size)
                             : Shape<24u * 1024u>::fan_chunk((uint32_t)cluster_size);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
        cudaSuccess)
        return DSMEM_ERR_CUDA;
    if (cluster_size > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster_size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(big ? 1024 : 256, 1, 1);
    cfg.gridDim = dim3((unsigned)cluster_size, 1, 1);
    cfg.dynamicSmemBytes = kSmem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess || clusters < 1) return DSMEM_ERR_CUDA;
    cfg.gridDim = dim3((unsigned)(clusters * cluster_size), 1, 1);
    unsigned* dev = nullptr;
    if (cudaMalloc(&dev, 2 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
    cudaMemset(dev, 0, 2 * sizeof(unsigned));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    std::vector<float> t;
    dsmem_status st = DSMEM_OK;
    const unsigned long long limit = 1000000000ull;
    for (int i = 0; i < reps + 2 && st == DSMEM_OK; ++i) {
        int p = passes;
        unsigned* err = dev;
        unsigned* sink = dev + 1;
        unsigned long long lim = limit;
        void* args[] = {&p, &err, &sink, &lim};
        cudaEventRecord(e0);
        if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) st = DSMEM_ERR_CUDA;
        cudaEventRecord(e1);
        if (cudaEventSynchronize(e1) != cudaSuccess) st = DSMEM_ERR_CUDA;
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (i >= 2) t.push_back(ms);
    }
    unsigned h[2] = {0, 0};
    cudaMemcpy(h, dev, sizeof h, cudaMemcpyDeviceToHost);
    cudaFree(dev);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (st != DSMEM_OK) return st;
    if (h[0] & DSMEM_ERRBIT_TIMEOUT) return DSMEM_ERR_TIMEOUT;
    std::sort(t.begin(), t.end());
    if (ms_median) *ms_median = t[t.size() / 2];
    const long long per_pass = mode == 2 ? (long long)(cluster_size - 1) * fan : kTile;
    if (bytes_per_launch) *bytes_per_launch = (long long)clusters * cluster_size * passes * per_pass;
    if (clusters_out) *clusters_out = clusters;
    return DSMEM_OK;
}

}  // extern "C"
