// ext_ceilings_sm100.cu -- ceilings of this GPU beyond DSMEM and HBM, for hierarchical rooflines: the
// 5th-generation tensor cores, the L2 and the SMs' shared memory.
//
// The reference's ceiling suite (roofline/harness/ceilings, roofline/docs/DESIGN.md:28-48) measures DSMEM
// and HBM on H100; these are its sm_100a counterparts for the units the B200 kernels here lean on.
// Every measurement is 1 / slope of launch time over work (two or more work amounts per call), which
// removes the fixed cost of a launch:
//   tcgen05  one CTA per SM; one thread issues back-to-back tcgen05.mma.cta_group::1.kind::f16
//            (M = 128, N = n, K = 16, bf16 operands in shared memory with the 128-byte swizzle, fp32
//            accumulator in TMEM), `iters` x 4 per launch, then tcgen05.commit and a bounded wait;
//   l2       every thread of a full grid reads a buffer that fits the 126 MB L2 with 16-byte loads,
//            `passes` times (after one pass that brings it in), into a sink;
//   smem     every thread reads its CTA's 96 KiB shared-memory tile with 16-byte loads `passes` times.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"

namespace {

using namespace dsmem;

constexpr uint32_t kA = 1024;                    // A tile (128 x 64 bf16, 16 KiB) at 1 KiB
constexpr uint32_t kB = kA + 16384;              // B tile (n x 64 bf16, up to 32 KiB)
constexpr uint32_t kMmaSmem = 120u * 1024u;   // operands need ~50 KiB; the rest keeps one CTA per SM
constexpr uint32_t kTmemWord = 64, kDoneBar = 0;

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

__global__ void __launch_bounds__(128, 1) tcgen05_peak_kernel(int n, int iters, unsigned* err, unsigned* sink) {
    const uint32_t sa = smem_u32(dyn_smem_raw);
    const uint32_t base = ((sa + 1023u) & ~1023u) - sa;   // 1024-aligned window for the swizzle atoms
    const int warp = threadIdx.x >> 5;
    // operands: small integers as bf16 (exact sums), the same in every CTA
    uint16_t* a = reinterpret_cast<uint16_t*>(dyn_smem_raw + base + kA);
    for (uint32_t i = threadIdx.x; i < (16384u + 32768u) / 2u; i += blockDim.x) a[i] = (i & 7u) ? 0x3f80u : 0u;
    if (threadIdx.x == 0) {
        mbar_init(sa + base + 8u * kDoneBar, 1);
        fence_mbar_init();
    }
    fence_proxy_async_smem();
    const uint32_t cols = n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : 256u;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa + base + kTmemWord),
                     "r"(cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(dyn_smem_raw + base + kTmemWord);
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (((uint32_t)n >> 3) << 17) | ((128u >> 4) << 24);
    if (threadIdx.x == 0) {
        const uint32_t aa = sa + base + kA, bb = sa + base + kB;
        for (int it = 0; it < iters; ++it)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t acc = (it | k) != 0 ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
                    "l"(desc_sw128(aa + 32u * k)), "l"(desc_sw128(bb + 32u * k)), "r"(idesc), "r"(acc)
                    : "memory");
            }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         sa + base + 8u * kDoneBar)
                     : "memory");
    }
    // bounded wait for the accumulator (1 s)
    const unsigned long long until = globaltimer() + 1000000000ull;
    if (!mbar_wait_parity_until(sa + base + 8u * kDoneBar, 0u, until) && threadIdx.x == 0) atomicOr(err, 1u);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) {   // one value out, so the work is observable
        uint32_t v;
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(tmem));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (threadIdx.x == 0 && v == 0x7fffffffu) atomicAdd(sink, 1u);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
}

__global__ void __launch_bounds__(256) l2_read_kernel(const uint4* buf, size_t n16, int passes, unsigned* sink) {
    uint32_t x = 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (int p = 0; p < passes; ++p)
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
            uint4 v;
            asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(buf + i));
            x ^= v.x ^ v.y ^ v.z ^ v.w;
        }
    if (x == 0x12345678u) atomicAdd(sink, 1u);
}

constexpr uint32_t kSmemTile = 96u * 1024u;

__global__ void __launch_bounds__(1024, 1) smem_read_kernel(int passes, unsigned* sink) {
    uint4* t = reinterpret_cast<uint4*>(dyn_smem_raw);
    for (uint32_t i = threadIdx.x; i < kSmemTile / 16; i += blockDim.x) t[i] = make_uint4(i, i + 1, i + 2, i + 3);
    __syncthreads();
    uint32_t x = 0;
    for (int p = 0; p < passes; ++p)
#pragma unroll 4
        for (uint32_t i = threadIdx.x; i < kSmemTile / 16; i += blockDim.x) {
            uint4 v;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"(smem_u32(t + i)));   // volatile: every pass loads again
            x ^= v.x ^ v.y ^ v.z ^ v.w;
        }
    if (x == 0x12345678u) atomicAdd(sink, 1u);
}

// Median over `reps` of a launch's event time, in ms.
template <class F>
cudaError_t time_ms(F launch, int reps, double* ms) {
    cudaEvent_t e0, e1;
    cudaError_t r = cudaEventCreate(&e0);
    if (r != cudaSuccess) return r;
    if ((r = cudaEventCreate(&e1)) != cudaSuccess) return cudaEventDestroy(e0), r;
    std::vector<double> t;
    for (int i = 0; i < reps + 1 && r == cudaSuccess; ++i) {
        cudaEventRecord(e0);
        launch();
        cudaEventRecord(e1);
        if ((r = cudaEventSynchronize(e1)) != cudaSuccess) break;
        if ((r = cudaGetLastError()) != cudaSuccess) break;
        float f = 0.f;
        cudaEventElapsedTime(&f, e0, e1);
        if (i > 0) t.push_back(f);   // the first launch warms up
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (r != cudaSuccess) return r;
    std::sort(t.begin(), t.end());
    *ms = t[t.size() / 2];
    return cudaSuccess;
}

}  // namespace

extern "C" {

dsmem_status dsmem_ceiling_tcgen05(int n, int iters, int reps, double* ms_median, double* flops_per_launch,
                                   int* ctas) {
    if (!(n == 64 || n == 128 || n == 256) || iters < 1 || reps < 1 || ms_median == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    if (cudaFuncSetAttribute(tcgen05_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMmaSmem) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    unsigned* w = nullptr;   // error word, sink
    if (cudaMalloc(&w, 2 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
    cudaMemset(w, 0, 2 * sizeof(unsigned));
    const cudaError_t r = time_ms([&] { tcgen05_peak_kernel<<<sms, 128, kMmaSmem>>>(n, iters, w, w + 1); }, reps, ms_median);
    unsigned e = 0;
    if (r == cudaSuccess) cudaMemcpy(&e, w, sizeof e, cudaMemcpyDeviceToHost);
    cudaFree(w);
    if (r != cudaSuccess) return DSMEM_ERR_CUDA;
    if (e != 0) return DSMEM_ERR_TIMEOUT;
    if (flops_per_launch) *flops_per_launch = 2.0 * 128.0 * n * 16.0 * 4.0 * iters * sms;
    if (ctas) *ctas = sms;
    return DSMEM_OK;
}

dsmem_status dsmem_ceiling_l2_bw(long long bytes, int passes, int reps, double* ms_median, double* bytes_per_launch) {
    if (bytes < (1 << 20) || bytes % 16 || passes < 1 || reps < 1 || ms_median == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    void* buf = nullptr;
    unsigned* sink = nullptr;
    if (cudaMalloc(&buf, (size_t)bytes) != cudaSuccess) return DSMEM_ERR_CUDA;
    if (cudaMalloc(&sink, sizeof(unsigned)) != cudaSuccess) return cudaFree(buf), DSMEM_ERR_CUDA;
    cudaMemset(buf, 1, (size_t)bytes);
    const size_t n16 = (size_t)bytes / 16;
    const cudaError_t r = time_ms(
        [&] { l2_read_kernel<<<sms * 8, 256>>>(static_cast<const uint4*>(buf), n16, passes, sink); }, reps, ms_median);
    cudaFree(buf);
    cudaFree(sink);
    if (r != cudaSuccess) return DSMEM_ERR_CUDA;
    if (bytes_per_launch) *bytes_per_launch = (double)bytes * passes;
    return DSMEM_OK;
}

dsmem_status dsmem_ceiling_smem_bw(int passes, int reps, double* ms_median, double* bytes_per_launch) {
    if (passes < 1 || reps < 1 || ms_median == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    if (cudaFuncSetAttribute(smem_read_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTile) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    unsigned* sink = nullptr;
    if (cudaMalloc(&sink, sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
    const cudaError_t r = time_ms([&] { smem_read_kernel<<<sms, 1024, kSmemTile>>>(passes, sink); }, reps, ms_median);
    cudaFree(sink);
    if (r != cudaSuccess) return DSMEM_ERR_CUDA;
    if (bytes_per_launch) *bytes_per_launch = (double)kSmemTile * passes * sms;
    return DSMEM_OK;
}

}  // extern "C"
