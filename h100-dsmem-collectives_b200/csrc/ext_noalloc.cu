// ext_noalloc.cu -- batch two-shot AllReduce for callers that cannot allocate device memory.
//
// dsmem_collective_launch allocates a device error word with cudaMalloc the first time it runs on a
// device. Some callers cannot allow that: a framework whose caching allocator has reserved the GPU's
// memory up front and accounts for every byte (an allocation behind its back can fail, or push the
// framework itself out of memory later), and programs with a fixed, pre-planned memory map in which nothing
// is allocated after start-up. For them this file provides one entry point that allocates nothing: its
// scratch (the error word and one status word per cluster problem) is a file-scope static __device__
// array of fixed size, present on every GPU that loads the library until the process exits.
//
// Notes for callers:
//   * The first call on a device is its set-up, made with that device current: the entry point looks up
//     the array's device address (cudaGetSymbolAddress) and resolves every kernel it can launch (all three
//     dtypes and the four cluster sizes: attributes queried, so the CUDA runtime loads their code now
//     rather than on a later call, and shared-memory and cluster-size attributes set). The runtime may
//     claim device memory for that code during this first call; make it before any stream capture begins.
//     Later calls, whatever their dtype or cluster size, touch no device memory beyond the caller's
//     buffers and the array.
//   * Every call reuses the same array. The call clears the part it uses (cudaMemsetAsync on the caller's
//     stream) before the kernel runs, and the array keeps the last call's contents afterwards. Calls
//     whose kernels overlap on the GPU (different streams, or different host threads without ordering)
//     race on the array: serialise them.
//   * At most DSMEM_NOALLOC_MAX_PROBLEMS cluster problems per call; larger batches are rejected with
//     DSMEM_ERR_SCRATCH_LIMIT before anything is launched.
//   * A call with num_clusters == 0 launches nothing. With status_out given it reads back the previous
//     call's device error bits (the way to learn them after a call made with status_out == NULL).
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"

namespace {

constexpr int kMaxDevices = 64;
constexpr uint32_t kStatusBase = 64;   // word 0: error word; words [64, 64 + max): per-problem status

// The scratch: 4 * (64 + 65536) bytes = 256.25 KiB per device.
static __device__ __align__(256) unsigned g_noalloc_scratch[kStatusBase + DSMEM_NOALLOC_MAX_PROBLEMS];

// The plain batch driver of dsb::batch_kernel with one addition: after each problem, every CTA ORs the
// error bits it saw (any thread's timed-out wait) into status[problem].
template <class A>
__global__ void __launch_bounds__(256) batch_status_kernel(const dsb::BatchArgs a, unsigned* status) {
    using namespace dsmem;
    using T = typename A::T;
    constexpr int N = A::kN;
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    dsb::init_bars<A>(c);
    const uint64_t in_r = dsb::in_elems_per_rank<A>(a.M), out_r = dsb::out_elems_per_rank<A>(a.M);
    const long long step = (long long)num_clusters();
    for (long long p = (long long)cluster_id(); p < a.num_problems; p += step, ++c.unit) {
        const uint64_t slot = (uint64_t)p * N + c.rank;
        c.deadline = globaltimer() + c.wait_limit;
        A::load(c, static_cast<const T*>(a.in) + slot * in_r, a.M);
        cluster_sync();
        A::exec(c, a.M);
        A::store(c, static_cast<T*>(a.out) + slot * out_r, a.M);
        if (__syncthreads_or(c.dead ? 1 : 0) && threadIdx.x == 0) atomicOr(&status[p], DSMEM_ERR_BIT_TIMEOUT);
        cluster_sync();
    }
    dsb::finish(c);
}

template <int N, typename T>
const void* kernel_for() {
    return reinterpret_cast<const void*>(&batch_status_kernel<dsb::AR_TwoShotPush<N, T, dsmem::Sum>>);
}

template <typename T>
const void* kernel_for_n(int n) {
    switch (n) {
        case 2: return kernel_for<2, T>();
        case 4: return kernel_for<4, T>();
        case 8: return kernel_for<8, T>();
        case 16: return kernel_for<16, T>();
    }
    return nullptr;
}

template <typename T>
bool legal_for(int n, uint32_t m, uint64_t* smem) {
    switch (n) {
        case 2: *smem = dsb::AR_TwoShotPush<2, T, dsmem::Sum>::smem_bytes(m); return dsb::AR_TwoShotPush<2, T, dsmem::Sum>::legal(m);
        case 4: *smem = dsb::AR_TwoShotPush<4, T, dsmem::Sum>::smem_bytes(m); return dsb::AR_TwoShotPush<4, T, dsmem::Sum>::legal(m);
        case 8: *smem = dsb::AR_TwoShotPush<8, T, dsmem::Sum>::smem_bytes(m); return dsb::AR_TwoShotPush<8, T, dsmem::Sum>::legal(m);
        case 16: *smem = dsb::AR_TwoShotPush<16, T, dsmem::Sum>::smem_bytes(m); return dsb::AR_TwoShotPush<16, T, dsmem::Sum>::legal(m);
    }
    return false;
}

struct DeviceSetup {
    bool ready = false;
    unsigned* scratch = nullptr;   // device address of g_noalloc_scratch on this device
    int optin = 0;
    int occupancy[3][5] = {};      // [dtype][log2 N - 1] for the last smem size
    uint32_t occ_smem[3][5] = {};
};
std::mutex g_mu;
DeviceSetup g_dev[kMaxDevices];   // fixed table: no host allocation either

int slot_of(int n) { return n == 2 ? 1 : n == 4 ? 2 : n == 8 ? 3 : 4; }

const void* kernel_of(int dtype, int n) {
    return dtype == DSMEM_F32    ? kernel_for_n<float>(n)
           : dtype == DSMEM_BF16 ? kernel_for_n<__nv_bfloat16>(n)
                                 : kernel_for_n<int>(n);
}

// Once per device, with that device current (caller holds g_mu): the array's address, and every kernel
// this entry point can launch resolved now. cudaFuncGetAttributes makes the runtime load a kernel's code
// (with lazy module loading it would otherwise load on the first launch of each dtype and cluster size,
// and may claim device memory then); the attributes are set to the largest shared memory a call can ask
// for, so no later call changes them.
cudaError_t setup_device(DeviceSetup& d, int dev) {
    cudaError_t r = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), g_noalloc_scratch);
    if (r != cudaSuccess) return r;
    r = cudaDeviceGetAttribute(&d.optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (r != cudaSuccess) return r;
    const int max_smem = (int)std::min<uint64_t>((uint64_t)d.optin, dsb::kSmemLimit);
    for (int dt = DSMEM_F32; dt <= DSMEM_I32; ++dt)
        for (int n : {2, 4, 8, 16}) {
            const void* fn = kernel_of(dt, n);
            cudaFuncAttributes fa{};
            if ((r = cudaFuncGetAttributes(&fa, fn)) != cudaSuccess) return r;
            if (n > 8 && (r = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)) != cudaSuccess)
                return r;
            if ((r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess)
                return r;
        }
    d.ready = true;
    return cudaSuccess;
}

dsmem_status status_of(unsigned err) {
    if (err & DSMEM_ERRBIT_TIMEOUT) return DSMEM_ERR_TIMEOUT;
    if (err & DSMEM_ERRBIT_BOUNDS) return DSMEM_ERR_BOUNDS;
    return DSMEM_OK;
}

}  // namespace

extern "C" dsmem_status dsmem_allreduce_two_shot_noalloc(dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta,
                                                         const void* in, void* out, int num_clusters,
                                                         unsigned* status_out, dsmem_stream_t stream) {
    const cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    if (num_clusters == 0) {
        // launches nothing; with status_out, the previous call's device error bits (status_out[0])
        if (status_out == nullptr) return DSMEM_OK;
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSMEM_ERR_CUDA;
        unsigned* scratch = nullptr;
        {
            std::lock_guard<std::mutex> lock(g_mu);
            scratch = g_dev[dev].ready ? g_dev[dev].scratch : nullptr;
        }
        unsigned err = 0;
        if (scratch != nullptr) {
            if (cudaStreamSynchronize(cs) != cudaSuccess) return DSMEM_ERR_CUDA;
            if (cudaMemcpy(&err, scratch, sizeof err, cudaMemcpyDeviceToHost) != cudaSuccess) return DSMEM_ERR_CUDA;
        }
        status_out[0] = err;
        return status_of(err);
    }
    const int n = cluster_size;
    if (!(n == 2 || n == 4 || n == 8 || n == 16) || dtype < DSMEM_F32 || dtype > DSMEM_I32 || num_clusters < 0 ||
        in == nullptr || out == nullptr)
        return DSMEM_ERR_INVALID_ARGUMENT;
    if (num_clusters > DSMEM_NOALLOC_MAX_PROBLEMS) return DSMEM_ERR_SCRATCH_LIMIT;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) return DSMEM_ERR_INVALID_ARGUMENT;
    const size_t eb = dtype == DSMEM_BF16 ? 2 : 4;
    if (bytes_per_cta == 0 || bytes_per_cta % eb || bytes_per_cta / eb > 0xffffffffull) return DSMEM_ERR_ILLEGAL_CONFIG;
    const uint32_t m = (uint32_t)(bytes_per_cta / eb);
    uint64_t smem = 0;
    const bool legal = dtype == DSMEM_F32    ? legal_for<float>(n, m, &smem)
                       : dtype == DSMEM_BF16 ? legal_for<__nv_bfloat16>(n, m, &smem)
                                             : legal_for<int>(n, m, &smem);
    if (!legal) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (smem > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    const void* fn = kernel_of(dtype, n);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSMEM_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = cs;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    unsigned* scratch = nullptr;
    int resident = 0;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        DeviceSetup& d = g_dev[dev];
        if (!d.ready && setup_device(d, dev) != cudaSuccess) return DSMEM_ERR_CUDA;
        if (smem > (uint64_t)d.optin) return DSMEM_ERR_SMEM_LIMIT;
        const int di = (int)dtype, ni = slot_of(n);
        if (d.occ_smem[di][ni] != (uint32_t)smem) {
            cfg.gridDim = dim3((unsigned)n, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&d.occupancy[di][ni], fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
            d.occ_smem[di][ni] = (uint32_t)smem;
        }
        resident = d.occupancy[di][ni];
        scratch = d.scratch;
    }
    if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;
    // clear the error word and this call's status words (the array keeps the previous call's contents)
    if (cudaMemsetAsync(scratch, 0, sizeof(unsigned) * (kStatusBase + (size_t)num_clusters), cs) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    dsb::BatchArgs a{};
    a.in = in;
    a.out = out;
    a.num_problems = num_clusters;
    a.err = scratch;
    a.wait_limit_ns = 1000000000ull;
    a.M = m;
    a.smem_bytes = (uint32_t)smem;
    a.sub = 1;
    unsigned* status = scratch + kStatusBase;
    cfg.gridDim = dim3((unsigned)(std::min<long long>(num_clusters, resident) * n), 1, 1);
    void* args[] = {&a, &status};
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return DSMEM_ERR_CUDA;
    if (status_out == nullptr) return DSMEM_OK;
    if (cudaStreamSynchronize(cs) != cudaSuccess) return DSMEM_ERR_CUDA;
    if (cudaMemcpy(status_out, status, sizeof(unsigned) * (size_t)num_clusters, cudaMemcpyDeviceToHost) != cudaSuccess)
        return DSMEM_ERR_CUDA;
    unsigned err = 0;
    if (cudaMemcpy(&err, scratch, sizeof err, cudaMemcpyDeviceToHost) != cudaSuccess) return DSMEM_ERR_CUDA;
    return status_of(err);
}
