// ext_host.cu -- the collective catalogue on HOST buffers: copies in, the batch, copies out, overlapped.
//
// The reference's host-side check computes a collective on host arrays (collectives/harness/main.cu:129-149,
// reference()); a host caller of the B200 catalogue wants the same shape of call: host input, host output,
// results on return. dsmem_collective_host streams the batch through double-buffered device staging in chunks
// of whole cluster problems on three streams: the host-to-device copy of chunk i+1, the collective on chunk i
// (dsmem_collective_launch_ex, the batch regime) and the device-to-host copy of chunk i-1 run at the same time,
// so a PCIe-bound call costs about one direction's copy time instead of the sum of both.
//
// Chunk i uses staging slot b = i % 2. Ordering, all by events recorded in host issue order:
//   copy-in(i)   waits for the collective of chunk i-2 (it read in[b]);
//   collective(i) waits for copy-in(i) and for copy-out(i-2) (it read out[b]);
//   copy-out(i)  waits for collective(i).
// The call returns after the last copy-out and the device error check (dsmem_check on the compute stream).
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/dsmem_b200.h"

namespace {

struct HostPipe {
    bool ready = false;
    cudaStream_t s[3] = {};   // copy-in, compute, copy-out
    cudaEvent_t in_done[2] = {}, k_done[2] = {}, out_done[2] = {};
    void* din[2] = {};
    void* dout[2] = {};
    size_t cap_in = 0, cap_out = 0;   // bytes per staging buffer
};
std::mutex g_mu[64];   // one host pipeline per device at a time (its staging is shared)
HostPipe g_pipe[64];

constexpr size_t kChunkTarget = 64ull << 20;   // bytes of the larger side (in or out) per chunk

bool init(HostPipe& p) {
    if (p.ready) return true;
    for (auto& s : p.s)
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return false;
    for (int b = 0; b < 2; ++b)
        if (cudaEventCreateWithFlags(&p.in_done[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&p.k_done[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&p.out_done[b], cudaEventDisableTiming) != cudaSuccess)
            return false;
    p.ready = true;
    return true;
}

bool reserve(void** buf, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return true;
    for (int b = 0; b < 2; ++b) {
        if (buf[b] != nullptr && cudaFree(buf[b]) != cudaSuccess) return false;
        buf[b] = nullptr;
    }
    *cap = 0;
    for (int b = 0; b < 2; ++b)
        if (cudaMalloc(&buf[b], bytes) != cudaSuccess) return false;
    *cap = bytes;
    return true;
}

}  // namespace

extern "C" dsmem_status dsmem_collective_host(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                              size_t bytes_per_cta, const void* host_in, void* host_out,
                                              long long num_clusters, long long chunk_clusters) {
    if (host_in == nullptr || host_out == nullptr || num_clusters < 0) return DSMEM_ERR_INVALID_ARGUMENT;
    if ((int)op < 0 || (int)op > 7 || (int)dtype < 0 || (int)dtype > 2) return DSMEM_ERR_INVALID_ARGUMENT;
    if (!(cluster_size == 2 || cluster_size == 4 || cluster_size == 8 || cluster_size == 16))
        return DSMEM_ERR_INVALID_ARGUMENT;
    // elements per rank block (the payload convention of dsmem_collective_launch)
    const size_t n = (size_t)cluster_size, eb = dtype == DSMEM_BF16 ? 2 : 4;
    const bool per_peer_in = op == DSMEM_OP_REDUCESCATTER || op == DSMEM_OP_ALLTOALL || op == DSMEM_OP_SCATTER;
    const bool per_peer_out = op == DSMEM_OP_ALLGATHER || op == DSMEM_OP_ALLTOALL || op == DSMEM_OP_GATHER;
    // the rooted Reduce and Gather write rank 0's out block only: only those blocks are copied back, so the
    // other ranks' blocks of host_out keep their contents, as on the device
    const bool root_out_only = op == DSMEM_OP_REDUCE || op == DSMEM_OP_GATHER;
    const size_t unit = eb * (op == DSMEM_OP_ALLREDUCE || op == DSMEM_OP_BROADCAST || op == DSMEM_OP_REDUCE ? 1 : n);
    if (bytes_per_cta == 0 || bytes_per_cta % unit != 0) return DSMEM_ERR_ILLEGAL_CONFIG;
    const size_t m = bytes_per_cta / unit;
    const size_t in_pp = n * (per_peer_in ? n : 1) * m * eb;     // input bytes per cluster problem
    const size_t out_pp = n * (per_peer_out ? n : 1) * m * eb;   // output bytes per cluster problem
    const size_t out_root = (per_peer_out ? n : 1) * m * eb;     // bytes of rank 0's out block
    if (num_clusters == 0) return DSMEM_OK;
    long long cc = chunk_clusters > 0 ? chunk_clusters
                                      : std::max<long long>(1, (long long)(kChunkTarget / std::max(in_pp, out_pp)));
    cc = std::min(cc, num_clusters);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    // every chunk runs the algorithm AUTO picks for the whole batch, so a short last chunk computes exactly
    // what the one-launch batch would (the summation order depends on the algorithm)
    if (alg == DSMEM_ALG_AUTO) alg = dsmem_autotune_pick_ex(op, dtype, cluster_size, bytes_per_cta, num_clusters);
    std::lock_guard<std::mutex> lock(g_mu[dev]);
    HostPipe& p = g_pipe[dev];
    if (!init(p) || !reserve(p.din, &p.cap_in, (size_t)cc * in_pp) || !reserve(p.dout, &p.cap_out, (size_t)cc * out_pp))
        return DSMEM_ERR_CUDA;
    const long long chunks = (num_clusters + cc - 1) / cc;
    dsmem_status status = DSMEM_OK;
    for (long long i = 0; i < chunks && status == DSMEM_OK; ++i) {
        const int b = (int)(i & 1);
        const long long p0 = i * cc, np = std::min(cc, num_clusters - p0);
        const char* src = static_cast<const char*>(host_in) + (size_t)p0 * in_pp;
        char* dst = static_cast<char*>(host_out) + (size_t)p0 * out_pp;
        bool ok = true;
        if (i >= 2) ok = ok && cudaStreamWaitEvent(p.s[0], p.k_done[b], 0) == cudaSuccess;
        ok = ok && cudaMemcpyAsync(p.din[b], src, (size_t)np * in_pp, cudaMemcpyHostToDevice, p.s[0]) == cudaSuccess;
        ok = ok && cudaEventRecord(p.in_done[b], p.s[0]) == cudaSuccess;
        ok = ok && cudaStreamWaitEvent(p.s[1], p.in_done[b], 0) == cudaSuccess;
        if (i >= 2) ok = ok && cudaStreamWaitEvent(p.s[1], p.out_done[b], 0) == cudaSuccess;
        if (!ok) {
            status = DSMEM_ERR_CUDA;
            break;
        }
        status = dsmem_collective_launch_ex(op, alg, dtype, cluster_size, bytes_per_cta, p.din[b], p.dout[b], np,
                                            nullptr, nullptr, 0, reinterpret_cast<dsmem_stream_t>(p.s[1]));
        if (status != DSMEM_OK) break;
        ok = cudaEventRecord(p.k_done[b], p.s[1]) == cudaSuccess &&
             cudaStreamWaitEvent(p.s[2], p.k_done[b], 0) == cudaSuccess &&
             (root_out_only ? cudaMemcpy2DAsync(dst, out_pp, p.dout[b], out_pp, out_root, (size_t)np,
                                                cudaMemcpyDeviceToHost, p.s[2])
                            : cudaMemcpyAsync(dst, p.dout[b], (size_t)np * out_pp, cudaMemcpyDeviceToHost, p.s[2])) ==
                 cudaSuccess &&
             cudaEventRecord(p.out_done[b], p.s[2]) == cudaSuccess;
        if (!ok) status = DSMEM_ERR_CUDA;
    }
    // drain every stream (also after an error, so no copy into or out of the caller's buffers outlives the call)
    const bool drained = cudaStreamSynchronize(p.s[0]) == cudaSuccess && cudaStreamSynchronize(p.s[2]) == cudaSuccess;
    const dsmem_status chk = dsmem_check(reinterpret_cast<dsmem_stream_t>(p.s[1]));
    if (status != DSMEM_OK) return status;
    if (!drained) return DSMEM_ERR_CUDA;
    return chk;
}
