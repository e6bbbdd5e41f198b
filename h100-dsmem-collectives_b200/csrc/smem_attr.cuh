// smem_attr.cuh -- per-kernel dynamic shared-memory opt-in that only ever grows.
//
// cudaFuncAttributeMaxDynamicSharedMemorySize belongs to the kernel (per device), not to a launch: a launch that
// asks for more dynamic shared memory than the kernel's current value fails with an invalid-argument error.
// One kernel launched with several shared-memory sizes (shapes) therefore keeps its attribute at the largest
// size requested so far; lowering it for a small launch would break the next large one.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <utility>

namespace dsb_attr {

// Raise fn's dynamic shared-memory limit on device `dev` to at least `smem` bytes (and, the first time, allow
// non-portable cluster sizes when asked and prefer the largest shared-memory carveout).
inline cudaError_t ensure_smem(const void* fn, int dev, uint32_t smem, bool nonportable_cluster = false,
                               bool max_carveout = true) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, uint32_t> cur;   // largest value set per (kernel, device)
    std::lock_guard<std::mutex> lock(mu);
    auto it = cur.find({fn, dev});
    cudaError_t r;
    if (it == cur.end()) {
        if (nonportable_cluster &&
            (r = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)) != cudaSuccess)
            return r;
        if (max_carveout && (r = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                      cudaSharedmemCarveoutMaxShared)) != cudaSuccess)
            return r;
        it = cur.emplace(std::make_pair(fn, dev), 0u).first;
    }
    if (smem > it->second) {
        if ((r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
            return r;
        it->second = smem;
    }
    return cudaSuccess;
}

}  // namespace dsb_attr
