// shim_launcher.cu -- launches one reference-harness plugin file (collectives/<op>__<alg>__<src>.cu) the way
// the reference harness does, so the 29 harness-compatible files are built and run outside that harness.
//
// Compiled once per (file, N, element type) with the harness's knobs (collectives/harness/driver.py:233-239):
//   -DCOLLECTIVE_FILE="<path>" -DCLUSTER_N=<N> -DMSG_ELEMS=<M> -DELEM_T=<float|int> -DSHIM_TAG=<unique tag>
// The plugin file defines `collective_kernel` and `struct CollectiveSmem`; both are renamed per tag so that
// every build links into one library (lib/libdsmem_shims.so). Illegal (N, M) stay the compile errors the
// reference classifies (static_assert -> SKIP:static_assert; CollectiveSmem above 227 KiB -> SKIP:smem,
// collectives/harness/main.cu:90-92), and the builder (dsmem_b200/shims.py) records them as skips.
//
// Each build exports
//   int <tag>_launch(in, out, ts, smid, stream)   one cluster of CLUSTER_N CTAs, 256 threads, dynamic shared
//                                                 memory sizeof(CollectiveSmem) with the opt-in attribute and,
//                                                 for N > 8, the non-portable cluster-size attribute
//                                                 (main.cu:207-214, :273); returns the cudaError_t
//   size_t <tag>_smem(void)                       sizeof(CollectiveSmem)
//   unsigned <tag>_take_error(void)               the build's device error word (bounded waits that gave up,
//                                                 bounds checks), read and cleared; synchronous
#include <cuda_runtime.h>

#define DSB_CAT2(a, b) a##b
#define DSB_CAT(a, b) DSB_CAT2(a, b)
#define collective_kernel DSB_CAT(SHIM_TAG, _kernel)
#define CollectiveSmem DSB_CAT(SHIM_TAG, _smem_t)

#include COLLECTIVE_FILE

static_assert(sizeof(CollectiveSmem) <= 232448u, "SMEM_LIMIT: CollectiveSmem exceeds the 227 KiB a block may opt in to");

extern "C" int DSB_CAT(SHIM_TAG, _launch)(const void* in, void* out, unsigned long long* ts, unsigned* smid,
                                          cudaStream_t stream) {
    cudaError_t r = cudaSuccess;
    if (CLUSTER_N > 8) r = cudaFuncSetAttribute(collective_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (r == cudaSuccess)
        r = cudaFuncSetAttribute(collective_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(CollectiveSmem));
    if (r != cudaSuccess) return (int)r;
    collective_kernel<<<CLUSTER_N, 256, sizeof(CollectiveSmem), stream>>>(static_cast<const ELEM_T*>(in),
                                                                         static_cast<ELEM_T*>(out), ts, smid);
    return (int)cudaGetLastError();
}

extern "C" size_t DSB_CAT(SHIM_TAG, _smem)(void) { return sizeof(CollectiveSmem); }

extern "C" unsigned DSB_CAT(SHIM_TAG, _take_error)(void) {
    unsigned v = 0, z = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyFromSymbol(&v, dsmem_wait_error, sizeof v) != cudaSuccess) return 0xffffffffu;
    if (cudaMemcpyToSymbol(dsmem_wait_error, &z, sizeof z) != cudaSuccess) return 0xffffffffu;
    return v;
}
