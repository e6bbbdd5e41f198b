// ref_rowwise.cu -- TEST INFRASTRUCTURE ONLY: launchers for the reference's own clustered row-wise kernels.
//
// Compiled once per workload (oracle/Makefile, target `ref-rowwise`) with -DREF_WL=<0..5> and
// -DREF_FILE="<reference checkout>/kernels/<name>__reduction_reuse__credit.cu"; the reference file is included
// unmodified and its cluster kernel is launched as the reference launches it: one cluster of P CTAs per row
// (gridDim = rows * P), blockDim = kBlockThreads (256), slice_elems = ceil(cols / P), dynamic shared memory =
// the staged slices. tests/golden/make_rowwise_golden.py runs these on a GPU to record golden outputs.
// Nothing under h100-dsmem-collectives_b200/ links or loads this.
#include REF_FILE

#include <cuda_runtime.h>

#include <cstdint>

namespace {

template <class K, class... Args>
int launch_rows(K kernel, int rows, int cols, int p, int arrays, Args... args) {
    if (rows <= 0 || cols <= 0 || p < 1 || p > kMaxClusterSize) return 1;
    const int slice = (cols + p - 1) / p;
    const size_t smem = (size_t)slice * sizeof(float) * arrays;
    if (smem > 232448) return 2;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 3;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(rows * p), 1, 1);
    cfg.blockDim = dim3(kBlockThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kernel, args..., slice) != cudaSuccess) return 4;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 5;
}

}  // namespace

extern "C" {

#if REF_WL == 0
int ref_rowwise_quant(const float* x, int8_t* q, float* scales, int rows, int cols, int p) {
    return launch_rows(cluster_quant_staged_kernel<kBlockThreads, kMaxClusterSize>, rows, cols, p, 1, x, q, scales,
                       rows, cols);
}
#elif REF_WL == 1
int ref_lars_momentum(const float* w, const float* g, const float* m, float* w_out, float* m_out, int rows, int cols,
                      int p) {
    return launch_rows(cluster_lars_staged_kernel<kBlockThreads, kMaxClusterSize>, rows, cols, p, 3, w, g, m, w_out,
                       m_out, rows, cols);
}
#elif REF_WL == 2
int ref_layernorm_backward(const float* x, const float* dy, const float* gamma, float* dx, int rows, int cols,
                           float eps, int p) {
    return launch_rows(cluster_bwd_staged_kernel<kBlockThreads, kMaxClusterSize>, rows, cols, p, 1, x, dy, gamma, dx,
                       rows, cols, eps);
}
#elif REF_WL == 3
int ref_pearson_backward(const float* x, const float* y, const float* grad, float* dx, float* dy, int rows, int cols,
                         float eps, int p) {
    return launch_rows(cluster_bwd_staged_kernel<kBlockThreads, kMaxClusterSize>, rows, cols, p, 2, x, y, grad, dx, dy,
                       rows, cols, eps);
}
#elif REF_WL == 4
int ref_softmax_logits_backward(const float* z, const float* dy, float* dx, int rows, int cols, int p) {
    return launch_rows(cluster_softmax_logits_bwd_staged_kernel<kBlockThreads, kMaxClusterSize>, rows, cols, p, 2, z,
                       dy, dx, rows, cols);
}
#elif REF_WL == 5
int ref_weighted_var_backward(const float* x, const float* w, const float* dy, float* dx, int rows, int cols, int p) {
    return launch_rows(cluster_bwd_staged_kernel<kBlockThreads, kMaxClusterSize>, rows, cols, p, 3, x, w, dy, dx, rows,
                       cols);
}
#endif

}  // extern "C"
