// ref_rmsnorm.cu -- TEST INFRASTRUCTURE ONLY: a launcher for the reference's own cluster RMSNorm kernel.
//
// Compiled by oracle/Makefile (target `ref-rmsnorm`) with -DREF_FILE="<reference checkout>/kernels/
// rmsnorm__llama__clusterfusion.cu"; that file is included unmodified, with its compile-time shape
// (BATCH_SIZE x HIDDEN_DIM fp16 rows, CLUSTER_SIZE CTAs per row, BLOCK_SIZE threads), and its RMSNormKernel is
// launched as ClusterFusion launches it: one cluster per row, gridDim = BATCH_SIZE * CLUSTER_SIZE. The kernel has
// no waits of its own (two cluster barriers and one remote atomicAdd). tests/golden/make_rmsnorm_golden.py runs
// it on a GPU to record golden outputs. Nothing under h100-dsmem-collectives_b200/ links or loads this.
#include REF_FILE

extern "C" void ref_rmsnorm_shape(int* rows, int* hidden, int* cluster_size) {
    *rows = BATCH_SIZE;
    *hidden = HIDDEN_DIM;
    *cluster_size = CLUSTER_SIZE;
}

// x, w, y: device pointers to fp16 [BATCH_SIZE][HIDDEN_DIM], [HIDDEN_DIM], [BATCH_SIZE][HIDDEN_DIM].
extern "C" int ref_rmsnorm_launch(const void* x, const void* w, void* y) {
    RMSNormKernel<<<BATCH_SIZE * CLUSTER_SIZE, BLOCK_SIZE>>>(static_cast<half*>(y), const_cast<half*>(static_cast<const half*>(x)),
                                                           const_cast<half*>(static_cast<const half*>(w)));
    if (cudaGetLastError() != cudaSuccess) return 1;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}
