// registry.h -- host-side table of the compiled collective kernels (one entry per op x alg x dtype x N).
#pragma once
#include <cstdint>
#include <vector>

namespace dsb {

struct KernelEntry {
    int op;                              // dsmem_op
    int alg;                             // dsmem_alg
    int dtype;                           // dsmem_dtype
    int n;                               // cluster size
    int elem_bytes;                      // sizeof(T)
    const void* fn;                      // __global__ batch_kernel<A>
    bool (*legal)(uint32_t m);           // static N/M constraints of the reference file
    uint64_t (*smem_bytes)(uint32_t m);  // dynamic shared memory per CTA
    // Optional pipelined batch driver (same collective, overlapped HBM traffic), used for batches of more
    // than one problem when its shared memory fits; nullptr if the algorithm has none.
    const void* fn_pipe = nullptr;
    uint64_t (*smem_pipe)(uint32_t m) = nullptr;
    // Streamed drivers (a ring of stages, warp-specialised): bytes of one stage for a unit of m elements
    // (nullptr: not streamed; the window is smem_pipe(m)) and the block size of fn_pipe.
    uint64_t (*stage_pipe)(uint32_t m) = nullptr;
    uint64_t (*in_stage_pipe)(uint32_t m) = nullptr;   // the input part of a stage (the slot part is the rest)
    int threads_pipe = 256;
};

using Registry = std::vector<KernelEntry>;

// One registration function per (op, dtype) translation unit (instantiate.cu).
void register_op0_dt0(Registry&);
void register_op0_dt1(Registry&);
void register_op0_dt2(Registry&);
void register_op1_dt0(Registry&);
void register_op1_dt1(Registry&);
void register_op1_dt2(Registry&);
void register_op2_dt0(Registry&);
void register_op2_dt1(Registry&);
void register_op2_dt2(Registry&);
void register_op3_dt0(Registry&);
void register_op3_dt1(Registry&);
void register_op3_dt2(Registry&);
void register_op4_dt0(Registry&);
void register_op4_dt1(Registry&);
void register_op4_dt2(Registry&);
void register_op5_dt0(Registry&);
void register_op5_dt1(Registry&);
void register_op5_dt2(Registry&);
void register_op6_dt0(Registry&);
void register_op6_dt1(Registry&);
void register_op6_dt2(Registry&);
void register_op7_dt0(Registry&);
void register_op7_dt1(Registry&);
void register_op7_dt2(Registry&);

}  // namespace dsb
