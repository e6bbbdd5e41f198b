// allgather__direct_replicated_push__credit.cu -- harness-compatible B200 build of the reference algorithm of the same name
// (reference: collectives/allgather__direct_replicated_push__credit.cu:20-29; plain remote stores into every CTA).
// Same contract as the reference file: included by collectives/harness/main.cu with -DCLUSTER_N
// -DMSG_ELEMS -DELEM_T, one cluster per launch, `struct CollectiveSmem` sized for MSG_ELEMS, and
// illegal (N, M) rejected by static_assert. The algorithm itself is dsb::AG_DirectReplicatedPush in
// dsmem_b200_algos.cuh, the same code the C ABI runs on persistent multi-cluster batches.
#include "dsmem_b200_algos.cuh"
using namespace dsmem;   // the harness names kStamps unqualified, as every reference file allows

using DsbAlg = dsb::AG_DirectReplicatedPush<CLUSTER_N, ELEM_T, dsmem::Sum>;
static_assert(DsbAlg::legal(MSG_ELEMS), "N/M constraint of allgather__direct_replicated_push__credit (see dsb::AG_DirectReplicatedPush::legal)");

struct CollectiveSmem {
    __align__(128) unsigned char raw[DsbAlg::smem_bytes(MSG_ELEMS)];
};

__global__ void __cluster_dims__(CLUSTER_N, 1, 1)
collective_kernel(const ELEM_T* in, ELEM_T* out, unsigned long long* ts, unsigned* smid_out) {
    dsb::run_single<DsbAlg>(in, out, ts, smid_out, MSG_ELEMS, (uint32_t)sizeof(CollectiveSmem));
}
