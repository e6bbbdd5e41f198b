// instantiate.cu -- compiled once per (op, dtype) with -DDSB_OP=<0..7> -DDSB_DT=<0..2>; instantiates
// batch_kernel<Alg<N, T, Sum>> for every algorithm of that op and every cluster size the algorithm's
// static constraints allow, and registers them for the C ABI.
#include "../collectives/dsmem_b200_algos.cuh"
#include "registry.h"

#ifndef DSB_OP
#error "compile with -DDSB_OP=<0 allreduce|1 allgather|2 reducescatter|3 alltoall|4 broadcast|5 reduce|6 gather|7 scatter>"
#endif
#ifndef DSB_DT
#error "compile with -DDSB_DT=<0 f32|1 bf16|2 i32>"
#endif

#if DSB_DT == 0
using ElemT = float;
#elif DSB_DT == 1
using ElemT = __nv_bfloat16;
#else
using ElemT = int;
#endif

namespace dsb {
namespace {

template <class A>
bool legal_fn(uint32_t m) {
    return A::legal(m);
}
template <class A>
uint64_t smem_fn(uint32_t m) {
    return A::smem_bytes(m);
}

// Algorithm ids (dsmem_alg in include/dsmem_b200.h).
enum : int {
    kRing = 1, kRecursiveDoubling = 2, kShiftAccBulk = 3, kShiftAccAtomic = 4, kDirectReplicatedPush = 5,
    kPullRsPushAg = 6, kRabenseifner = 7, kOneShotPull = 8, kTwoShotPush = 9, kReduceBcastBinomial = 10,
    kAtomicAllPush = 11, kMesh2D = 12, kDirectShift = 13, kBruck = 14, kDirectPull = 15,
    kGatherBcastBinomial = 16, kRecursiveHalving = 17, kDirectPush = 18, kPairwiseExchange = 19,
    kPairwiseXor = 20, kShift = 21, kRsPushGlobalAg = 22, kRingCredit = 23, kRecursiveDoublingCredit = 24,
    kBinomial = 25, kBruckCredit = 26, kRecursiveHalvingCredit = 27, kRabenseifnerCredit = 28,
    kPairwiseXorCredit = 29, kBinomialCredit = 30, kShiftAccBulkCredit = 31
};

template <template <int, typename, class> class A, int N>
void add(Registry& r, int alg) {
    using Alg = A<N, ElemT, Sum>;
    r.push_back(KernelEntry{DSB_OP, alg, DSB_DT, N, (int)sizeof(ElemT),
                            reinterpret_cast<const void*>(&batch_kernel<Alg>), &legal_fn<Alg>, &smem_fn<Alg>});
}
template <template <int, typename, class> class A>
void add_all_n(Registry& r, int alg) {
    add<A, 2>(r, alg);
    add<A, 4>(r, alg);
    add<A, 8>(r, alg);
    add<A, 16>(r, alg);
}

// Attach the pipelined batch driver P<N> to the entry of (alg, N) just registered.
template <template <int, typename, class> class P, int N>
void add_pipelined(Registry& r, int alg) {
    using PP = P<N, ElemT, Sum>;
    for (KernelEntry& e : r)
        if (e.op == 0 && e.alg == alg && e.dtype == DSB_DT && e.n == N) {
            e.fn_pipe = reinterpret_cast<const void*>(&two_shot_pipelined_kernel<PP>);
            e.smem_pipe = &smem_fn<PP>;
        }
}
template <class A>
uint64_t stage_fn(uint32_t m) {
    return A::stage_bytes(m);
}
template <class A>
uint64_t in_stage_fn(uint32_t m) {
    return A::in_stage_bytes(m);
}
// Attach the streamed batch driver P<N> to the entry of (this op, alg, N): the AllReduce's is
// rs_global_ag_stream_kernel, the other ops' collective_stream_kernel (the same body).
template <template <int, typename, class> class P, int N>
void add_streamed(Registry& r, int alg) {
    using PP = P<N, ElemT, Sum>;
    const void* fn = PP::kOp == OpKind::AllReduce ? reinterpret_cast<const void*>(&rs_global_ag_stream_kernel<PP>)
                                                   : reinterpret_cast<const void*>(&collective_stream_kernel<PP>);
    for (KernelEntry& e : r)
        if (e.op == DSB_OP && e.alg == alg && e.dtype == DSB_DT && e.n == N) {
            e.fn_pipe = fn;
            e.smem_pipe = &smem_fn<PP>;
            e.stage_pipe = &stage_fn<PP>;
            e.in_stage_pipe = &in_stage_fn<PP>;
            e.threads_pipe = PP::kThreads;
        }
}
template <template <int, typename, class> class P>
void add_streamed_all_n(Registry& r, int alg) {
    add_streamed<P, 2>(r, alg);
    add_streamed<P, 4>(r, alg);
    add_streamed<P, 8>(r, alg);
    add_streamed<P, 16>(r, alg);
}
template <template <int, typename, class> class P>
void add_pipelined_all_n(Registry& r, int alg) {
    add_pipelined<P, 2>(r, alg);
    add_pipelined<P, 4>(r, alg);
    add_pipelined<P, 8>(r, alg);
    add_pipelined<P, 16>(r, alg);
}

}  // namespace

#define DSB_CAT3(a, b, c, d) a##b##c##d
#define DSB_REG_NAME(op, dt) DSB_CAT3(register_op, op, _dt, dt)

void DSB_REG_NAME(DSB_OP, DSB_DT)(Registry& r) {
#if DSB_OP == 0
    add_all_n<AR_RecursiveDoubling>(r, kRecursiveDoubling);
    add<AR_ShiftAccumulateBulk, 4>(r, kShiftAccBulk);
    add<AR_ShiftAccumulateBulkCredit, 4>(r, kShiftAccBulkCredit);
    add<AR_ShiftAccumulateAtomic, 2>(r, kShiftAccAtomic);
    add<AR_ShiftAccumulateAtomic, 4>(r, kShiftAccAtomic);
    add_all_n<AR_DirectReplicatedPush>(r, kDirectReplicatedPush);
    add_all_n<AR_PullRsPushAg>(r, kPullRsPushAg);
    add_all_n<AR_Ring>(r, kRing);
    add_all_n<AR_Rabenseifner>(r, kRabenseifner);
    add_all_n<AR_OneShotPull>(r, kOneShotPull);
    add_all_n<AR_TwoShotPush>(r, kTwoShotPush);
    add_pipelined_all_n<AR_TwoShotPipelined>(r, kTwoShotPush);
    add_all_n<AR_RsPushGlobalAg>(r, kRsPushGlobalAg);
    add_streamed_all_n<AR_RsGlobalAgStream>(r, kRsPushGlobalAg);
    add_all_n<AR_ReduceBcastBinomial>(r, kReduceBcastBinomial);
    add_all_n<AR_AtomicAllPush>(r, kAtomicAllPush);
    add_all_n<AR_Mesh2D>(r, kMesh2D);
    add<AR_RingCredit, 2>(r, kRingCredit);   // 2 (N - 1) barriers: N <= 8
    add<AR_RingCredit, 4>(r, kRingCredit);
    add<AR_RingCredit, 8>(r, kRingCredit);
    add_all_n<AR_RecursiveDoublingCredit>(r, kRecursiveDoublingCredit);
    add_all_n<AR_RabenseifnerCredit>(r, kRabenseifnerCredit);
    add_all_n<AR_ReduceBcastBinomialCredit>(r, kBinomialCredit);
#elif DSB_OP == 1
    add_all_n<AG_RecursiveDoubling>(r, kRecursiveDoubling);
    add_all_n<AG_DirectShift>(r, kDirectShift);
    add_all_n<AG_DirectReplicatedPush>(r, kDirectReplicatedPush);
    add_all_n<AG_Ring>(r, kRing);
    add_all_n<AG_Bruck>(r, kBruck);
    add_all_n<AG_DirectPull>(r, kDirectPull);
    add_all_n<AG_GatherBcastBinomial>(r, kGatherBcastBinomial);
    add_all_n<AG_RingCredit>(r, kRingCredit);
    add_all_n<AG_RecursiveDoublingCredit>(r, kRecursiveDoublingCredit);
    add_all_n<AG_BruckCredit>(r, kBruckCredit);
    add_all_n<AG_GatherBcastBinomialCredit>(r, kBinomialCredit);
    add_streamed_all_n<AG_ReplicatedPushStream>(r, kDirectReplicatedPush);
#elif DSB_OP == 2
    add_all_n<RS_Ring>(r, kRing);
    add_all_n<RS_RecursiveHalving>(r, kRecursiveHalving);
    add_all_n<RS_DirectPush>(r, kDirectPush);
    add_all_n<RS_DirectPull>(r, kDirectPull);
    add_all_n<RS_RingCredit>(r, kRingCredit);
    add_all_n<RS_RecursiveHalvingCredit>(r, kRecursiveHalvingCredit);
    add_streamed_all_n<RS_DirectPushStream>(r, kDirectPush);
#elif DSB_OP == 4
    add_all_n<BC_DirectPush>(r, kDirectPush);
    add_all_n<BC_DirectPull>(r, kDirectPull);
    add_all_n<BC_Binomial>(r, kBinomial);
#elif DSB_OP == 5
    add_all_n<RD_DirectPush>(r, kDirectPush);
    add_all_n<RD_DirectPull>(r, kDirectPull);
    add_all_n<RD_Binomial>(r, kBinomial);
#elif DSB_OP == 6
    add_all_n<GA_DirectPush>(r, kDirectPush);
    add_all_n<GA_DirectPull>(r, kDirectPull);
    add_all_n<GA_Binomial>(r, kBinomial);
#elif DSB_OP == 7
    add_all_n<SC_DirectPush>(r, kDirectPush);
    add_all_n<SC_DirectPull>(r, kDirectPull);
    add_all_n<SC_Binomial>(r, kBinomial);
#elif DSB_OP == 3
    add<A2A_PairwiseExchange, 2>(r, kPairwiseExchange);
    add_all_n<A2A_DirectPush>(r, kDirectPush);
    add_all_n<A2A_PairwiseXor>(r, kPairwiseXor);
    add_all_n<A2A_Shift>(r, kShift);
    add_all_n<A2A_Bruck>(r, kBruck);
    add_all_n<A2A_PairwiseXorCredit>(r, kPairwiseXorCredit);
    add_all_n<A2A_BruckCredit>(r, kBruckCredit);
    add_all_n<A2A_DirectPull>(r, kDirectPull);
    add_streamed_all_n<A2A_DirectPushStream>(r, kDirectPush);
#endif
}

}  // namespace dsb
