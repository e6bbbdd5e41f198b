// dsmem_b200_algos.cuh -- the DSMEM collective catalogue for B200 (sm_100a), one template per algorithm.
//
// Every algorithm of the reference catalogue (collectives/<op>__<alg>__<src>.cu, 29 files) is a struct
//   template <int N, typename T, class Op> struct <Alg> {
//     static constexpr OpKind kOp;  static constexpr int kBars;           // op and mbarriers used
//     static constexpr bool   legal(uint32_t M);                           // N/M constraints
//     static constexpr uint32_t smem_bytes(uint32_t M);                    // dynamic smem of one CTA
//     static __device__ void load(Ctx&, const T* g, uint32_t M);          // HBM -> smem of this rank
//     static __device__ void exec(Ctx&, uint32_t M);                      // the collective proper
//     static __device__ void store(Ctx&, T* g, uint32_t M);               // smem -> HBM of this rank
//   };
// with the message size M (elements per rank block, MSG_ELEMS in the reference) a RUNTIME value, so one
// instantiation serves every payload. Rounds, partners and message sizes follow the reference file named
// in each struct's comment. Two drivers run them:
//   * batch_kernel<A>: persistent clusters; cluster q processes problems q, q + nclusters, ... of a batch
//     (one independent collective per problem, per-cluster offsets from %clusterid), with one entry and
//     one exit cluster barrier per problem.
//   * run_single<A>: the reference harness contract (one cluster per launch, collective_kernel).
// Synchronisation differences from the reference (results identical):
//   * Barriers that only protected buffers against the "next stage" (the reference's trailing
//     cluster_sync inside one-shot pull, direct pulls, replicated push, hpcops' leading sync) are dropped
//     where the driver's exit/entry cluster barrier already gives the same guarantee.
//   * mbarrier waits are deadline-bounded (Ctx::deadline); after a time-out the CTA records the error
//     and later waits of the launch return at once. Every CTA executes the same sequence of
//     barrier.cluster instructions, so a time-out can never turn into a hang.
//   * Bulk pushes check 16-B alignment and the window bounds in the issuing thread and record
//     DSMEM_ERR_BIT_BOUNDS instead of issuing an out-of-range copy.
// Layout of the dynamic shared-memory window: bytes [0, kBarArea) hold up to 15 mbarriers and, at byte
// 120, the end-of-kernel flag word (finish()); data buffers start at kD0 and are 16-B aligned (every
// legal M makes M*sizeof(T) a multiple of 16).
#pragma once
#include "dsmem_primitives.cuh"

namespace dsb {
using namespace dsmem;

enum class OpKind : int {
    AllReduce = 0, AllGather = 1, ReduceScatter = 2, AllToAll = 3, Broadcast = 4, Reduce = 5, Gather = 6, Scatter = 7
};

constexpr uint32_t kBarArea = 128;
constexpr uint32_t kD0 = kBarArea;
constexpr uint32_t kSmemLimit = 232448;   // 227 KiB: the per-block opt-in maximum of sm_100a

__host__ __device__ constexpr bool is_pow2(int n) { return n > 0 && (n & (n - 1)) == 0; }
__host__ __device__ constexpr int ilog2(int n) { return n <= 1 ? 0 : 1 + ilog2(n / 2); }

// --------------------------------------------------------------------------- per-CTA context
struct Ctx {
    unsigned char* sm;                // generic pointer to the dynamic window
    uint32_t sa;                      // its shared::cta address
    uint32_t smem_bytes;              // bytes of the window valid in this launch
    uint32_t rank;                    // %cluster_ctarank
    uint32_t phase;                   // parity bit per mbarrier (bit i <-> barrier i)
    bool dead;                        // a wait timed out: later waits do not block
    unsigned long long wait_limit;    // ns per problem
    unsigned long long deadline;      // %globaltimer value after which waits give up
    unsigned* err;                    // error words [4] (nullptr: this translation unit's dsmem_wait_error)
    uint32_t unit;                    // problem / unit counter of this CTA (error detail)
    Stamps st;

    __device__ __forceinline__ uint32_t bar(int i) const { return sa + 8u * (uint32_t)i; }
    template <class U>
    __device__ __forceinline__ U* ptr(uint32_t off) const { return reinterpret_cast<U*>(sm + off); }
};

__device__ __forceinline__ void report(Ctx& c, unsigned bits) {
    atomicOr(c.err != nullptr ? c.err : &dsmem_wait_error, bits);
}

// Wait for the current phase of barrier i (all threads). Bounded by c.deadline.
// Record a wait that gave up: the error bit, and (first one only, library kernels) a detail word
// 0x80000000 | barrier << 24 | rank << 16 | unit (low 16 bits) in err[1] and the cluster id in err[2].
__device__ __forceinline__ void report_timeout(Ctx& c, int bar_id) {
    report(c, DSMEM_ERR_BIT_TIMEOUT);
    if (c.err != nullptr &&
        atomicCAS(c.err + 1, 0u, 0x80000000u | ((uint32_t)bar_id & 0x7fu) << 24 | (c.rank & 0xffu) << 16 |
                                     (c.unit & 0xffffu)) == 0u)
        c.err[2] = cluster_id();
}

__device__ __forceinline__ void wait(Ctx& c, int i) {
    const uint32_t par = (c.phase >> i) & 1u;
    c.phase ^= 1u << i;
    if (c.dead) return;
    if (mbar_try_wait_parity(c.bar(i), par)) return;
    if (!mbar_wait_parity_until(c.bar(i), par, c.deadline)) {
        c.dead = true;
        if ((threadIdx.x & 31) == 0) report_timeout(c, i);
    }
}

// End of a kernel: a CTA whose wait gave up may have stopped waiting for bytes peers still push into
// it. A CTA that gave up sets the flag word (byte 120 of the barrier area) of every CTA of the cluster
// before the final cluster barrier; after it each CTA reads its own flag (no remote access after the
// last barrier), and if any CTA gave up, all of them linger kSettleNs and meet once more, so those
// copies land before any CTA of the cluster exits. flag_init must precede the kernel's first
// cluster barrier.
constexpr uint32_t kFlagOff = 120;
constexpr unsigned long long kSettleNs = 20000000ull;
__device__ __forceinline__ void flag_init(Ctx& c) {
    if (threadIdx.x == 0) *c.ptr<uint32_t>(kFlagOff) = 0u;
}
__device__ __forceinline__ void finish(Ctx& c) {
    const bool dead = __syncthreads_or(c.dead ? 1 : 0) != 0;
    if (dead && threadIdx.x < cluster_size()) st_cluster_u32(mapa(c.sa + kFlagOff, threadIdx.x), 1u);
    cluster_sync();
    if (*c.ptr<volatile uint32_t>(kFlagOff) != 0u) {
        const unsigned long long until = globaltimer() + kSettleNs;
        while (globaltimer() < until) {
        }
        cluster_sync();
    }
}

// Checked bulk push of `bytes` from local window offset `src` to CTA `dst_rank`'s window offset `dst`,
// completing on that CTA's barrier `bi`. One thread.
template <int N>
__device__ __forceinline__ void push(Ctx& c, uint32_t dst_rank, uint32_t dst, uint32_t src, uint32_t bytes, int bi) {
    const bool ok = dst_rank < (uint32_t)N && bytes != 0u && ((dst | src | bytes) & 15u) == 0u && dst >= kD0 &&
                    src >= kD0 && dst + bytes <= c.smem_bytes && src + bytes <= c.smem_bytes;
    if (!ok) {
        report(c, DSMEM_ERR_BIT_BOUNDS);
        return;
    }
    bulk_push(dst_rank, c.sa + dst, c.sa + src, bytes, c.bar(bi));
}

__device__ __forceinline__ void arm(Ctx& c, int bi, uint32_t bytes) { mbar_arrive_expect_tx(c.bar(bi), bytes); }

// --------------------------------------------------------------------------- 16-byte packets
// Arithmetic on 16-byte packets of T. Multi-operand reductions accumulate in Acc (fp32 for bf16, so a
// CTA-local reduction of k operands rounds to bf16 once).
template <typename T, class Op>
struct Pk;

template <class Op>
struct Pk<float, Op> {
    struct Acc {
        float v[4];
    };
    static __device__ __forceinline__ Acc open(uint4 p) {
        return Acc{{__uint_as_float(p.x), __uint_as_float(p.y), __uint_as_float(p.z), __uint_as_float(p.w)}};
    }
    static __device__ __forceinline__ void add(Acc& a, uint4 p) {
        const Op op{};
        a.v[0] = op(a.v[0], __uint_as_float(p.x));
        a.v[1] = op(a.v[1], __uint_as_float(p.y));
        a.v[2] = op(a.v[2], __uint_as_float(p.z));
        a.v[3] = op(a.v[3], __uint_as_float(p.w));
    }
    static __device__ __forceinline__ uint4 close(const Acc& a) {
        return make_uint4(__float_as_uint(a.v[0]), __float_as_uint(a.v[1]), __float_as_uint(a.v[2]),
                          __float_as_uint(a.v[3]));
    }
    static __device__ __forceinline__ uint4 identity() {
        const uint32_t w = __float_as_uint(Op::template identity<float>());
        return make_uint4(w, w, w, w);
    }
};

template <class Op>
struct Pk<int, Op> {
    struct Acc {
        int v[4];
    };
    static __device__ __forceinline__ Acc open(uint4 p) { return Acc{{(int)p.x, (int)p.y, (int)p.z, (int)p.w}}; }
    static __device__ __forceinline__ void add(Acc& a, uint4 p) {
        const Op op{};
        a.v[0] = op(a.v[0], (int)p.x);
        a.v[1] = op(a.v[1], (int)p.y);
        a.v[2] = op(a.v[2], (int)p.z);
        a.v[3] = op(a.v[3], (int)p.w);
    }
    static __device__ __forceinline__ uint4 close(const Acc& a) {
        return make_uint4((uint32_t)a.v[0], (uint32_t)a.v[1], (uint32_t)a.v[2], (uint32_t)a.v[3]);
    }
    static __device__ __forceinline__ uint4 identity() {
        const uint32_t w = (uint32_t)Op::template identity<int>();
        return make_uint4(w, w, w, w);
    }
};

template <class Op>
struct Pk<__nv_bfloat16, Op> {
    struct Acc {
        float v[8];
    };
    static __device__ __forceinline__ float2 f2(uint32_t w) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
    }
    static __device__ __forceinline__ uint32_t b2(float lo, float hi) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    static __device__ __forceinline__ Acc open(uint4 p) {
        Acc a;
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = f2(w[k]);
            a.v[2 * k] = f.x;
            a.v[2 * k + 1] = f.y;
        }
        return a;
    }
    static __device__ __forceinline__ void add(Acc& a, uint4 p) {
        const Op op{};
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = f2(w[k]);
            a.v[2 * k] = op(a.v[2 * k], f.x);
            a.v[2 * k + 1] = op(a.v[2 * k + 1], f.y);
        }
    }
    static __device__ __forceinline__ uint4 close(const Acc& a) {
        return make_uint4(b2(a.v[0], a.v[1]), b2(a.v[2], a.v[3]), b2(a.v[4], a.v[5]), b2(a.v[6], a.v[7]));
    }
    static __device__ __forceinline__ uint4 identity() {
        const float i = Op::template identity<float>();
        const uint32_t w = b2(i, i);
        return make_uint4(w, w, w, w);
    }
};

template <typename T, class Op>
__device__ __forceinline__ uint4 pk_op(uint4 a, uint4 b) {
    auto x = Pk<T, Op>::open(a);
    Pk<T, Op>::add(x, b);
    return Pk<T, Op>::close(x);
}

// dst[u] = a[u] op b[u] for `bytes` bytes (window offsets; all threads).
template <typename T, class Op>
__device__ __forceinline__ void reduce2(const Ctx& c, uint32_t dst, uint32_t a, uint32_t b, uint32_t bytes) {
    const uint4* pa = c.ptr<const uint4>(a);
    const uint4* pb = c.ptr<const uint4>(b);
    uint4* pd = c.ptr<uint4>(dst);
    const uint32_t n = bytes >> 4;
#pragma unroll 4
    for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) pd[u] = pk_op<T, Op>(pa[u], pb[u]);
}

// Global <-> shared copies of whole 16-B units, all threads, streaming cache hints.
__device__ __forceinline__ void g2s(const Ctx& c, uint32_t off, const void* g, uint32_t bytes) {
    const uint4* src = static_cast<const uint4*>(g);
    uint4* dst = c.ptr<uint4>(off);
    const uint32_t n = bytes >> 4, st = blockDim.x;
    uint32_t i = threadIdx.x;
    for (; i + 3u * st < n; i += 4u * st) {
        const uint4 v0 = __ldcs(src + i), v1 = __ldcs(src + i + st), v2 = __ldcs(src + i + 2u * st),
                    v3 = __ldcs(src + i + 3u * st);
        dst[i] = v0;
        dst[i + st] = v1;
        dst[i + 2u * st] = v2;
        dst[i + 3u * st] = v3;
    }
    for (; i < n; i += st) dst[i] = __ldcs(src + i);
}
__device__ __forceinline__ void s2g(const Ctx& c, void* g, uint32_t off, uint32_t bytes) {
    uint4* dst = static_cast<uint4*>(g);
    const uint4* src = c.ptr<const uint4>(off);
    const uint32_t n = bytes >> 4;
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) __stcs(dst + i, src[i]);
}
// Local copy inside the window.
__device__ __forceinline__ void s2s(const Ctx& c, uint32_t dst, uint32_t src, uint32_t bytes) {
    const uint4* s = c.ptr<const uint4>(src);
    uint4* d = c.ptr<uint4>(dst);
    const uint32_t n = bytes >> 4;
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

#define DSB_TRAITS(OPKIND, NBARS)                  \
    static constexpr OpKind kOp = OpKind::OPKIND; \
    static constexpr int kBars = NBARS;           \
    static constexpr int kN = N_;                 \
    using T = T_;                                 \
    using Op = Op_;                               \
    static constexpr uint32_t B = sizeof(T_);

// Sum-only algorithms (hardware remote adds) test the reduction functor with this trait.
template <class Op>
struct IsSum {
    static constexpr bool value = false;
};
template <>
struct IsSum<Sum> {
    static constexpr bool value = true;
};

__host__ __device__ constexpr bool mult16(uint32_t bytes) { return bytes != 0u && (bytes & 15u) == 0u; }
__host__ __device__ constexpr bool fits(uint64_t bytes) { return bytes <= (uint64_t)kSmemLimit; }

// =====================================================================================================
//                                              ALLREDUCE
// Per rank: in[M] -> out[M] = op over ranks.
// =====================================================================================================

// allreduce__recursive_doubling__clusterfusion.cu:27-52. log2 N rounds, stride s = 1,2,..: push the
// running vector to (b+s) mod N's scratch, reduce into the ping-pong buffer, one cluster barrier per round.
template <int N_, typename T_, class Op_>
struct AR_RecursiveDoubling {
    DSB_TRAITS(AllReduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 3ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, scr = kD0 + 2 * MB;
        uint32_t cur = kD0, oth = kD0 + MB;
        int round = 0;
        for (int s = 1; s < N_; s <<= 1, ++round) {
            if (threadIdx.x == 0) {
                arm(c, 0, MB);
                push<N_>(c, (c.rank + s) % N_, scr, cur, MB, 0);
            }
            wait(c, 0);
            reduce2<T, Op>(c, oth, cur, scr, MB);   // cur may still be read by my own outgoing push
            fence_proxy_async_smem();
            cluster_sync();
            const uint32_t t = cur;
            cur = oth;
            oth = t;
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, (ilog2(N_) % 2 == 0) ? kD0 : kD0 + M * B, M * B);
    }
};

// ---- mbarrier-credit ("DSMEM-native") variants: the reference's deferred design (per-round buffers and
// barriers instead of a barrier.cluster per round, collectives/ROADMAP.md:38-45). B200 extensions: same
// schedules and the same arithmetic (operands added in the same order) as the barrier-per-round originals.
// Every round's bytes land in a buffer and on an mbarrier of their own (each used once per problem, between
// the batch driver's entry and exit cluster barriers), and a CTA forwards only what it has itself received
// or reduced, so a round waits for its one incoming copy and nothing else. No buffer that a bulk copy may
// still be reading is written again within the problem.

// Ring AllReduce (allreduce__ring__nccl.cu:25-60 schedule): reduce-scatter rounds s = 0..N-2 push chunk
// (b - s) into slot s of CTA b+1, which adds it into its chunk (b - s - 1); all-gather rounds push the
// owned chunk (b + 1), then each received chunk, into slot s of the all-gather area of CTA b+1. Barriers
// 0..N-2 count the reduce-scatter rounds, N-1..2N-3 the all-gather rounds (so N <= 8).
template <int N_, typename T_, class Op_>
struct AR_RingCredit {
    DSB_TRAITS(AllReduce, 2 * (N_ - 1))
    __host__ __device__ static constexpr bool legal(uint32_t M) {
        return N_ <= 8 && M % N_ == 0 && mult16((M / N_) * B);
    }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + 1ull * M * B + 2ull * (N_ - 1) * (M / N_) * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t CB = (M / N_) * B, rs0 = kD0 + M * B, ag0 = rs0 + (N_ - 1) * CB, next = (c.rank + 1) % N_;
        if (threadIdx.x == 0)
            for (int k = 0; k < 2 * (N_ - 1); ++k) arm(c, k, CB);
        int round = 0;
        for (int s = 0; s < N_ - 1; ++s, ++round) {
            const uint32_t send_c = (c.rank + N_ - s) % N_, recv_c = (c.rank + 2 * N_ - s - 1) % N_;
            if (threadIdx.x == 0) push<N_>(c, next, rs0 + s * CB, kD0 + send_c * CB, CB, s);
            wait(c, s);
            reduce2<T, Op>(c, kD0 + recv_c * CB, kD0 + recv_c * CB, rs0 + s * CB, CB);
            fence_proxy_async_smem();
            __syncthreads();   // the reduced chunk is whole before thread 0 pushes it on
            c.st.round(round);
        }
        for (int s = 0; s < N_ - 1; ++s, ++round) {
            const uint32_t src = s == 0 ? kD0 + ((c.rank + 1) % N_) * CB : ag0 + (s - 1) * CB;
            if (threadIdx.x == 0) push<N_>(c, next, ag0 + s * CB, src, CB, N_ - 1 + s);
            wait(c, N_ - 1 + s);
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        const uint32_t C = M / N_, CB = C * B, ag0 = kD0 + M * B + (N_ - 1) * CB;
        const uint32_t own = (c.rank + 1) % N_;
        s2g(c, g + own * C, kD0 + own * CB, CB);
        for (int s = 0; s < N_ - 1; ++s) s2g(c, g + ((c.rank + N_ - s) % N_) * C, ag0 + s * CB, CB);
    }
};

// Recursive-doubling AllReduce (allreduce__recursive_doubling__clusterfusion.cu:27-52 schedule): round k
// pushes the running vector to CTA b + 2^k into its buffer k, which then holds buffer k + running vector
// and becomes the running vector pushed in round k + 1. log2 N buffers and barriers.
template <int N_, typename T_, class Op_>
struct AR_RecursiveDoublingCredit {
    DSB_TRAITS(AllReduce, ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + (1ull + ilog2(N_)) * M * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k) arm(c, k, MB);
        uint32_t cur = kD0;
        for (int k = 0; k < L; ++k) {
            const uint32_t buf = kD0 + (uint32_t)(k + 1) * MB;
            if (threadIdx.x == 0) push<N_>(c, (c.rank + (1u << k)) % N_, buf, cur, MB, k);
            wait(c, k);
            reduce2<T, Op>(c, buf, cur, buf, MB);   // the reference's order: running vector + received
            fence_proxy_async_smem();
            __syncthreads();   // the new running vector is whole before thread 0 pushes it
            cur = buf;
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + (uint32_t)ilog2(N_) * M * B, M * B);
    }
};

// allreduce__shift_accumulate_bulk__clusterfusion.cu:29-51 (as shipped: only N == 4 reduces correctly).
// Rounds i = 1..N-2: push the running vector to (b+i) mod N, add what arrives from (b-i).
template <int N_, typename T_, class Op_>
struct AR_ShiftAccumulateBulk {
    DSB_TRAITS(AllReduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return N_ == 4 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 3ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, scr = kD0 + 2 * MB;
        uint32_t cur = kD0, oth = kD0 + MB;
        for (int i = 1; i < N_ - 1; ++i) {
            if (threadIdx.x == 0) {
                arm(c, 0, MB);
                push<N_>(c, (c.rank + i) % N_, scr, cur, MB, 0);
            }
            wait(c, 0);
            reduce2<T, Op>(c, oth, cur, scr, MB);
            fence_proxy_async_smem();
            cluster_sync();
            const uint32_t t = cur;
            cur = oth;
            oth = t;
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, ((N_ - 2) % 2 == 0) ? kD0 : kD0 + M * B, M * B);
    }
};

// Shift-accumulate bulk (allreduce__shift_accumulate_bulk__clusterfusion.cu:29-51 schedule, N == 4) with a buffer
// and an mbarrier per round: round i pushes the running vector into buffer i of CTA b + i (barrier i - 1), which
// then holds running vector + received and becomes the running vector; the original's operand order.
template <int N_, typename T_, class Op_>
struct AR_ShiftAccumulateBulkCredit {
    DSB_TRAITS(AllReduce, N_ - 2)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return N_ == 4 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (N_ - 1ull) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int i = 1; i < N_ - 1; ++i) arm(c, i - 1, MB);
        uint32_t cur = kD0;
        for (int i = 1; i < N_ - 1; ++i) {
            const uint32_t buf = kD0 + (uint32_t)i * MB;
            if (threadIdx.x == 0) push<N_>(c, (c.rank + i) % N_, buf, cur, MB, i - 1);
            wait(c, i - 1);
            reduce2<T, Op>(c, buf, cur, buf, MB);
            fence_proxy_async_smem();
            __syncthreads();   // the new running vector is whole before thread 0 pushes it
            cur = buf;
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + (N_ - 2u) * M * B, M * B);
    }
};

// Accumulator element of the remote-atomic algorithms: bf16 sums accumulate in fp32 (a chain of N-1
// remote adds rounded to bf16 after each add drifted beyond the bf16 tolerance at N = 16); f32 and int32
// accumulate in their own type. Values are widened on load and narrowed on store.
template <typename T>
struct AccOf {
    using type = T;
};
template <>
struct AccOf<__nv_bfloat16> {
    using type = float;
};

// Remote element-wise add of one 16-byte packet of accumulator elements into a peer (fire-and-forget).
__device__ __forceinline__ void red_add_packet(float, uint32_t a, uint4 v) {
    red_cluster_add_f32(a, __uint_as_float(v.x));
    red_cluster_add_f32(a + 4, __uint_as_float(v.y));
    red_cluster_add_f32(a + 8, __uint_as_float(v.z));
    red_cluster_add_f32(a + 12, __uint_as_float(v.w));
}
__device__ __forceinline__ void red_add_packet(int, uint32_t a, uint4 v) {
    red_cluster_add_u32(a, v.x);
    red_cluster_add_u32(a + 4, v.y);
    red_cluster_add_u32(a + 8, v.z);
    red_cluster_add_u32(a + 12, v.w);
}

// Global T[M] -> shared accumulator array (widening bf16 to fp32), all threads.
template <typename T>
__device__ __forceinline__ void g2s_acc(const Ctx& c, uint32_t off, const T* g, uint32_t M) {
    if constexpr (sizeof(typename AccOf<T>::type) == sizeof(T)) {
        g2s(c, off, g, M * (uint32_t)sizeof(T));
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(g);
        uint4* dst = c.ptr<uint4>(off);
        const uint32_t n = (M * (uint32_t)sizeof(T)) >> 4;   // 8 bf16 per packet -> 2 fp32 packets
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const auto a = Pk<__nv_bfloat16, Sum>::open(__ldcs(src + i));
            dst[2 * i] = make_uint4(__float_as_uint(a.v[0]), __float_as_uint(a.v[1]), __float_as_uint(a.v[2]),
                                    __float_as_uint(a.v[3]));
            dst[2 * i + 1] = make_uint4(__float_as_uint(a.v[4]), __float_as_uint(a.v[5]), __float_as_uint(a.v[6]),
                                        __float_as_uint(a.v[7]));
        }
    }
}
// Shared accumulator array -> global T[M] (narrowing fp32 to bf16), all threads.
template <typename T>
__device__ __forceinline__ void s2g_acc(const Ctx& c, T* g, uint32_t off, uint32_t M) {
    if constexpr (sizeof(typename AccOf<T>::type) == sizeof(T)) {
        s2g(c, g, off, M * (uint32_t)sizeof(T));
    } else {
        const uint4* src = c.ptr<const uint4>(off);
        uint4* dst = reinterpret_cast<uint4*>(g);
        const uint32_t n = (M * (uint32_t)sizeof(T)) >> 4;
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const uint4 lo = src[2 * i], hi = src[2 * i + 1];
            typename Pk<__nv_bfloat16, Sum>::Acc a{{__uint_as_float(lo.x), __uint_as_float(lo.y), __uint_as_float(lo.z),
                                                    __uint_as_float(lo.w), __uint_as_float(hi.x), __uint_as_float(hi.y),
                                                    __uint_as_float(hi.z), __uint_as_float(hi.w)}};
            __stcs(dst + i, Pk<__nv_bfloat16, Sum>::close(a));
        }
    }
}

// allreduce__shift_accumulate_atomic__clusterfusion.cu:27-40 (sum only; N in {2,4}; 1 round at N = 2,
// N-2 rounds at N = 4). Per round: snapshot the running value, barrier, remote add of the snapshot into
// (b+i) mod N, barrier.
template <int N_, typename T_, class Op_>
struct AR_ShiftAccumulateAtomic {
    DSB_TRAITS(AllReduce, 0)
    using AccT = typename AccOf<T_>::type;
    static constexpr uint32_t AB = sizeof(AccT);
    __host__ __device__ static constexpr bool legal(uint32_t M) {
        return (N_ == 2 || N_ == 4) && mult16(M * B) && IsSum<Op_>::value;
    }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * M * AB; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s_acc<T>(c, kD0, g, M); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MA = M * AB, val = kD0, snap = kD0 + MA, n = MA >> 4;
        constexpr int rounds = (N_ == 2) ? 1 : N_ - 2;
        for (int i = 1; i <= rounds; ++i) {
            s2s(c, snap, val, MA);
            cluster_sync();   // every CTA snapshotted before any remote add lands in its `val`
            const uint32_t peer_val = mapa(c.sa + val, (c.rank + i) % N_);
            const uint4* sp = c.ptr<const uint4>(snap);
            for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) red_add_packet(AccT{}, peer_val + 16u * u, sp[u]);
            cluster_sync();   // remote adds complete and visible
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g_acc<T>(c, g, kD0, M);
    }
};

// allreduce__direct_replicated_push__credit.cu:26-44. Plain remote 16-B stores of my vector into
// slot[b] of every CTA (self included), one cluster barrier, local reduction of the N slots.
template <int N_, typename T_, class Op_>
struct AR_DirectReplicatedPush {
    DSB_TRAITS(AllReduce, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (N_ + 2ull) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, mine = kD0, slots = kD0 + MB, res = kD0 + (N_ + 1) * MB, n = MB >> 4;
        const uint4* pm = c.ptr<const uint4>(mine);
        for (uint32_t idx = threadIdx.x; idx < N_ * n; idx += blockDim.x) {
            const uint32_t p = idx / n, u = idx - p * n;
            st_cluster_v4(mapa(c.sa + slots + c.rank * MB + 16u * u, p), pm[u]);
        }
        cluster_sync();   // all pushed partials visible
        c.st.round(0);
        const uint4* ps = c.ptr<const uint4>(slots);
        uint4* pr = c.ptr<uint4>(res);
        for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
            uint4 v[N_];
#pragma unroll
            for (int r = 0; r < N_; ++r) v[r] = ps[r * n + u];
            auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
            for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
            pr[u] = Pk<T, Op>::close(a);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + (N_ + 1) * M * B, M * B);
    }
};

// Unit helpers for the lane-group algorithm: U = uint4 (16-B packet) or a single element.
template <typename T, class Op, typename U>
struct Unit;
template <typename T, class Op>
struct Unit<T, Op, uint4> {
    static __device__ __forceinline__ uint4 ld(uint32_t a) { return ld_cluster_v4(a); }
    static __device__ __forceinline__ void st(uint32_t a, uint4 v) { st_cluster_v4(a, v); }
    static __device__ __forceinline__ uint4 op(uint4 a, uint4 b) { return pk_op<T, Op>(a, b); }
    static __device__ __forceinline__ uint4 identity() { return Pk<T, Op>::identity(); }
    static __device__ __forceinline__ uint4 shfl_xor(uint4 v, int off, int width) {
        return make_uint4(__shfl_xor_sync(0xffffffffu, v.x, off, width), __shfl_xor_sync(0xffffffffu, v.y, off, width),
                          __shfl_xor_sync(0xffffffffu, v.z, off, width), __shfl_xor_sync(0xffffffffu, v.w, off, width));
    }
};
template <class Op>
struct Unit<float, Op, float> {
    static __device__ __forceinline__ float ld(uint32_t a) { return ld_cluster_f32(a); }
    static __device__ __forceinline__ void st(uint32_t a, float v) { st_cluster_f32(a, v); }
    static __device__ __forceinline__ float op(float a, float b) { return Op{}(a, b); }
    static __device__ __forceinline__ float identity() { return Op::template identity<float>(); }
    static __device__ __forceinline__ float shfl_xor(float v, int off, int w) { return __shfl_xor_sync(0xffffffffu, v, off, w); }
};
template <class Op>
struct Unit<int, Op, int> {
    static __device__ __forceinline__ int ld(uint32_t a) { return (int)ld_cluster_u32(a); }
    static __device__ __forceinline__ void st(uint32_t a, int v) { st_cluster_u32(a, (uint32_t)v); }
    static __device__ __forceinline__ int op(int a, int b) { return Op{}(a, b); }
    static __device__ __forceinline__ int identity() { return Op::template identity<int>(); }
    static __device__ __forceinline__ int shfl_xor(int v, int off, int w) { return __shfl_xor_sync(0xffffffffu, v, off, w); }
};
template <class Op>
struct Unit<__nv_bfloat16, Op, __nv_bfloat16> {
    static __device__ __forceinline__ __nv_bfloat16 ld(uint32_t a) { return __ushort_as_bfloat16(ld_cluster_u16(a)); }
    static __device__ __forceinline__ void st(uint32_t a, __nv_bfloat16 v) { st_cluster_u16(a, __bfloat16_as_ushort(v)); }
    static __device__ __forceinline__ __nv_bfloat16 op(__nv_bfloat16 a, __nv_bfloat16 b) {
        return __float2bfloat16_rn(Op{}(__bfloat162float(a), __bfloat162float(b)));
    }
    static __device__ __forceinline__ __nv_bfloat16 identity() {
        return __float2bfloat16_rn(Op::template identity<float>());
    }
    static __device__ __forceinline__ __nv_bfloat16 shfl_xor(__nv_bfloat16 v, int off, int w) {
        return __ushort_as_bfloat16((unsigned short)__shfl_xor_sync(0xffffffffu, (int)__bfloat16_as_ushort(v), off, w));
    }
};

// allreduce__pull_reduce_scatter_push_allgather__hpcops.cu:27-49. CTA b owns elements [b*C, (b+1)*C),
// C = M/N. Groups of N lanes: lane j of a group loads the owned unit from CTA j, the group reduces with
// __shfl_xor, lane j stores the total back into CTA j. One round.
template <int N_, typename T_, class Op_>
struct AR_PullRsPushAg {
    DSB_TRAITS(AllReduce, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) {
        return (32 % N_) == 0 && M % N_ == 0 && mult16(M * B);
    }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    template <typename U>
    static __device__ void run_units(Ctx& c, uint32_t units_per_rank) {
        using X = Unit<T, Op, U>;
        const uint32_t total = units_per_rank * N_;
        for (uint32_t base = 0; base < total; base += blockDim.x) {   // same trip count on every thread
            const uint32_t linear = base + threadIdx.x;
            const bool active = linear < total;
            const uint32_t e = c.rank * units_per_rank + (active ? linear : 0u) / N_;
            const uint32_t peer = linear % N_;
            const uint32_t a = mapa(c.sa + kD0 + e * (uint32_t)sizeof(U), peer);
            U v = active ? X::ld(a) : X::identity();
#pragma unroll
            for (int off = N_ / 2; off > 0; off >>= 1) v = X::op(v, X::shfl_xor(v, off, N_));
            if (active) X::st(a, v);
        }
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t CB = (M / N_) * B;
        if ((CB & 15u) == 0u) run_units<uint4>(c, CB >> 4);
        else run_units<T>(c, M / N_);
        c.st.round(0);
        cluster_sync();   // every copy holds the total before anyone stores
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// allreduce__ring__nccl.cu:25-60. Ring reduce-scatter (N-1 steps: push chunk (b-s) to the successor's
// scratch, add chunk (b-s-1)) then ring all-gather (N-1 steps forwarding into the same slot).
template <int N_, typename T_, class Op_>
struct AR_Ring {
    DSB_TRAITS(AllReduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return M % N_ == 0 && mult16((M / N_) * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B + (M / N_) * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t CB = (M / N_) * B, scr = kD0 + M * B, next = (c.rank + 1) % N_;
        int round = 0;
        for (int s = 0; s < N_ - 1; ++s, ++round) {
            const uint32_t send_c = (c.rank + N_ - s) % N_, recv_c = (c.rank + 2 * N_ - s - 1) % N_;
            if (threadIdx.x == 0) {
                arm(c, 0, CB);
                push<N_>(c, next, scr, kD0 + send_c * CB, CB, 0);
            }
            wait(c, 0);
            reduce2<T, Op>(c, kD0 + recv_c * CB, kD0 + recv_c * CB, scr, CB);
            fence_proxy_async_smem();
            cluster_sync();   // scratch free again, updated chunk visible to the next push
            c.st.round(round);
        }
        for (int s = 0; s < N_ - 1; ++s, ++round) {
            const uint32_t send_c = (c.rank + 1 + N_ - s) % N_;
            if (threadIdx.x == 0) {
                arm(c, 0, CB);
                push<N_>(c, next, kD0 + send_c * CB, kD0 + send_c * CB, CB, 0);
            }
            wait(c, 0);
            cluster_sync();   // received chunk stable before it is forwarded
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// allreduce__rabenseifner__mpich.cu:25-67. Recursive-halving reduce-scatter with XOR partners
// (d = N/2 .. 1), then recursive-doubling all-gather of the live ranges (d = 1 .. N/2).
template <int N_, typename T_, class Op_>
struct AR_Rabenseifner {
    DSB_TRAITS(AllReduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) {
        return is_pow2(N_) && M % N_ == 0 && mult16((M / N_) * B);
    }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B + (M / 2) * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t scr = kD0 + M * B;
        uint32_t lo = 0, hi = M;
        int round = 0;
        for (int d = N_ / 2; d >= 1; d >>= 1, ++round) {
            const uint32_t partner = c.rank ^ (uint32_t)d, mid = (lo + hi) / 2, len = hi - mid;
            const bool upper = (c.rank & (uint32_t)d) != 0u;
            const uint32_t send_lo = upper ? lo : mid, keep_lo = upper ? mid : lo;
            if (threadIdx.x == 0) {
                arm(c, 0, len * B);
                push<N_>(c, partner, scr, kD0 + send_lo * B, len * B, 0);
            }
            wait(c, 0);
            reduce2<T, Op>(c, kD0 + keep_lo * B, kD0 + keep_lo * B, scr, len * B);
            lo = keep_lo;
            hi = keep_lo + len;
            fence_proxy_async_smem();
            cluster_sync();
            c.st.round(round);
        }
        for (int d = 1; d < N_; d <<= 1, ++round) {
            const uint32_t partner = c.rank ^ (uint32_t)d, len = hi - lo;
            if (threadIdx.x == 0) {
                arm(c, 0, len * B);
                push<N_>(c, partner, kD0 + lo * B, kD0 + lo * B, len * B, 0);
            }
            wait(c, 0);
            if (c.rank & (uint32_t)d) lo -= len;
            else hi += len;
            cluster_sync();
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Rabenseifner (allreduce__rabenseifner__mpich.cu:25-67 schedule) with a buffer and an mbarrier per round: the
// reduce-scatter half sent in round k lands in the partner's scratch range k (M/2, M/4, .. elements) on barrier
// k; all-gather round k pushes the live range straight into the partner's vector on barrier log2 N + k. That
// range is exactly what the partner sent this CTA in the reduce-scatter round of the same distance, which this
// CTA had received (and waited for) before: no copy still reads it. Same halves and operand order as the
// original.
template <int N_, typename T_, class Op_>
struct AR_RabenseifnerCredit {
    DSB_TRAITS(AllReduce, 2 * ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) {
        return is_pow2(N_) && N_ >= 2 && M % N_ == 0 && mult16((M / N_) * B);
    }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + 1ull * M * B + (1ull * M - M / N_) * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k) {
                arm(c, k, (M >> (k + 1)) * B);
                arm(c, L + k, ((M / N_) << k) * B);
            }
        uint32_t lo = 0, hi = M, scr = kD0 + M * B;
        int k = 0;
        for (int d = N_ / 2; d >= 1; d >>= 1, ++k) {
            const uint32_t partner = c.rank ^ (uint32_t)d, mid = (lo + hi) / 2, len = hi - mid;
            const bool upper = (c.rank & (uint32_t)d) != 0u;
            const uint32_t send_lo = upper ? lo : mid, keep_lo = upper ? mid : lo;
            if (threadIdx.x == 0) push<N_>(c, partner, scr, kD0 + send_lo * B, len * B, k);
            wait(c, k);
            reduce2<T, Op>(c, kD0 + keep_lo * B, kD0 + keep_lo * B, scr, len * B);
            fence_proxy_async_smem();
            __syncthreads();   // the kept half is reduced before thread 0 sends part of it on
            lo = keep_lo;
            hi = keep_lo + len;
            scr += len * B;
            c.st.round(k);
        }
        for (int d = 1, j = 0; d < N_; d <<= 1, ++j) {
            const uint32_t partner = c.rank ^ (uint32_t)d, len = hi - lo;
            if (threadIdx.x == 0) push<N_>(c, partner, kD0 + lo * B, kD0 + lo * B, len * B, L + j);
            wait(c, L + j);
            if (c.rank & (uint32_t)d) lo -= len;
            else hi += len;
            c.st.round(L + j);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// allreduce__one_shot_pull__trtllm.cu:22-44. Every CTA loads all N vectors (16-B ld.shared::cluster,
// all N loads of a packet in flight together) and reduces in rank order, so every CTA ends with the
// same bits.
template <int N_, typename T_, class Op_>
struct AR_OneShotPull {
    DSB_TRAITS(AllReduce, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, n = MB >> 4;
        uint4* pr = c.ptr<uint4>(kD0 + MB);
        uint32_t base[N_];
#pragma unroll
        for (int r = 0; r < N_; ++r) base[r] = mapa(c.sa + kD0, r);
        for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
            uint4 v[N_];
#pragma unroll
            for (int r = 0; r < N_; ++r) v[r] = ld_cluster_v4(base[r] + 16u * u);
            auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
            for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
            pr[u] = Pk<T, Op>::close(a);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + M * B, M * B);
    }
};

// allreduce__two_shot_push__trtllm.cu:23-59. Shot 1: bulk-push chunk j into slot[b] of CTA j for all
// j != b (one aggregate barrier), reduce my chunk. Shot 2: bulk-push my reduced chunk into position b
// of every peer. No cluster barrier between the shots.
template <int N_, typename T_, class Op_>
struct AR_TwoShotPush {
    DSB_TRAITS(AllReduce, 2)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return M % N_ == 0 && mult16((M / N_) * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    // Shot 1: thread 0 pushes chunk j into slot [b] of CTA j (bulk copies). Shot 2 is fused with the reduction:
    // each thread stores the 16-byte units it reduced straight into every peer's copy of chunk b (st.async on
    // the peer's barrier 1), with no block barrier or bulk copy between the two shots. Both barriers are armed
    // before this CTA's first push, so no peer's second shot can reach barrier 1 before its arm. A peer's
    // region for chunk b is free once my barrier 0 completed: its shot-1 copy out of it had landed here.
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t CB = (M / N_) * B, slots = kD0 + M * B, n = CB >> 4;
        if (threadIdx.x == 0) {
            arm(c, 0, (N_ - 1) * CB);
            arm(c, 1, (N_ - 1) * CB);
            for (uint32_t j = 1; j < (uint32_t)N_; ++j) {
                const uint32_t dst = (c.rank + j) % N_;
                push<N_>(c, dst, slots + c.rank * CB, kD0 + dst * CB, CB, 0);
            }
        }
        wait(c, 0);   // every peer's partial of my chunk has landed (so their reads of it are done)
        const uint32_t own = kD0 + c.rank * CB;
        uint4* mine = c.ptr<uint4>(own);
        const uint4* ps = c.ptr<const uint4>(slots);
        for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
            uint4 v[N_];
#pragma unroll
            for (int r = 0; r < N_; ++r) v[r] = (r == (int)c.rank) ? mine[u] : ps[r * n + u];
            auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
            for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
            const uint4 red = Pk<T, Op>::close(a);
            mine[u] = red;
#pragma unroll
            for (uint32_t j = 1; j < (uint32_t)N_; ++j)
                st_async_v4((c.rank + j) % N_, c.sa + own + u * 16u, red, c.bar(1));   // shared::cta addresses
        }
        c.st.round(0);
        wait(c, 1);
        c.st.round(1);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// B200 extension, not one of the reference files: the reduce-scatter shot of the two-shot AllReduce
// (allreduce__two_shot_push__trtllm.cu:31-45) over the SM-to-SM network, then the all-gather through the
// outputs: every rank's output row of a problem is the same vector, so CTA b writes its reduced chunk
// straight into position b of all N output rows instead of first pushing it into the peers' shared
// memory. Same result, half the SM-to-SM bytes ((N-1)/N * P per CTA), the same HBM bytes.
template <int N_, typename T_, class Op_>
struct AR_RsPushGlobalAg {
    DSB_TRAITS(AllReduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return AR_TwoShotPush<N_, T_, Op_>::legal(M); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t CB = (M / N_) * B, slots = kD0 + M * B, n = CB >> 4;
        if (threadIdx.x == 0) {
            arm(c, 0, (N_ - 1) * CB);
            for (uint32_t j = 1; j < (uint32_t)N_; ++j) {
                const uint32_t dst = (c.rank + j) % N_;
                push<N_>(c, dst, slots + c.rank * CB, kD0 + dst * CB, CB, 0);
            }
        }
        wait(c, 0);
        uint4* mine = c.ptr<uint4>(kD0 + c.rank * CB);
        const uint4* ps = c.ptr<const uint4>(slots);
        for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
            uint4 v[N_];
#pragma unroll
            for (int r = 0; r < N_; ++r) v[r] = (r == (int)c.rank) ? mine[u] : ps[r * n + u];
            auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
            for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
            mine[u] = Pk<T, Op>::close(a);
        }
        c.st.round(0);
    }
    // g is this rank's output row; the problem's rows are contiguous, row r at g + (r - b) * M.
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        const uint32_t C = M / N_, CB = C * B;
        for (int r = 0; r < N_; ++r) s2g(c, g + ((long long)r - (long long)c.rank) * M + c.rank * C, kD0 + c.rank * CB, CB);
    }
};

// allreduce__reduce_bcast_binomial__mpich.cu:23-61. Binomial reduce to rank 0 (d = 1,2,..: a rank with
// bit d set pushes its partial to b-d and drops out), then binomial broadcast (d = N/2 .. 1).
template <int N_, typename T_, class Op_>
struct AR_ReduceBcastBinomial {
    DSB_TRAITS(AllReduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, scr = kD0 + MB;
        int round = 0;
        bool active = true;
        for (int d = 1; d < N_; d <<= 1, ++round) {
            if (active) {
                if (c.rank & (uint32_t)d) {
                    if (threadIdx.x == 0) push<N_>(c, c.rank - d, scr, kD0, MB, 0);
                    active = false;
                } else {
                    if (threadIdx.x == 0) arm(c, 0, MB);
                    wait(c, 0);
                    reduce2<T, Op>(c, kD0, kD0, scr, MB);
                    fence_proxy_async_smem();
                }
            }
            cluster_sync();
            c.st.round(round);
        }
        for (int d = N_ / 2; d >= 1; d >>= 1, ++round) {
            const uint32_t m = c.rank % (2u * d);
            if (m == 0u) {
                if (threadIdx.x == 0) push<N_>(c, c.rank + d, kD0, kD0, MB, 0);
            } else if (m == (uint32_t)d) {
                if (threadIdx.x == 0) arm(c, 0, MB);
                wait(c, 0);
            }
            cluster_sync();
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Binomial reduce + broadcast (allreduce__reduce_bcast_binomial__mpich.cu:23-61 schedule) with a buffer and an
// mbarrier per round: in reduce round k (d = 2^k) a rank with b mod 2d == d pushes its partial into scratch k of
// b - d (barrier k), which adds it; broadcast round d (d = N/2 .. 1) pushes the result from b (b mod 2d == 0)
// into b + d's vector (barrier log2 N + log2 d). A rank waits only for the copies it receives. The broadcast
// overwrites a vector that its owner pushed during the reduction only after the root has received everything,
// so that push had completed. Same pairs and operand order as the original.
template <int N_, typename T_, class Op_>
struct AR_ReduceBcastBinomialCredit {
    DSB_TRAITS(AllReduce, 2 * ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + (1ull + ilog2(N_)) * M * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k) {
                const uint32_t d = 1u << k;
                if (c.rank % (2u * d) == 0u) arm(c, k, MB);       // receives a partial in reduce round k
                if (c.rank % (2u * d) == d) arm(c, L + k, MB);    // receives the result at broadcast distance d
            }
        for (int k = 0; k < L; ++k) {
            const uint32_t d = 1u << k, m = c.rank % (2u * d), scr = kD0 + (uint32_t)(k + 1) * MB;
            if (m == d) {
                if (threadIdx.x == 0) push<N_>(c, c.rank - d, scr, kD0, MB, k);
                c.st.round(k);
                break;   // this rank's partial is handed on: it drops out of the reduction
            }
            wait(c, k);
            reduce2<T, Op>(c, kD0, kD0, scr, MB);
            fence_proxy_async_smem();
            __syncthreads();   // the partial is whole before thread 0 pushes it on
            c.st.round(k);
        }
        for (int k = L - 1; k >= 0; --k) {
            const uint32_t d = 1u << k, m = c.rank % (2u * d);
            if (m == 0u) {
                if (threadIdx.x == 0) push<N_>(c, c.rank + d, kD0, kD0, MB, L + k);
            } else if (m == d) {
                wait(c, L + k);
            }
            c.st.round(2 * L - 1 - k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// allreduce__atomic_all_push__generic.cu:25-41 (sum only). Accumulator = own input; every element is
// added into every peer's accumulator with red.shared::cluster.add; one cluster barrier.
template <int N_, typename T_, class Op_>
struct AR_AtomicAllPush {
    DSB_TRAITS(AllReduce, 0)
    using AccT = typename AccOf<T_>::type;
    static constexpr uint32_t AB = sizeof(AccT);
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B) && IsSum<Op_>::value; }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * M * AB; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s_acc<T>(c, kD0, g, M);
        __syncthreads();
        s2s(c, kD0 + M * AB, kD0, M * AB);   // accumulator starts as my own vector
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MA = M * AB, n = MA >> 4;
        const uint4* pm = c.ptr<const uint4>(kD0);
        for (uint32_t idx = threadIdx.x; idx < (N_ - 1) * n; idx += blockDim.x) {
            const uint32_t k = idx / n, u = idx - k * n;
            const uint32_t peer = (c.rank + 1 + k) % N_;
            red_add_packet(AccT{}, mapa(c.sa + kD0 + MA + 16u * u, peer), pm[u]);
        }
        c.st.round(0);
        cluster_sync();   // all remote adds performed and visible
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g_acc<T>(c, g, kD0 + M * AB, M);
    }
};

template <int N>
struct Grid2D {
    static constexpr int R = (N >= 16) ? 4 : (N >= 4 ? 2 : 1);
    static constexpr int C = N / R;
};

// allreduce__2d_mesh__generic.cu:27-96. R x C grid (16 = 4x4, 8 = 2x4, 4 = 2x2, 2 = 1x2): row
// reduce-scatter push, column all-reduce push of the row partial, row all-gather push. No cluster
// barrier inside; one aggregate mbarrier per phase.
template <int N_, typename T_, class Op_>
struct AR_Mesh2D {
    DSB_TRAITS(AllReduce, 3)
    static constexpr int R = Grid2D<N_>::R, C = Grid2D<N_>::C;
    __host__ __device__ static constexpr bool legal(uint32_t M) {
        return R * C == N_ && M % C == 0 && mult16((M / C) * B);
    }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + 1ull * M * B + (C + R + 1ull) * (M / C) * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t KB = (M / C) * B, n = KB >> 4;
        const uint32_t buf = kD0, rs = kD0 + M * B, cs = rs + C * KB, chunk = cs + R * KB;
        const uint32_t row = c.rank / C, col = c.rank % C;
        // phase 1: row reduce-scatter
        if (threadIdx.x == 0) {
            arm(c, 0, (C - 1) * KB);
            for (uint32_t j = 1; j < (uint32_t)C; ++j) {
                const uint32_t dc = (col + j) % C;
                push<N_>(c, row * C + dc, rs + col * KB, buf + dc * KB, KB, 0);
            }
        }
        wait(c, 0);
        {
            uint4* pb = c.ptr<uint4>(buf + col * KB);
            const uint4* pr = c.ptr<const uint4>(rs);
            for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
                auto a = Pk<T, Op>::open(pb[u]);
#pragma unroll
                for (int k = 0; k < C; ++k)
                    if (k != (int)col) Pk<T, Op>::add(a, pr[k * n + u]);
                pb[u] = Pk<T, Op>::close(a);
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        c.st.round(0);
        // phase 2: column all-reduce of chunk `col`
        if (R > 1) {
            if (threadIdx.x == 0) {
                arm(c, 1, (R - 1) * KB);
                for (uint32_t j = 1; j < (uint32_t)R; ++j) {
                    const uint32_t dr = (row + j) % R;
                    push<N_>(c, dr * C + col, cs + row * KB, buf + col * KB, KB, 1);
                }
            }
            wait(c, 1);
            const uint4* pb = c.ptr<const uint4>(buf + col * KB);
            const uint4* pc = c.ptr<const uint4>(cs);
            uint4* pk = c.ptr<uint4>(chunk);
            for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {   // my column push may still read buf
                auto a = Pk<T, Op>::open(pb[u]);
#pragma unroll
                for (int k = 0; k < R; ++k)
                    if (k != (int)row) Pk<T, Op>::add(a, pc[k * n + u]);
                pk[u] = Pk<T, Op>::close(a);
            }
        } else {
            s2s(c, chunk, buf + col * KB, KB);
        }
        fence_proxy_async_smem();
        __syncthreads();
        c.st.round(1);
        // phase 3: row all-gather
        if (threadIdx.x == 0) {
            arm(c, 2, (C - 1) * KB);
            for (uint32_t j = 1; j < (uint32_t)C; ++j) {
                const uint32_t dst = row * C + (col + j) % C;
                push<N_>(c, dst, buf + col * KB, chunk, KB, 2);
            }
        }
        wait(c, 2);
        c.st.round(2);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        const uint32_t KB = (M / C) * B, nk = KB >> 4, n = (M * B) >> 4, col = c.rank % C;
        const uint4* pb = c.ptr<const uint4>(kD0);
        const uint4* pk = c.ptr<const uint4>(kD0 + M * B + (C + R) * KB);
        uint4* dst = reinterpret_cast<uint4*>(g);
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t k = i / nk;
            __stcs(dst + i, (k == col) ? pk[i - k * nk] : pb[i]);
        }
    }
};

// =====================================================================================================
//                                              ALLGATHER
// Per rank: in[M] -> out[N*M], slot r = rank r's vector.
// =====================================================================================================

// Store a rotated gather buffer: slot k of D holds rank (b + sign*k) mod N.
template <int N, int SIGN>
__device__ __forceinline__ void store_rotated(const Ctx& c, void* g, uint32_t MB) {
    const uint32_t nb = MB >> 4, n = N * nb;
    const uint4* D = c.ptr<const uint4>(kD0);
    uint4* o = static_cast<uint4*>(g);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t k = i / nb, e = i - k * nb;
        const uint32_t r = (SIGN > 0) ? (c.rank + k) % N : (c.rank + N - k) % N;
        __stcs(o + r * nb + e, D[i]);
    }
}

// allgather__recursive_doubling__clusterfusion.cu:22-42 (+ un-rotation :66-72). Own data in slot 0;
// stride s = 1,2,..: push D[0:s) to (b+s) mod N's D[s:2s). Slot k ends holding rank (b-k) mod N.
template <int N_, typename T_, class Op_>
struct AG_RecursiveDoubling {
    DSB_TRAITS(AllGather, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        int round = 0;
        for (int s = 1; s < N_; s <<= 1, ++round) {
            const uint32_t bytes = s * MB;
            if (threadIdx.x == 0) {
                arm(c, 0, bytes);
                push<N_>(c, (c.rank + s) % N_, kD0 + bytes, kD0, bytes, 0);
            }
            wait(c, 0);
            cluster_sync();
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        store_rotated<N_, -1>(c, g, M * B);
    }
};

// allgather__direct_shift__clusterfusion.cu:24-43. Own data in slot b. N-1 rounds; round i arms a fresh
// barrier, cluster barrier, pushes slot b to (b+i) mod N, waits, cluster barrier. The reference re-runs
// mbarrier.init on one barrier every round; re-initialising a barrier that has completed a phase timed
// out on sm_100a, so each round owns its own barrier (initialised once per launch, phase-tracked across
// problems). Rounds, partners, messages and the two cluster barriers per round are unchanged.
template <int N_, typename T_, class Op_>
struct AG_DirectShift {
    DSB_TRAITS(AllGather, N_ - 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0 + c.rank * M * B, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, seg = kD0 + c.rank * MB;
        for (int i = 1; i < N_; ++i) {
            if (threadIdx.x == 0) arm(c, i - 1, MB);
            cluster_sync();   // armed everywhere before anyone pushes
            if (threadIdx.x == 0) push<N_>(c, (c.rank + i) % N_, seg, seg, MB, i - 1);
            wait(c, i - 1);
            cluster_sync();
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// allgather__direct_replicated_push__credit.cu:20-29. Plain remote 16-B stores of my vector into
// slot[b] of every CTA (self included), one cluster barrier.
template <int N_, typename T_, class Op_>
struct AG_DirectReplicatedPush {
    DSB_TRAITS(AllGather, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (N_ + 1ull) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, n = MB >> 4, slots = kD0 + MB;
        const uint4* pm = c.ptr<const uint4>(kD0);
        for (uint32_t idx = threadIdx.x; idx < N_ * n; idx += blockDim.x) {
            const uint32_t p = idx / n, u = idx - p * n;
            st_cluster_v4(mapa(c.sa + slots + c.rank * MB + 16u * u, p), pm[u]);
        }
        cluster_sync();
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + M * B, N_ * M * B);
    }
};

// allgather__ring__nccl.cu:19-36. Own data in slot b; step s forwards slot (b-s) to the successor's
// same slot. N-1 steps.
template <int N_, typename T_, class Op_>
struct AG_Ring {
    DSB_TRAITS(AllGather, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0 + c.rank * M * B, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, next = (c.rank + 1) % N_;
        for (int s = 0; s < N_ - 1; ++s) {
            const uint32_t slot = (c.rank + N_ - s) % N_;
            if (threadIdx.x == 0) {
                arm(c, 0, MB);
                push<N_>(c, next, kD0 + slot * MB, kD0 + slot * MB, MB, 0);
            }
            wait(c, 0);
            cluster_sync();
            c.st.round(s);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// allgather__bruck__mpich.cu:22-41 (+ un-rotation :66-70). Own data in slot 0; d = 1,2,4..: send the
// first min(d, N-d) slots to (b-d) mod N, which stores them at slots [d, d+cnt). Slot k ends holding
// rank (b+k) mod N. Any N.
template <int N_, typename T_, class Op_>
struct AG_Bruck {
    DSB_TRAITS(AllGather, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        int round = 0;
        for (int d = 1; d < N_; d <<= 1, ++round) {
            const uint32_t cnt = (d < N_ - d) ? d : N_ - d, bytes = cnt * MB;
            if (threadIdx.x == 0) {
                arm(c, 0, bytes);
                push<N_>(c, (c.rank + N_ - d) % N_, kD0 + d * MB, kD0, bytes, 0);
            }
            wait(c, 0);
            cluster_sync();
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        store_rotated<N_, +1>(c, g, M * B);
    }
};

// ---- mbarrier-credit AllGather variants (B200 extensions; see the AllReduce credit variants): the same
// rounds, partners and messages as the originals, each round's bytes landing in slots written once per
// problem and on a barrier of their own, so a round waits for its one incoming copy and there is no
// barrier.cluster between rounds.

// Ring (allgather__ring__nccl.cu:19-36 schedule): round s forwards slot (b - s) to the successor's same
// slot, on barrier s. N - 1 barriers.
template <int N_, typename T_, class Op_>
struct AG_RingCredit {
    DSB_TRAITS(AllGather, N_ - 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0 + c.rank * M * B, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, next = (c.rank + 1) % N_;
        if (threadIdx.x == 0)
            for (int s = 0; s < N_ - 1; ++s) arm(c, s, MB);
        for (int s = 0; s < N_ - 1; ++s) {
            const uint32_t slot = (c.rank + N_ - s) % N_;   // own data, then what round s - 1 brought
            if (threadIdx.x == 0) push<N_>(c, next, kD0 + slot * MB, kD0 + slot * MB, MB, s);
            wait(c, s);
            c.st.round(s);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// Recursive doubling (allgather__recursive_doubling__clusterfusion.cu:22-42 schedule): round k pushes
// D[0:2^k) to (b + 2^k)'s D[2^k:2^(k+1)) on barrier k; slot k ends holding rank (b - k) mod N.
template <int N_, typename T_, class Op_>
struct AG_RecursiveDoublingCredit {
    DSB_TRAITS(AllGather, ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; (1 << k) < N_; ++k) arm(c, k, (1u << k) * MB);
        for (int k = 0; (1 << k) < N_; ++k) {
            const uint32_t bytes = (1u << k) * MB;
            if (threadIdx.x == 0) push<N_>(c, (c.rank + (1u << k)) % N_, kD0 + bytes, kD0, bytes, k);
            wait(c, k);
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        store_rotated<N_, -1>(c, g, M * B);
    }
};

// Bruck (allgather__bruck__mpich.cu:22-41 schedule): round k (d = 2^k) sends the first min(d, N - d) slots
// to (b - d) mod N, which stores them at slots [d, d + cnt), on barrier k. Any N.
template <int N_, typename T_, class Op_>
struct AG_BruckCredit {
    DSB_TRAITS(AllGather, ilog2(N_ - 1) + 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; (1 << k) < N_; ++k) {
                const uint32_t d = 1u << k, cnt = (d < N_ - d) ? d : N_ - d;
                arm(c, k, cnt * MB);
            }
        for (int k = 0; (1 << k) < N_; ++k) {
            const uint32_t d = 1u << k, cnt = (d < N_ - d) ? d : N_ - d;
            if (threadIdx.x == 0) push<N_>(c, (c.rank + N_ - d) % N_, kD0 + d * MB, kD0, cnt * MB, k);
            wait(c, k);
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        store_rotated<N_, +1>(c, g, M * B);
    }
};

// allgather__direct_pull__generic.cu:17-33. Every CTA copies slot r straight out of CTA r's input
// with 16-B ld.shared::cluster (own slot copied locally).
template <int N_, typename T_, class Op_>
struct AG_DirectPull {
    DSB_TRAITS(AllGather, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (N_ + 1ull) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, n = MB >> 4;
        const uint4* pm = c.ptr<const uint4>(kD0);
        uint4* D = c.ptr<uint4>(kD0 + MB);
        for (uint32_t idx = threadIdx.x; idx < N_ * n; idx += blockDim.x) {
            const uint32_t r = idx / n, u = idx - r * n;
            D[idx] = (r == c.rank) ? pm[u] : ld_cluster_v4(mapa(c.sa + kD0 + 16u * u, r));
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + M * B, N_ * M * B);
    }
};

// allgather__gather_bcast_binomial__mpich.cu:24-57. Binomial gather to rank 0 (a rank with bit d set
// sends its d accumulated slots to b-d's slots [d, 2d)), then binomial broadcast of all N slots.
template <int N_, typename T_, class Op_>
struct AG_GatherBcastBinomial {
    DSB_TRAITS(AllGather, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        int round = 0;
        bool active = true;
        for (int d = 1; d < N_; d <<= 1, ++round) {
            if (active) {
                if (c.rank & (uint32_t)d) {
                    if (threadIdx.x == 0) push<N_>(c, c.rank - d, kD0 + d * MB, kD0, d * MB, 0);
                    active = false;
                } else {
                    if (threadIdx.x == 0) arm(c, 0, d * MB);
                    wait(c, 0);
                }
            }
            cluster_sync();
            c.st.round(round);
        }
        for (int d = N_ / 2; d >= 1; d >>= 1, ++round) {
            const uint32_t m = c.rank % (2u * d);
            if (m == 0u) {
                if (threadIdx.x == 0) push<N_>(c, c.rank + d, kD0, kD0, N_ * MB, 0);
            } else if (m == (uint32_t)d) {
                if (threadIdx.x == 0) arm(c, 0, N_ * MB);
                wait(c, 0);
            }
            cluster_sync();
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// Binomial gather + broadcast (allgather__gather_bcast_binomial__mpich.cu:24-57 schedule) with an mbarrier per
// round: in gather round k (d = 2^k) a rank with b mod 2d == d pushes its d accumulated slots into slots
// [d, 2d) of b - d (barrier k); broadcast round d pushes all N slots from b (b mod 2d == 0) to b + d (barrier
// log2 N + log2 d). Each slot range is written once per problem before the broadcast, and the broadcast
// overwrites a rank's slots only after the root has gathered everything (so that rank's gather push had
// completed).
template <int N_, typename T_, class Op_>
struct AG_GatherBcastBinomialCredit {
    DSB_TRAITS(AllGather, 2 * ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k) {
                const uint32_t d = 1u << k;
                if (c.rank % (2u * d) == 0u) arm(c, k, d * MB);
                if (c.rank % (2u * d) == d) arm(c, L + k, N_ * MB);
            }
        for (int k = 0; k < L; ++k) {
            const uint32_t d = 1u << k, m = c.rank % (2u * d);
            if (m == d) {
                if (threadIdx.x == 0) push<N_>(c, c.rank - d, kD0 + d * MB, kD0, d * MB, k);
                c.st.round(k);
                break;
            }
            wait(c, k);
            c.st.round(k);
        }
        for (int k = L - 1; k >= 0; --k) {
            const uint32_t d = 1u << k, m = c.rank % (2u * d);
            if (m == 0u) {
                if (threadIdx.x == 0) push<N_>(c, c.rank + d, kD0, kD0, N_ * MB, L + k);
            } else if (m == d) {
                wait(c, L + k);
            }
            c.st.round(2 * L - 1 - k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// =====================================================================================================
//                                            REDUCESCATTER
// Per rank: in[N*M] (chunk j for rank j) -> out[M] = op over ranks of chunk b.
// =====================================================================================================

// reducescatter__ring__nccl.cu:18-37. Step s pushes the partial of chunk (b-s-1) to the successor's
// scratch and adds the received partial into chunk (b-s-2); chunk b completes on b.
template <int N_, typename T_, class Op_>
struct RS_Ring {
    DSB_TRAITS(ReduceScatter, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (N_ + 1ull) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, scr = kD0 + N_ * MB, next = (c.rank + 1) % N_;
        for (int s = 0; s < N_ - 1; ++s) {
            const uint32_t send_c = (c.rank + 2 * N_ - s - 1) % N_, recv_c = (c.rank + 2 * N_ - s - 2) % N_;
            if (threadIdx.x == 0) {
                arm(c, 0, MB);
                push<N_>(c, next, scr, kD0 + send_c * MB, MB, 0);
            }
            wait(c, 0);
            reduce2<T, Op>(c, kD0 + recv_c * MB, kD0 + recv_c * MB, scr, MB);
            fence_proxy_async_smem();
            cluster_sync();
            c.st.round(s);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + c.rank * M * B, M * B);
    }
};

// reducescatter__recursive_halving__mpich.cu:19-44. XOR halving over the N*M buffer; the live range
// ends as chunk b.
template <int N_, typename T_, class Op_>
struct RS_RecursiveHalving {
    DSB_TRAITS(ReduceScatter, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + 1ull * N_ * M * B + (N_ / 2ull) * M * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t scr = kD0 + N_ * M * B;
        uint32_t lo = 0, hi = N_ * M;
        int round = 0;
        for (int d = N_ / 2; d >= 1; d >>= 1, ++round) {
            const uint32_t partner = c.rank ^ (uint32_t)d, mid = (lo + hi) / 2, len = hi - mid;
            const bool upper = (c.rank & (uint32_t)d) != 0u;
            const uint32_t send_lo = upper ? lo : mid, keep_lo = upper ? mid : lo;
            if (threadIdx.x == 0) {
                arm(c, 0, len * B);
                push<N_>(c, partner, scr, kD0 + send_lo * B, len * B, 0);
            }
            wait(c, 0);
            reduce2<T, Op>(c, kD0 + keep_lo * B, kD0 + keep_lo * B, scr, len * B);
            lo = keep_lo;
            hi = keep_lo + len;
            fence_proxy_async_smem();
            cluster_sync();
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + c.rank * M * B, M * B);
    }
};

// ---- mbarrier-credit ReduceScatter variants (B200 extensions; see the AllReduce credit variants).

// Ring (reducescatter__ring__nccl.cu:18-37 schedule): round s pushes the partial of chunk (b - s - 1) into
// receive slot s of the successor, which adds it into its chunk (b - s - 2); chunk b completes on b.
// N - 1 slots and barriers.
template <int N_, typename T_, class Op_>
struct RS_RingCredit {
    DSB_TRAITS(ReduceScatter, N_ - 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (2ull * N_ - 1) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, scr0 = kD0 + N_ * MB, next = (c.rank + 1) % N_;
        if (threadIdx.x == 0)
            for (int s = 0; s < N_ - 1; ++s) arm(c, s, MB);
        for (int s = 0; s < N_ - 1; ++s) {
            const uint32_t send_c = (c.rank + 2 * N_ - s - 1) % N_, recv_c = (c.rank + 2 * N_ - s - 2) % N_;
            if (threadIdx.x == 0) push<N_>(c, next, scr0 + s * MB, kD0 + send_c * MB, MB, s);
            wait(c, s);
            reduce2<T, Op>(c, kD0 + recv_c * MB, kD0 + recv_c * MB, scr0 + s * MB, MB);
            fence_proxy_async_smem();
            __syncthreads();   // the reduced chunk is whole before thread 0 pushes it on
            c.st.round(s);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + c.rank * M * B, M * B);
    }
};

// Recursive halving (reducescatter__recursive_halving__mpich.cu:19-44 schedule): XOR partners d = N/2 .. 1,
// the half sent in round k lands in the partner's scratch range k (N*M/2, N*M/4, .. elements) on barrier k.
template <int N_, typename T_, class Op_>
struct RS_RecursiveHalvingCredit {
    DSB_TRAITS(ReduceScatter, ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (2ull * N_ - 1) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        if (threadIdx.x == 0) {
            uint32_t len = N_ * M / 2;
            for (int k = 0; k < ilog2(N_); ++k, len /= 2) arm(c, k, len * B);
        }
        uint32_t lo = 0, hi = N_ * M, scr = kD0 + N_ * M * B;
        int k = 0;
        for (int d = N_ / 2; d >= 1; d >>= 1, ++k) {
            const uint32_t partner = c.rank ^ (uint32_t)d, mid = (lo + hi) / 2, len = hi - mid;
            const bool upper = (c.rank & (uint32_t)d) != 0u;
            const uint32_t send_lo = upper ? lo : mid, keep_lo = upper ? mid : lo;
            if (threadIdx.x == 0) push<N_>(c, partner, scr, kD0 + send_lo * B, len * B, k);
            wait(c, k);
            reduce2<T, Op>(c, kD0 + keep_lo * B, kD0 + keep_lo * B, scr, len * B);
            fence_proxy_async_smem();
            __syncthreads();   // the kept half is reduced before thread 0 sends part of it on
            lo = keep_lo;
            hi = keep_lo + len;
            scr += len * B;
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + c.rank * M * B, M * B);
    }
};

// reducescatter__direct_push__generic.cu:19-40. N-1 bulk pushes of chunk j into slot[b] of CTA j,
// one aggregate barrier, local reduction.
template <int N_, typename T_, class Op_>
struct RS_DirectPush {
    DSB_TRAITS(ReduceScatter, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (2ull * N_ + 1) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, n = MB >> 4, slots = kD0 + N_ * MB, res = slots + N_ * MB;
        if (threadIdx.x == 0) {
            arm(c, 0, (N_ - 1) * MB);
            for (uint32_t j = 1; j < (uint32_t)N_; ++j) {
                const uint32_t dst = (c.rank + j) % N_;
                push<N_>(c, dst, slots + c.rank * MB, kD0 + dst * MB, MB, 0);
            }
        }
        wait(c, 0);
        const uint4* mine = c.ptr<const uint4>(kD0 + c.rank * MB);
        const uint4* ps = c.ptr<const uint4>(slots);
        uint4* pr = c.ptr<uint4>(res);
        for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
            uint4 v[N_];
#pragma unroll
            for (int r = 0; r < N_; ++r) v[r] = (r == (int)c.rank) ? mine[u] : ps[r * n + u];
            auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
            for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
            pr[u] = Pk<T, Op>::close(a);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + 2 * N_ * M * B, M * B);
    }
};

// reducescatter__direct_pull__generic.cu:16-39. 16-B remote loads of chunk b from all N CTAs.
template <int N_, typename T_, class Op_>
struct RS_DirectPull {
    DSB_TRAITS(ReduceScatter, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + (N_ + 1ull) * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, N_ * M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, n = MB >> 4;
        uint4* pr = c.ptr<uint4>(kD0 + N_ * MB);
        uint32_t base[N_];
#pragma unroll
        for (int r = 0; r < N_; ++r) base[r] = mapa(c.sa + kD0 + c.rank * MB, r);
        for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
            uint4 v[N_];
#pragma unroll
            for (int r = 0; r < N_; ++r) v[r] = ld_cluster_v4(base[r] + 16u * u);
            auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
            for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
            pr[u] = Pk<T, Op>::close(a);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + N_ * M * B, M * B);
    }
};

// =====================================================================================================
//                                              ALLTOALL
// Per rank: in[N*M] (chunk j for rank j) -> out[N*M], slot r = rank r's chunk b.
// =====================================================================================================

// alltoall__pairwise_exchange__fa4.cu:28-44 (N = 2). The sender arms the RECEIVER's mbarrier with a
// remote arrive.expect_tx, then one bulk push of the half the peer owns.
template <int N_, typename T_, class Op_>
struct A2A_PairwiseExchange {
    DSB_TRAITS(AllToAll, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return N_ == 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 3ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, 2 * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, peer = c.rank ^ 1u;
        __syncthreads();
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx_remote(c.bar(0), peer, MB);
            push<N_>(c, peer, kD0 + 2 * MB, kD0 + peer * MB, MB, 0);
        }
        wait(c, 0);
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        const uint32_t MB = M * B;
        s2g(c, g + c.rank * M, kD0 + c.rank * MB, MB);
        s2g(c, g + (c.rank ^ 1u) * M, kD0 + 2 * MB, MB);
    }
};

// alltoall__direct_push__generic.cu:17-33. N-1 bulk pushes (chunk j -> CTA j's recv[b]), one aggregate
// barrier; own chunk copied locally.
template <int N_, typename T_, class Op_>
struct A2A_DirectPush {
    DSB_TRAITS(AllToAll, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, recv = kD0 + N_ * MB;
        if (threadIdx.x == 0) {
            arm(c, 0, (N_ - 1) * MB);
            for (uint32_t j = 1; j < (uint32_t)N_; ++j) {
                const uint32_t dst = (c.rank + j) % N_;
                push<N_>(c, dst, recv + c.rank * MB, kD0 + dst * MB, MB, 0);
            }
        }
        s2s(c, recv + c.rank * MB, kD0 + c.rank * MB, MB);
        wait(c, 0);
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + N_ * M * B, N_ * M * B);
    }
};

// alltoall__pairwise_xor__mpich.cu:19-38. Round i: partner b^i, one push + wait + cluster barrier.
template <int N_, typename T_, class Op_>
struct A2A_PairwiseXor {
    DSB_TRAITS(AllToAll, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, recv = kD0 + N_ * MB;
        s2s(c, recv + c.rank * MB, kD0 + c.rank * MB, MB);
        for (int i = 1; i < N_; ++i) {
            const uint32_t p = c.rank ^ (uint32_t)i;
            if (threadIdx.x == 0) {
                arm(c, 0, MB);
                push<N_>(c, p, recv + c.rank * MB, kD0 + p * MB, MB, 0);
            }
            wait(c, 0);
            cluster_sync();
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + N_ * M * B, N_ * M * B);
    }
};

// Pairwise XOR (alltoall__pairwise_xor__mpich.cu:19-38 schedule) with an mbarrier per round: round i pushes the
// chunk for partner b ^ i into its receive slot [b] on barrier i - 1 and waits for the partner's chunk on its
// own barrier i - 1. Every receive slot is written once per problem, so no cluster barrier is needed between
// rounds (N - 1 barriers: N <= 16).
template <int N_, typename T_, class Op_>
struct A2A_PairwiseXorCredit {
    DSB_TRAITS(AllToAll, N_ - 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, recv = kD0 + N_ * MB;
        if (threadIdx.x == 0)
            for (int i = 1; i < N_; ++i) arm(c, i - 1, MB);
        s2s(c, recv + c.rank * MB, kD0 + c.rank * MB, MB);
        for (int i = 1; i < N_; ++i) {
            const uint32_t p = c.rank ^ (uint32_t)i;
            if (threadIdx.x == 0) push<N_>(c, p, recv + c.rank * MB, kD0 + p * MB, MB, i - 1);
            wait(c, i - 1);
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + N_ * M * B, N_ * M * B);
    }
};

// alltoall__shift__generic.cu:19-37. Round i: push chunk (b+i) to CTA b+i, receive from b-i.
template <int N_, typename T_, class Op_>
struct A2A_Shift {
    DSB_TRAITS(AllToAll, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, N_ * M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, recv = kD0 + N_ * MB;
        s2s(c, recv + c.rank * MB, kD0 + c.rank * MB, MB);
        for (int i = 1; i < N_; ++i) {
            const uint32_t dst = (c.rank + i) % N_;
            if (threadIdx.x == 0) {
                arm(c, 0, MB);
                push<N_>(c, dst, recv + c.rank * MB, kD0 + dst * MB, MB, 0);
            }
            wait(c, 0);
            cluster_sync();
            c.st.round(i - 1);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + N_ * M * B, N_ * M * B);
    }
};

// alltoall__bruck__mpich.cu:24-56 (rotations :75-94). Load rotated (position i holds the chunk for rank
// (b+i) mod N); round d sends the N/2 blocks whose position has bit d set to (b+d) mod N's staging
// area, barrier, copy back, barrier; store with the inverse rotation.
template <int N_, typename T_, class Op_>
struct A2A_Bruck {
    DSB_TRAITS(AllToAll, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + 1ull * N_ * M * B + (N_ / 2ull) * M * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        const uint32_t nb = (M * B) >> 4, n = N_ * nb;
        const uint4* src = reinterpret_cast<const uint4*>(g);
        uint4* D = c.ptr<uint4>(kD0);
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t j = i / nb, e = i - j * nb;
            D[((j + N_ - c.rank) % N_) * nb + e] = __ldcs(src + i);
        }
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, nb = MB >> 4, tmp = kD0 + N_ * MB;
        int round = 0;
        for (int d = 1; d < N_; d <<= 1, ++round) {
            const uint32_t to = (c.rank + d) % N_;
            if (threadIdx.x == 0) {
                arm(c, 0, (N_ / 2) * MB);
                uint32_t s = 0;
                for (uint32_t pos = 0; pos < (uint32_t)N_; ++pos)
                    if (pos & (uint32_t)d) {
                        push<N_>(c, to, tmp + s * MB, kD0 + pos * MB, MB, 0);
                        ++s;
                    }
            }
            wait(c, 0);
            cluster_sync();   // my outgoing blocks were read: they may be overwritten
            const uint4* pt = c.ptr<const uint4>(tmp);
            uint4* D = c.ptr<uint4>(kD0);
            for (uint32_t i = threadIdx.x; i < (N_ / 2) * nb; i += blockDim.x) {
                const uint32_t s = i / nb, e = i - s * nb;
                const uint32_t pos = (s / d) * 2u * d + d + (s % d);   // s-th position with bit d set
                D[pos * nb + e] = pt[i];
            }
            fence_proxy_async_smem();
            cluster_sync();   // staging free and D stable before the next round's pushes
            c.st.round(round);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        const uint32_t nb = (M * B) >> 4, n = N_ * nb;
        const uint4* D = c.ptr<const uint4>(kD0);
        uint4* o = reinterpret_cast<uint4*>(g);
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t pos = i / nb, e = i - pos * nb;
            __stcs(o + ((c.rank + N_ - pos) % N_) * nb + e, D[i]);
        }
    }
};

// Bruck AlltoAll (alltoall__bruck__mpich.cu:24-56 schedule, rotations :75-94) with a staging range and an
// mbarrier per round: round k (d = 2^k) sends the N/2 blocks whose position has bit k set to (b + d) mod N's
// staging range k (barrier k). Instead of copying staging back, a block's current place is tracked: after
// round k a position with bit k set lives in staging range k (at its index among those positions), otherwise
// where it was; so every range is written once per problem and no cluster barrier is needed. Stored with the
// inverse rotation from each position's final place.
template <int N_, typename T_, class Op_>
struct A2A_BruckCredit {
    DSB_TRAITS(AllToAll, ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + 1ull * N_ * M * B + ilog2(N_) * (N_ / 2ull) * M * B;
    }
    // Window offset of the block at position `pos` once rounds 0..k-1 are done: staging range j of the highest
    // round j < k whose bit is set in pos (at pos's index among the positions with bit j set), else D[pos].
    static __device__ __forceinline__ uint32_t place(uint32_t pos, int k, uint32_t MB) {
        const uint32_t low = pos & ((1u << k) - 1u);
        if (low == 0u) return kD0 + pos * MB;
        const uint32_t j = 31u - __clz(low), d = 1u << j;
        const uint32_t idx = (pos / (2u * d)) * d + (pos % d);
        return kD0 + N_ * MB + (j * (N_ / 2u) + idx) * MB;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        const uint32_t nb = (M * B) >> 4, n = N_ * nb;
        const uint4* src = reinterpret_cast<const uint4*>(g);
        uint4* D = c.ptr<uint4>(kD0);
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t j = i / nb, e = i - j * nb;
            D[((j + N_ - c.rank) % N_) * nb + e] = __ldcs(src + i);
        }
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k) arm(c, k, (N_ / 2) * MB);
        for (int k = 0; k < L; ++k) {
            const uint32_t d = 1u << k, to = (c.rank + d) % N_, stage = kD0 + N_ * MB + (uint32_t)k * (N_ / 2) * MB;
            if (threadIdx.x == 0) {
                uint32_t s = 0;
                for (uint32_t pos = 0; pos < (uint32_t)N_; ++pos)
                    if (pos & d) {
                        push<N_>(c, to, stage + s * MB, place(pos, k, MB), MB, k);
                        ++s;
                    }
            }
            wait(c, k);
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        const uint32_t MB = M * B, nb = MB >> 4, n = N_ * nb;
        uint4* o = reinterpret_cast<uint4*>(g);
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t pos = i / nb, e = i - pos * nb;
            const uint4* src = c.ptr<const uint4>(place(pos, ilog2(N_), MB));
            __stcs(o + ((c.rank + N_ - pos) % N_) * nb + e, src[e]);
        }
    }
};

// alltoall__direct_pull__generic.cu:16-31. 16-B remote loads of chunk b from every peer's send buffer.
template <int N_, typename T_, class Op_>
struct A2A_DirectPull {
    DSB_TRAITS(AllToAll, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 2ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, N_ * M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, nb = MB >> 4;
        const uint4* mine = c.ptr<const uint4>(kD0 + c.rank * MB);
        uint4* recv = c.ptr<uint4>(kD0 + N_ * MB);
        const uint32_t my_chunk = c.sa + kD0 + c.rank * MB;
        for (uint32_t idx = threadIdx.x; idx < N_ * nb; idx += blockDim.x) {
            const uint32_t r = idx / nb, u = idx - r * nb;
            recv[idx] = (r == c.rank) ? mine[u] : ld_cluster_v4(mapa(my_chunk + 16u * u, r));
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0 + N_ * M * B, N_ * M * B);
    }
};

// --------------------------------------------------------------------------- element counts per rank
// One rank block of M elements in: AllReduce, AllGather, Broadcast, Reduce, Gather; N blocks (one per peer):
// ReduceScatter, AlltoAll, Scatter. Out: one block for AllReduce, ReduceScatter, Broadcast, Reduce, Scatter;
// N blocks for AllGather, AlltoAll, Gather.
__host__ __device__ constexpr bool one_block_in(OpKind k) {
    return k == OpKind::AllReduce || k == OpKind::AllGather || k == OpKind::Broadcast || k == OpKind::Reduce ||
           k == OpKind::Gather;
}
__host__ __device__ constexpr bool one_block_out(OpKind k) {
    return k == OpKind::AllReduce || k == OpKind::ReduceScatter || k == OpKind::Broadcast || k == OpKind::Reduce ||
           k == OpKind::Scatter;
}
template <class A>
__host__ __device__ constexpr uint64_t in_elems_per_rank(uint32_t M) {
    return one_block_in(A::kOp) ? (uint64_t)M : (uint64_t)A::kN * M;
}
template <class A>
__host__ __device__ constexpr uint64_t out_elems_per_rank(uint32_t M) {
    return one_block_out(A::kOp) ? (uint64_t)M : (uint64_t)A::kN * M;
}

// --------------------------------------------------------------------------- drivers
struct BatchArgs {
    const void* in;
    void* out;
    long long num_problems;           // independent cluster problems in the batch
    unsigned long long* stamps;       // nullable: [num_problems][N][kStamps]
    unsigned* smid;                   // nullable: [num_problems][N]
    unsigned* err;                    // error word (device memory)
    unsigned long long wait_limit_ns; // per problem
    uint32_t M;                       // elements per rank block
    uint32_t smem_bytes;              // dynamic shared memory of the launch
    uint32_t sub;                     // pipelined drivers: units per problem (M / sub elements each)
    uint32_t depth;                   // streamed drivers: stages of the ring (bounded by the window)
    uint32_t lag;                     // streamed drivers: units of reduce-scatter in flight
};

__device__ __forceinline__ void ctx_init(Ctx& c, uint32_t smem_bytes, unsigned* err, unsigned long long limit) {
    c.sm = dyn_smem_raw;
    c.sa = smem_u32(dyn_smem_raw);
    c.smem_bytes = smem_bytes;
    c.rank = cluster_rank();
    c.phase = 0u;
    c.dead = false;
    c.wait_limit = limit;
    c.deadline = 0ull;
    c.err = err;
    c.unit = 0u;
    c.st.base = nullptr;
}

template <class A>
__device__ __forceinline__ void init_bars(Ctx& c) {
    static_assert(A::kBars >= 0 && 8 * A::kBars <= (int)kFlagOff, "mbarriers overlap the finish flag");
    if (A::kBars > 0 && threadIdx.x == 0) {
        for (int i = 0; i < A::kBars; ++i) mbar_init(c.bar(i), 1);
        fence_mbar_init();
    }
}

// Persistent batch driver: grid = (#resident clusters) x N CTAs, cluster dims (N,1,1).
template <class A>
__global__ void __launch_bounds__(256) batch_kernel(const BatchArgs a) {
    using T = typename A::T;
    constexpr int N = A::kN;
    Ctx c;
    ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    flag_init(c);
    init_bars<A>(c);
    const uint64_t in_r = in_elems_per_rank<A>(a.M), out_r = out_elems_per_rank<A>(a.M);
    const long long step = (long long)num_clusters();
    for (long long p = (long long)cluster_id(); p < a.num_problems; p += step, ++c.unit) {
        const uint64_t slot = (uint64_t)p * N + c.rank;
        c.deadline = globaltimer() + c.wait_limit;
        c.st.base = a.stamps != nullptr ? a.stamps + slot * kStamps : nullptr;
        A::load(c, static_cast<const T*>(a.in) + slot * in_r, a.M);
        if (a.smid != nullptr && threadIdx.x == 0) a.smid[slot] = smid();
        cluster_sync();   // entry: inputs loaded, barriers initialised, previous problem fully retired
        c.st.mark(0);
        A::exec(c, a.M);
        c.st.mark(1);
        A::store(c, static_cast<T*>(a.out) + slot * out_r, a.M);
        cluster_sync();   // exit: no peer still reads or writes my window for this problem
    }
    finish(c);
}

// ---- Broadcast from rank 0 (B200 extension: the rooted collectives the reference's roadmap lists as
// candidates, collectives/ROADMAP.md:268-270; binomial, direct push and direct pull, no TMA multicast).
// Per rank M elements in and out: out of every rank = in of rank 0 (the other ranks' inputs are unused).

// Rank 0 pushes its vector into every peer (N-1 bulk copies, one round).
template <int N_, typename T_, class Op_>
struct BC_DirectPush {
    DSB_TRAITS(Broadcast, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        if (c.rank == 0) {
            g2s(c, kD0, g, M * B);
            fence_proxy_async_smem();
        }
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        if (c.rank == 0) {
            if (threadIdx.x == 0)
                for (uint32_t p = 1; p < (uint32_t)N_; ++p) push<N_>(c, p, kD0, kD0, MB, 0);
        } else {
            if (threadIdx.x == 0) arm(c, 0, MB);
            wait(c, 0);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Every rank but 0 copies rank 0's vector into its own buffer with 16-byte remote loads (one round).
template <int N_, typename T_, class Op_>
struct BC_DirectPull {
    DSB_TRAITS(Broadcast, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        if (c.rank == 0) g2s(c, kD0, g, M * B);
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        if (c.rank != 0) {
            const uint32_t n = (M * B) >> 4, src = mapa(c.sa + kD0, 0u);
            uint4* dst = c.ptr<uint4>(kD0);
#pragma unroll 4
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = ld_cluster_v4(src + 16u * i);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Binomial tree: in round k the ranks below 2^k (which hold the vector) push it to rank + 2^k. Rank r > 0
// receives once, in round floor(log2 r), on its one barrier, then forwards it in the later rounds; no
// cluster barrier between rounds. Any N.
template <int N_, typename T_, class Op_>
struct BC_Binomial {
    DSB_TRAITS(Broadcast, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        if (c.rank == 0) {
            g2s(c, kD0, g, M * B);
            fence_proxy_async_smem();
        }
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        int k0 = 0;   // first round in which this rank sends
        if (c.rank != 0) {
            if (threadIdx.x == 0) arm(c, 0, MB);
            wait(c, 0);
            k0 = ilog2((int)c.rank) + 1;
        }
        if (threadIdx.x == 0)
            for (int k = k0; (1 << k) < N_; ++k) {
                const uint32_t dst = c.rank + (1u << k);
                if (dst < (uint32_t)N_) push<N_>(c, dst, kD0, kD0, MB, 0);
            }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// ---- Reduce, Gather and Scatter rooted at rank 0 (B200 extensions, no reference file: the other rooted
// collectives beside the Broadcast; direct push, direct pull and binomial, no TMA multicast). Per rank:
//   Reduce   in[M] -> out[M] of rank 0 = op over the ranks' vectors; the other ranks' out blocks are not written;
//   Gather   in[M] -> out[N*M] of rank 0 = the ranks' vectors in rank order; the other ranks' out blocks are not
//            written;
//   Scatter  in[N*M] of rank 0 (the other ranks' in blocks are not read) -> out[M] of rank r = block r of it.
// Payload convention: P = M * sizeof(T) for the Reduce (as the AllReduce), P = N * M * sizeof(T) for the Gather
// and the Scatter (as the AllGather and the ReduceScatter). Every CTA of a launch has the same window, sized for
// the root's buffers.

// Every rank but 0 pushes its vector into slot b of rank 0 (one bulk copy, one aggregate barrier); rank 0 sums
// the N slots in rank order, accumulating in fp32 for bf16 (one rounding).
template <int N_, typename T_, class Op_>
struct RD_DirectPush {
    DSB_TRAITS(Reduce, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();   // the bulk push reads it through the async proxy
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B, n = MB >> 4;
        if (c.rank == 0) {
            if (threadIdx.x == 0) arm(c, 0, (N_ - 1) * MB);
            wait(c, 0);
            uint4* p = c.ptr<uint4>(kD0);
            for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
                uint4 v[N_];
#pragma unroll
                for (int r = 0; r < N_; ++r) v[r] = p[r * n + u];
                auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
                for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
                p[u] = Pk<T, Op>::close(a);
            }
        } else if (threadIdx.x == 0) {
            push<N_>(c, 0, kD0 + c.rank * MB, kD0, MB, 0);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        if (c.rank != 0) return;
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Rank 0 reads every peer's vector with 16-byte remote loads and sums them in rank order into its own buffer
// (fp32 accumulation for bf16); the driver's exit cluster barrier keeps the peers' buffers until it is done.
template <int N_, typename T_, class Op_>
struct RD_DirectPull {
    DSB_TRAITS(Reduce, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        if (c.rank == 0) {
            const uint32_t n = (M * B) >> 4;
            uint4* p = c.ptr<uint4>(kD0);
            uint32_t base[N_];
#pragma unroll
            for (int r = 1; r < N_; ++r) base[r] = mapa(c.sa + kD0, r);
            for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
                uint4 v[N_];
                v[0] = p[u];
#pragma unroll
                for (int r = 1; r < N_; ++r) v[r] = ld_cluster_v4(base[r] + 16u * u);
                auto a = Pk<T, Op>::open(v[0]);
#pragma unroll
                for (int r = 1; r < N_; ++r) Pk<T, Op>::add(a, v[r]);
                p[u] = Pk<T, Op>::close(a);
            }
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        if (c.rank != 0) return;
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Binomial tree to rank 0, the reduce half of the binomial AllReduce with a buffer and an mbarrier per round:
// in round k (d = 2^k) a rank with b mod 2d == d pushes its partial into scratch k of b - d and drops out; b - d
// adds it into its own partial. A rank waits only for the copies it receives; no cluster barrier between
// rounds. The element type rounds once per round (as the AllReduce's binomial).
template <int N_, typename T_, class Op_>
struct RD_Binomial {
    DSB_TRAITS(Reduce, ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) {
        return kD0 + (1ull + ilog2(N_)) * M * B;
    }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k)
                if (c.rank % (2u << k) == 0u) arm(c, k, MB);   // receives a partial in round k
        for (int k = 0; k < L; ++k) {
            const uint32_t d = 1u << k, m = c.rank % (2u * d), scr = kD0 + (uint32_t)(k + 1) * MB;
            if (m == d) {
                if (threadIdx.x == 0) push<N_>(c, c.rank - d, scr, kD0, MB, k);
                c.st.round(k);
                break;
            }
            wait(c, k);
            reduce2<T, Op>(c, kD0, kD0, scr, MB);
            fence_proxy_async_smem();
            __syncthreads();   // the partial is whole before thread 0 pushes it on
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        if (c.rank != 0) return;
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Every rank but 0 pushes its vector into slot b of rank 0 (one bulk copy, one aggregate barrier).
template <int N_, typename T_, class Op_>
struct GA_DirectPush {
    DSB_TRAITS(Gather, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        if (c.rank == 0) {
            if (threadIdx.x == 0) arm(c, 0, (N_ - 1) * MB);
            wait(c, 0);
        } else if (threadIdx.x == 0) {
            push<N_>(c, 0, kD0 + c.rank * MB, kD0, MB, 0);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        if (c.rank != 0) return;
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// Rank 0 reads every peer's vector into slot b with 16-byte remote loads.
template <int N_, typename T_, class Op_>
struct GA_DirectPull {
    DSB_TRAITS(Gather, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) { g2s(c, kD0, g, M * B); }
    static __device__ void exec(Ctx& c, uint32_t M) {
        if (c.rank == 0) {
            const uint32_t n = (M * B) >> 4;
            uint4* D = c.ptr<uint4>(kD0);
            for (uint32_t idx = n + threadIdx.x; idx < N_ * n; idx += blockDim.x) {
                const uint32_t r = idx / n, u = idx - r * n;
                D[idx] = ld_cluster_v4(mapa(c.sa + kD0 + 16u * u, r));
            }
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        if (c.rank != 0) return;
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// Binomial tree to rank 0, the gather half of the binomial AllGather with an mbarrier per round: in round k
// (d = 2^k) a rank with b mod 2d == d sends the d blocks it holds (its own and those gathered so far, ranks
// b .. b + d - 1) into blocks [d, 2d) of b - d, and drops out. No cluster barrier between rounds.
template <int N_, typename T_, class Op_>
struct GA_Binomial {
    DSB_TRAITS(Gather, ilog2(N_))
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        g2s(c, kD0, g, M * B);
        fence_proxy_async_smem();
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        constexpr int L = ilog2(N_);
        const uint32_t MB = M * B;
        if (threadIdx.x == 0)
            for (int k = 0; k < L; ++k)
                if (c.rank % (2u << k) == 0u) arm(c, k, (1u << k) * MB);
        for (int k = 0; k < L; ++k) {
            const uint32_t d = 1u << k, m = c.rank % (2u * d);
            if (m == d) {
                if (threadIdx.x == 0) push<N_>(c, c.rank - d, kD0 + d * MB, kD0, d * MB, k);
                c.st.round(k);
                break;
            }
            wait(c, k);
            c.st.round(k);
        }
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        if (c.rank != 0) return;
        __syncthreads();
        s2g(c, g, kD0, N_ * M * B);
    }
};

// Rank 0 pushes block r of its input into rank r (N - 1 bulk copies, one round).
template <int N_, typename T_, class Op_>
struct SC_DirectPush {
    DSB_TRAITS(Scatter, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        if (c.rank == 0) {
            g2s(c, kD0, g, N_ * M * B);
            fence_proxy_async_smem();
        }
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        if (c.rank == 0) {
            if (threadIdx.x == 0)
                for (uint32_t r = 1; r < (uint32_t)N_; ++r) push<N_>(c, r, kD0, kD0 + r * MB, MB, 0);
        } else {
            if (threadIdx.x == 0) arm(c, 0, MB);
            wait(c, 0);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Every rank but 0 reads block b of rank 0's input with 16-byte remote loads.
template <int N_, typename T_, class Op_>
struct SC_DirectPull {
    DSB_TRAITS(Scatter, 0)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        if (c.rank == 0) g2s(c, kD0, g, N_ * M * B);
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        if (c.rank != 0) {
            const uint32_t n = (M * B) >> 4, src = mapa(c.sa + kD0 + c.rank * M * B, 0u);
            uint4* dst = c.ptr<uint4>(kD0);
#pragma unroll 4
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = ld_cluster_v4(src + 16u * i);
        }
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// Binomial tree from rank 0: rounds d = N/2 .. 1; a rank holding blocks of ranks b .. b + 2d - 1 (blocks
// [0, 2d) of its buffer) sends the upper half, blocks [d, 2d), into blocks [0, d) of b + d. Rank r > 0 receives
// once, from r - lowbit(r), on its one barrier, and forwards in the later (smaller) rounds; no cluster barrier
// between rounds.
template <int N_, typename T_, class Op_>
struct SC_Binomial {
    DSB_TRAITS(Scatter, 1)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return is_pow2(N_) && N_ >= 2 && mult16(M * B); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 1ull * N_ * M * B; }
    static __device__ void load(Ctx& c, const T* g, uint32_t M) {
        if (c.rank == 0) {
            g2s(c, kD0, g, N_ * M * B);
            fence_proxy_async_smem();
        }
    }
    static __device__ void exec(Ctx& c, uint32_t M) {
        const uint32_t MB = M * B;
        uint32_t span = (uint32_t)N_;   // blocks this rank holds once its copy has landed
        if (c.rank != 0) {
            span = c.rank & (0u - c.rank);   // lowest set bit: blocks of ranks rank .. rank + span - 1
            if (threadIdx.x == 0) arm(c, 0, span * MB);
            wait(c, 0);
        }
        if (threadIdx.x == 0)
            for (uint32_t d = span / 2u; d >= 1u; d /= 2u) push<N_>(c, c.rank + d, kD0, kD0 + d * MB, d * MB, 0);
        c.st.round(0);
    }
    static __device__ void store(Ctx& c, T* g, uint32_t M) {
        __syncthreads();
        s2g(c, g, kD0, M * B);
    }
};

// -----------------------------------------------------------------------------------------------------
// Pipelined persistent driver of the two-shot AllReduce (allreduce__two_shot_push__trtllm.cu:23-59) for
// batches. Per problem the shots are exactly AR_TwoShotPush's (N-1 bulk pushes of chunk j into slot[b] of
// CTA j, reduce, N-1 bulk pushes of the reduced chunk into position b of every peer), but:
//   * the input arrives by a bulk global->shared copy into one of two X buffers, issued one problem ahead
//     (right after this problem's first shot), and the output leaves by a bulk shared->global copy, so
//     HBM traffic of neighbouring problems overlaps the SM-to-SM shots of the current one;
//   * there is no per-problem cluster barrier. The shot barriers already order everything:
//     my reduce(p) -> my shot 2(p) -> peer's shot-2 wait(p) -> peer's shot 1(p+1), so a peer writes my
//     slots for p+1 only after I have consumed them for p; and a peer's shot 2(p+1) into my X buffer needs
//     my shot 1(p+1), which I issue only after my load(p+1) has landed.
//   * a problem may be split into `sub` sub-vector units that each run the two shots (the element-wise sum
//     is separable), so large payloads keep a small shared-memory footprint and several CTAs per SM.
// Layout per unit of U elements: barriers 0/1 = input landed in X0/X1, 2 = shot 1 (reduce-scatter),
// 3 = shot 2 (all-gather); X0 = [kD0, +UB), X1 = [kD0+UB, +UB), slots = [kD0+2UB, +UB) (slot r at r*CB).
template <int N_, typename T_, class Op_>
struct AR_TwoShotPipelined {
    DSB_TRAITS(AllReduce, 4)
    __host__ __device__ static constexpr bool legal(uint32_t M) { return AR_TwoShotPush<N_, T_, Op_>::legal(M); }
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t M) { return kD0 + 3ull * M * B; }
};

template <class A>
__global__ void __launch_bounds__(256) two_shot_pipelined_kernel(const BatchArgs a) {
    using T = typename A::T;
    using Op = typename A::Op;
    constexpr int N = A::kN;
    constexpr int kLoad0 = 0, kRS = 2, kAG = 3;
    Ctx c;
    ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    flag_init(c);
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(c.bar(i), 1);
        fence_mbar_init();
    }
    cluster_sync();   // every barrier of the cluster initialised before any remote push
    const uint64_t total = (uint64_t)a.num_problems * N * a.M;   // elements of `in` and of `out`
    // A problem of M elements per rank flows through the pipeline as `sub` units of U = M / sub elements,
    // each a complete two-shot AllReduce of its sub-vector (the element-wise sum is separable).
    const uint32_t S = a.sub, U = a.M / S, UB = U * A::B, CB = UB / N, n = CB >> 4;
    const uint32_t slots = kD0 + 2u * UB;
    const T* in = static_cast<const T*>(a.in);
    T* out = static_cast<T*>(a.out);
    const long long step = (long long)num_clusters();
    const long long first = (long long)cluster_id();
    const long long mine = first < a.num_problems ? (a.num_problems - 1 - first) / step + 1 : 0;
    const long long units = mine * S;
    // element offset of unit k of this cluster (this rank's part)
    auto unit_off = [&](long long k) -> uint64_t {
        const long long p = first + (k / S) * step;
        return ((uint64_t)p * N + c.rank) * a.M + (uint64_t)(k % S) * U;
    };
    // checked one-CTA bulk load of unit k into X buffer xb (thread 0)
    auto load_unit = [&](long long k, uint32_t xb) {
        const uint64_t off = unit_off(k);
        if (off + U > total) {
            report(c, DSMEM_ERR_BIT_BOUNDS);
            return;
        }
        arm(c, kLoad0 + (int)xb, UB);
        bulk_load_g2s(c.sa + kD0 + xb * UB, in + off, UB, c.bar(kLoad0 + (int)xb));
    };
    if (threadIdx.x == 0 && units > 0) load_unit(0, 0);
    for (long long k = 0; k < units; ++k) {
        const uint32_t x = (uint32_t)(k & 1), X = kD0 + x * UB, s = (uint32_t)(k % S);
        const uint64_t slot = (uint64_t)(first + (k / S) * step) * N + c.rank;
        c.unit = (uint32_t)k;
        c.deadline = globaltimer() + c.wait_limit;
        c.st.base = a.stamps != nullptr ? a.stamps + slot * kStamps : nullptr;
        if (s == 0 && a.smid != nullptr && threadIdx.x == 0) a.smid[slot] = smid();
        wait(c, kLoad0 + (int)x);   // my input for unit k is in X
        if (s == 0) c.st.mark(0);
        if (threadIdx.x == 0) {
            // shot 1: chunk j of my input -> slot[b] of CTA j
            arm(c, kRS, (N - 1) * CB);
            for (uint32_t j = 1; j < (uint32_t)N; ++j) {
                const uint32_t dst = (c.rank + j) % N;
                push<N>(c, dst, slots + c.rank * CB, X + dst * CB, CB, kRS);
            }
            // prefetch the next unit into the other buffer once the store of the previous one read it
            if (k + 1 < units) {
                bulk_wait_read0();
                load_unit(k + 1, x ^ 1u);
            }
        }
        wait(c, kRS);   // all N-1 partials of my chunk landed (and the peers' reads of their chunk b are done)
        {
            uint4* my = c.ptr<uint4>(X + c.rank * CB);
            const uint4* ps = c.ptr<const uint4>(slots);
            for (uint32_t u = threadIdx.x; u < n; u += blockDim.x) {
                uint4 v[N];
#pragma unroll
                for (int r = 0; r < N; ++r) v[r] = (r == (int)c.rank) ? my[u] : ps[r * n + u];
                auto acc = Pk<T, Op>::open(v[0]);
#pragma unroll
                for (int r = 1; r < N; ++r) Pk<T, Op>::add(acc, v[r]);
                my[u] = Pk<T, Op>::close(acc);
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (s + 1 == S) c.st.round(0);
        if (threadIdx.x == 0) {
            // shot 2: my reduced chunk -> position b of every peer
            arm(c, kAG, (N - 1) * CB);
            for (uint32_t j = 1; j < (uint32_t)N; ++j) {
                const uint32_t dst = (c.rank + j) % N;
                push<N>(c, dst, X + c.rank * CB, X + c.rank * CB, CB, kAG);
            }
        }
        wait(c, kAG);   // every reduced chunk is in X
        if (s + 1 == S) {
            c.st.round(1);
            c.st.mark(1);
        }
        if (threadIdx.x == 0) {
            bulk_store_s2g(out + unit_off(k), c.sa + X, UB);
            bulk_commit();
        }
    }
    if (threadIdx.x == 0) bulk_wait_all0();
    finish(c);   // no CTA leaves while a peer may still push into it
}

// -----------------------------------------------------------------------------------------------------
// Streamed batch drivers (B200 extensions of the batch regime): warp-specialised, two rings, no cluster barrier
// per unit. A problem's per-rank data is cut into units (sub-ranges of U elements of every rank block) that flow
// through:
//   * an input ring of DX stages (the unit's input: one piece for AllReduce / AllGather, the N pieces for
//     ReduceScatter / AlltoAll) and a slot ring of DR stages (what the N - 1 peers push for the unit). A unit in
//     the exchange holds one of each; a unit being loaded holds only an input stage, so DX - DR loads stream in
//     while DR units are exchanged, and no slot buffer sits idle under a load;
//   * warp 0, one thread (producer): for unit k, waits until its input has landed, waits for the release of unit
//     k - DR (local consumers done with it, and the credits of all N - 1 peers: they consumed what this CTA
//     pushed for k - DR, so those bulk copies finished reading their input stage, and freed the slot stage unit k
//     is pushed into), arms its slot barrier, pushes to every peer j (slot (b - j - 1) mod N of CTA j, completing
//     on CTA j's slot barrier), then loads unit k + DX - DR into the input stage unit k - DR released;
//   * warps 1..W (consumers): wait for the unit's input and slots, combine, store from registers with 16-byte
//     streaming stores; after a named barrier one consumer thread arrives (relaxed) on the unit's credit barrier
//     of every peer and on the local `done` barrier of its input stage;
//   * barrier phases follow from the unit index (stage use (k / stages) & 1); before leaving, the producer drains
//     the credits of the last DR units, so no remote arrive or copy aimed at this CTA is in flight at exit.
// Per op (b = this rank, U elements per piece):
//   AllReduce (alg rs_push_global_ag): the reduce-scatter shot of the two-shot AllReduce
//     (allreduce__two_shot_push__trtllm.cu:31-45): chunk j (U / N elements) of the unit to CTA j; the consumers
//     sum the N partials of chunk b in rank order and store the sum into position b of all N output rows (the
//     all-gather through the outputs): (N-1)/N * P per CTA over DSMEM, half the two-shot's;
//   ReduceScatter (alg direct_push, reducescatter__direct_push__generic.cu:19-40): piece j to CTA j; the
//     consumers sum the N pieces for b in rank order (the plain driver's order) into this rank's output row;
//   AlltoAll (alg direct_push, alltoall__direct_push__generic.cu:17-33): piece j to CTA j; the consumers store
//     piece r (from rank r) into position r of this rank's output row;
//   AllGather (alg direct_replicated_push, allgather__direct_replicated_push__credit.cu:20-29): the whole unit to
//     every peer; the consumers store block r into position r of this rank's output row.
// Layout: mbarriers in a static array; dynamic window: input stages at kD0 + x * in_stage_bytes(U), then slot
// stages of slot_stage_bytes(U).
#define DSB_STREAM_TRAITS(OPKIND, PIECES, PUSH_ELEMS)                                                         \
    DSB_TRAITS(OPKIND, 0)                                                                                     \
    static constexpr int kMaxStages = 8;   /* per ring */                                                    \
    static constexpr int kConsumerWarps = 4;                                                                  \
    static constexpr int kThreads = 32 * (1 + kConsumerWarps);                                               \
    static constexpr uint32_t kPieces = PIECES; /* input pieces per unit */                                 \
    __host__ __device__ static constexpr uint32_t push_elems(uint32_t U) { return PUSH_ELEMS; }              \
    __host__ __device__ static constexpr uint64_t in_stage_bytes(uint32_t U) { return (uint64_t)kPieces * U * B; } \
    __host__ __device__ static constexpr uint64_t slot_stage_bytes(uint32_t U) {                             \
        return (uint64_t)(N_ - 1) * push_elems(U) * B;                                                        \
    }                                                                                                         \
    __host__ __device__ static constexpr uint64_t stage_bytes(uint32_t U) {                                  \
        return in_stage_bytes(U) + slot_stage_bytes(U);                                                       \
    }                                                                                                         \
    /* smallest launchable window: two input stages, one slot stage */                                       \
    __host__ __device__ static constexpr uint64_t smem_bytes(uint32_t U) {                                   \
        return kD0 + 2ull * in_stage_bytes(U) + slot_stage_bytes(U);                                          \
    }

template <int N_, typename T_, class Op_>
struct AR_RsGlobalAgStream {
    DSB_STREAM_TRAITS(AllReduce, 1u, U / N_)
    __host__ __device__ static constexpr bool legal(uint32_t U) { return AR_TwoShotPush<N_, T_, Op_>::legal(U); }
};
template <int N_, typename T_, class Op_>
struct RS_DirectPushStream {
    DSB_STREAM_TRAITS(ReduceScatter, (uint32_t)N_, U)
    __host__ __device__ static constexpr bool legal(uint32_t U) { return mult16(U * B); }
};
template <int N_, typename T_, class Op_>
struct A2A_DirectPushStream {
    DSB_STREAM_TRAITS(AllToAll, (uint32_t)N_, U)
    __host__ __device__ static constexpr bool legal(uint32_t U) { return mult16(U * B); }
};
template <int N_, typename T_, class Op_>
struct AG_ReplicatedPushStream {
    DSB_STREAM_TRAITS(AllGather, 1u, U)
    __host__ __device__ static constexpr bool legal(uint32_t U) { return mult16(U * B); }
};

template <class A>
__device__ __forceinline__ void stream_body(const BatchArgs& a) {
    using T = typename A::T;
    using Op = typename A::Op;
    constexpr int N = A::kN;
    constexpr OpKind kOp = A::kOp;
    constexpr uint32_t kNC = 32u * A::kConsumerWarps;   // consumer threads
    constexpr uint32_t kMax = A::kMaxStages;
    // full[x], done[x] per input stage; rs[r], credit[r] per slot stage
    __shared__ __align__(8) unsigned long long bars[4 * kMax];
    Ctx c;
    ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    flag_init(c);
    const uint32_t S = a.sub, U = a.M / S, UB = U * A::B;
    const uint32_t PB = A::push_elems(U) * A::B;                 // bytes pushed to each peer per unit
    const uint32_t XB = (uint32_t)A::in_stage_bytes(U), RB = (uint32_t)A::slot_stage_bytes(U);
    const uint32_t DX = min(max(a.depth, 2u), kMax), DR = min(max(a.lag, 1u), min(DX - 1u, kMax));
    const uint32_t slot_base = kD0 + DX * XB;
    auto full = [&](uint32_t x) { return smem_u32(&bars[x]); };
    auto done = [&](uint32_t x) { return smem_u32(&bars[kMax + x]); };
    auto rs = [&](uint32_t r) { return smem_u32(&bars[2 * kMax + r]); };
    auto credit = [&](uint32_t r) { return smem_u32(&bars[3 * kMax + r]); };
    auto X = [&](long long k) { return kD0 + (uint32_t)(k % DX) * XB; };
    auto R = [&](long long k) { return slot_base + (uint32_t)(k % DR) * RB; };   // slot i at R + i * PB
    if (threadIdx.x == 0) {
        for (uint32_t x = 0; x < DX; ++x) {
            mbar_init(full(x), 1);
            mbar_init(done(x), 1);
        }
        for (uint32_t r = 0; r < DR; ++r) {
            mbar_init(rs(r), 1);
            mbar_init(credit(r), N - 1);
        }
        fence_mbar_init();
    }
    cluster_sync();   // every barrier of the cluster initialised before any remote push or arrive
    const uint64_t in_r = in_elems_per_rank<A>(a.M), out_r = out_elems_per_rank<A>(a.M);
    const uint64_t total_in = (uint64_t)a.num_problems * N * in_r, total_out = (uint64_t)a.num_problems * N * out_r;
    const bool window_ok = slot_base + DR * RB <= a.smem_bytes;
    const T* in = static_cast<const T*>(a.in);
    T* out = static_cast<T*>(a.out);
    const long long step = (long long)num_clusters();
    const long long first = (long long)cluster_id();
    const long long mine = first < a.num_problems ? (a.num_problems - 1 - first) / step + 1 : 0;
    const long long units = window_ok ? mine * S : 0;
    if (!window_ok && threadIdx.x == 0) report(c, DSMEM_ERR_BIT_BOUNDS);
    auto problem_of = [&](long long k) { return first + (k / S) * step; };
    // rank r's row of unit k's problem, piece j (of M elements), sub-range k % S: element offsets
    auto in_off = [&](long long k, uint32_t r, uint32_t j) {
        return ((uint64_t)problem_of(k) * N + r) * in_r + (uint64_t)j * a.M + (uint64_t)(k % S) * U;
    };
    auto out_off = [&](long long k, uint32_t r, uint32_t j) {
        return ((uint64_t)problem_of(k) * N + r) * out_r + (uint64_t)j * a.M + (uint64_t)(k % S) * U;
    };
    // bounded wait for the phase of stage use `use` (parity use & 1) of barrier `bar`
    auto await = [&](uint32_t bar, long long use, int id) {
        const uint32_t par = (uint32_t)(use & 1);
        if (c.dead || mbar_try_wait_parity(bar, par)) return;
        if (!mbar_wait_parity_until(bar, par, c.deadline)) {
            c.dead = true;
            report_timeout(c, id);
        }
    };
    if (threadIdx.x == 0 && units > 0) {
        // ---------------------------------------------------------------- producer
        const long long ahead = (long long)(DX - DR);   // loads streaming in while DR units are exchanged
        auto issue_load = [&](long long k) {
            c.unit = (uint32_t)k;
            const uint32_t x = (uint32_t)(k % DX);
            if (in_off(k, c.rank, A::kPieces - 1) + U > total_in) {
                report(c, DSMEM_ERR_BIT_BOUNDS);
                return;
            }
            mbar_arrive_expect_tx(full(x), XB);
            for (uint32_t j = 0; j < A::kPieces; ++j)
                bulk_load_g2s(c.sa + X(k) + j * UB, in + in_off(k, c.rank, j), UB, full(x));
        };
        auto release = [&](long long j) {   // unit j consumed here and at every peer
            await(done((uint32_t)(j % DX)), j / DX, 3);
            await(credit((uint32_t)(j % DR)), j / DR, 2);
        };
        for (long long k = 0; k < units && k < ahead; ++k) issue_load(k);
        for (long long k = 0; k < units; ++k) {
            c.deadline = globaltimer() + c.wait_limit;
            if (k % S == 0 && a.smid != nullptr) a.smid[(uint64_t)problem_of(k) * N + c.rank] = smid();
            await(full((uint32_t)(k % DX)), k / DX, 0);
            if (k >= (long long)DR) release(k - DR);
            const uint32_t r = (uint32_t)(k % DR);
            mbar_arrive_expect_tx(rs(r), (N - 1) * PB);   // what the peers push for unit k
            for (uint32_t j = 1; j < (uint32_t)N; ++j) {
                const uint32_t dst = (c.rank + j) % N, slot = (c.rank + N - dst - 1) % N;
                // AllGather pushes the whole unit; the others the part owned by dst
                const uint32_t to = R(k) + slot * PB, from = X(k) + (kOp == OpKind::AllGather ? 0u : dst * PB);
                if (((to | from | PB) & 15u) != 0u || PB == 0u || to + PB > c.smem_bytes || from + PB > c.smem_bytes) {
                    report(c, DSMEM_ERR_BIT_BOUNDS);
                    continue;
                }
                bulk_push(dst, c.sa + to, c.sa + from, PB, rs(r));
            }
            // the input stage of unit k + DX - DR is unit k - DR's, released above
            if (k + ahead < units) issue_load(k + ahead);
        }
        c.deadline = globaltimer() + c.wait_limit;
        for (long long j = units > (long long)DR ? units - DR : 0; j < units; ++j)
            await(credit((uint32_t)(j % DR)), j / DR, 2);
    } else if (threadIdx.x >= 32) {
        // ---------------------------------------------------------------- consumers
        const uint32_t tc = threadIdx.x - 32, nl = PB >> 4;   // 16-byte lanes of one pushed part
        for (long long k = 0; k < units; ++k) {
            const uint32_t sub = (uint32_t)(k % S);
            c.unit = (uint32_t)k;
            c.deadline = globaltimer() + c.wait_limit;
            unsigned long long* st = a.stamps != nullptr && tc == 0
                                         ? a.stamps + ((uint64_t)problem_of(k) * N + c.rank) * kStamps
                                         : nullptr;
            await(full((uint32_t)(k % DX)), k / DX, 0);
            if (st != nullptr && sub == 0) st[0] = globaltimer();
            await(rs((uint32_t)(k % DR)), k / DR, 1);
            if (st != nullptr && sub + 1 == S) st[2] = globaltimer();
            // the part from rank r: this rank's own part from the input stage, the others from their slots
            const uint4* own = c.ptr<const uint4>(X(k) + (kOp == OpKind::AllGather ? 0u : c.rank * PB));
            const uint4* slots = c.ptr<const uint4>(R(k));
            auto part = [&](int r) { return r == (int)c.rank ? own : slots + ((r + N - (int)c.rank - 1) % N) * nl; };
            if constexpr (kOp == OpKind::AllReduce || kOp == OpKind::ReduceScatter) {
                // AllReduce: the sum of chunk b into position b of all N output rows; ReduceScatter: into this
                // rank's output row
                constexpr int kRows = kOp == OpKind::AllReduce ? N : 1;
                uint4* rows[kRows];
                bool ok = true;
#pragma unroll
                for (int r = 0; r < kRows; ++r) {
                    const uint64_t o = kOp == OpKind::AllReduce
                                           ? out_off(k, (uint32_t)r, 0) + (uint64_t)c.rank * A::push_elems(U)
                                           : out_off(k, c.rank, 0);
                    ok = ok && o + A::push_elems(U) <= total_out;
                    rows[r] = reinterpret_cast<uint4*>(out + o);
                }
                if (!ok) {
                    if (tc == 0) report(c, DSMEM_ERR_BIT_BOUNDS);
                } else {
                    for (uint32_t u = tc; u < nl; u += kNC) {
                        uint4 v[N];
#pragma unroll
                        for (int r = 0; r < N; ++r) v[r] = part(r)[u];
                        auto acc = Pk<T, Op>::open(v[0]);
#pragma unroll
                        for (int r = 1; r < N; ++r) Pk<T, Op>::add(acc, v[r]);
                        const uint4 res = Pk<T, Op>::close(acc);
#pragma unroll
                        for (int r = 0; r < kRows; ++r) __stcs(rows[r] + u, res);
                    }
                }
            } else {
                // AlltoAll / AllGather: the part from rank r into position r of this rank's output row
                if (out_off(k, c.rank, N - 1) + U > total_out) {
                    if (tc == 0) report(c, DSMEM_ERR_BIT_BOUNDS);
                } else {
                    uint4* row = reinterpret_cast<uint4*>(out + out_off(k, c.rank, 0));
                    const uint32_t stride = a.M * A::B >> 4;   // 16-byte units between the row's positions
                    for (uint32_t idx = tc; idx < (uint32_t)N * nl; idx += kNC) {
                        const uint32_t r = idx / nl, u = idx - r * nl;
                        __stcs(row + (uint64_t)r * stride + u, part((int)r)[u]);
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kNC) : "memory");   // every consumer has read the stages
            if (tc == 0) {
                // relaxed: the credits only release the stages' shared memory, whose reads are complete (their
                // values are already stored); a release arrive would also wait for the global stores just
                // issued (~4 us under load) and stall the consumers on every unit
                for (uint32_t j = 1; j < (uint32_t)N; ++j)
                    mbar_arrive_remote_relaxed(credit((uint32_t)(k % DR)), (c.rank + j) % N);
                mbar_arrive_relaxed(done((uint32_t)(k % DX)));
                if (st != nullptr && sub + 1 == S) st[1] = globaltimer();
            }
        }
    }
    finish(c);   // no CTA leaves while a peer may still push into it
}

// The AllReduce's streamed driver (the name the profiles and the bench name).
template <class A>
__global__ void __launch_bounds__(A::kThreads) rs_global_ag_stream_kernel(const BatchArgs a) {
    stream_body<A>(a);
}
// The streamed drivers of ReduceScatter, AlltoAll and AllGather.
template <class A>
__global__ void __launch_bounds__(A::kThreads) collective_stream_kernel(const BatchArgs a) {
    stream_body<A>(a);
}

// Reference harness contract (collectives/harness/main.cu): one cluster, compile-time M.
template <class A>
__device__ __forceinline__ void run_single(const typename A::T* in, typename A::T* out, unsigned long long* ts,
                                           unsigned* smid_out, uint32_t M, uint32_t smem_bytes) {
    Ctx c;
    ctx_init(c, smem_bytes, nullptr, DSMEM_WAIT_LIMIT_NS);
    flag_init(c);
    init_bars<A>(c);
    c.st.base = ts != nullptr ? ts + c.rank * kStamps : nullptr;
    c.deadline = globaltimer() + c.wait_limit;
    A::load(c, in + c.rank * in_elems_per_rank<A>(M), M);
    if (smid_out != nullptr && threadIdx.x == 0) smid_out[c.rank] = smid();
    cluster_sync();
    c.st.mark(0);
    A::exec(c, M);
    c.st.mark(1);
    A::store(c, out + c.rank * out_elems_per_rank<A>(M), M);
    finish(c);
}

}  // namespace dsb
