// ext_rmsnorm.cu -- cluster-fused RMSNorm for sm_100a.
//
// Computes, per row, y = h * rsqrt(mean(h^2) + eps) * w with h = x (+ residual, written back as the
// pre-norm row when requested), bf16 or f32 in/out, fp32 statistics. Reference kernels:
//   kernels/rmsnorm__llama__clusterfusion.cu:35-108   row per cluster, CTA b owns columns
//     [b*H/N, (b+1)*H/N), partial sum of squares by warp shuffles, cluster AllReduce of one float;
//   kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197   h = x + residual written back,
//     replicated-push scalar AllReduce (one store into slot[b] of every CTA) (:153-169).
// B200 design (one launch, persistent clusters of N CTAs, 256 threads = 8 warps per CTA):
//   * rows are taken in groups of R = 8*K (K = 4 rows per warp, 2 for 2 KiB slices); cluster q handles
//     groups q, q + nclusters, ...;
//   * each CTA streams the R row slices of a group with one-CTA bulk copies (cp.async.bulk, no
//     multicast) through a ring of 3 shared-memory stages (2 with a residual), refilled as soon as every
//     warp has moved its rows into registers (full/empty mbarriers);
//   * the AllReduce of the per-row partial sums is the replicated push of hpc-ops: lane 0 of each warp
//     writes its K partials into slot[parity][b][warp*K..] of every CTA of the cluster with one st.async
//     each, whose bytes complete on that CTA's mbarrier (armed for N*R*4 bytes per group), so no release
//     fence or cluster barrier is needed per group; a warp waits and sums the N slots of each of its rows.
//     Two slot sets alternate between groups; a peer can reuse a set only after it received all of this
//     CTA's partials of the following group, which are sent after this CTA has read the set;
//   * outputs leave from registers with 16-byte streaming stores.
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"

namespace {

using namespace dsmem;

constexpr int kWarps = 8;          // rows per group
constexpr int kThreadsRms = kWarps * 32;
constexpr int kMaxUnitsPerLane = 4;   // 16-byte units of a row slice per lane (slice <= 4*32*16 B = 2 KiB)

struct RmsArgs {
    const void* x;
    const void* res;     // nullable
    const void* w;
    void* y;
    void* pre;           // nullable: h = x + res
    unsigned* err;
    unsigned long long wait_limit_ns;
    long long rows;
    int hidden;
    float eps;
    uint32_t slice_bytes;   // bytes of one row slice of one CTA
    uint32_t smem_bytes;
};

template <typename T>
struct RmsElem;
template <>
struct RmsElem<__nv_bfloat16> {
    static constexpr int kPer16 = 8;
    static __device__ __forceinline__ void unpack(uint4 p, float* f) {
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
            f[2 * k] = v.x;
            f[2 * k + 1] = v.y;
        }
    }
    static __device__ __forceinline__ uint4 pack(const float* f) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
            w[k] = *reinterpret_cast<const uint32_t*>(&h);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};
template <>
struct RmsElem<float> {
    static constexpr int kPer16 = 4;
    static __device__ __forceinline__ void unpack(uint4 p, float* f) {
        f[0] = __uint_as_float(p.x);
        f[1] = __uint_as_float(p.y);
        f[2] = __uint_as_float(p.z);
        f[3] = __uint_as_float(p.w);
    }
    static __device__ __forceinline__ uint4 pack(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
};

// Rows per warp per iteration for UPL 16-byte units per lane: x stays in registers as K*UPL packets.
__host__ __device__ constexpr int rms_k(int upl) { return upl >= 4 ? 2 : 4; }
__host__ __device__ constexpr int rms_stages(bool residual) { return residual ? 2 : 3; }

// Shared-memory layout: [0,128) barriers | slots 2 x N x R floats | w slice | stages x R x slice (x2 with residual)
__host__ __device__ constexpr uint32_t rms_slots_off() { return 128u; }
__host__ __device__ constexpr uint32_t rms_w_off(int n, int r) { return 128u + ((2u * n * r * 4u + 15u) & ~15u); }
__host__ __device__ constexpr uint32_t rms_stage_off(int n, int r, uint32_t slice) { return rms_w_off(n, r) + slice; }
__host__ __device__ constexpr uint32_t rms_smem(int n, int r, uint32_t slice, bool residual) {
    return rms_stage_off(n, r, slice) + (uint32_t)rms_stages(residual) * r * slice * (residual ? 2u : 1u);
}

// One K-float remote store with completion on the destination's mbarrier (st.async, no release fence).
template <int K>
__device__ __forceinline__ void st_async_partials(uint32_t dst_rank, uint32_t dst, const float* v, uint32_t bar) {
    const uint32_t rd = mapa(dst, dst_rank), rb = mapa(bar, dst_rank);
    if constexpr (K == 4) {
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1,%2,%3,%4}, [%5];" ::"r"(rd),
                     "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "r"(rb)
                     : "memory");
    } else {
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1,%2}, [%3];" ::"r"(rd),
                     "f"(v[0]), "f"(v[1]), "r"(rb)
                     : "memory");
    }
}

template <int N, typename T, bool RES, int UPL>
__global__ void __launch_bounds__(kThreadsRms, 2) rmsnorm_cluster_kernel(const RmsArgs a) {
    using E = RmsElem<T>;
    constexpr int K = rms_k(UPL);          // rows per warp per iteration
    constexpr int R = kWarps * K;          // rows per CTA per iteration
    constexpr int NS = rms_stages(RES);
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t slice = a.slice_bytes, units = slice >> 4;   // 16-B units per row slice (<= 32 * UPL)
    const uint32_t slots = rms_slots_off(), woff = rms_w_off(N, R), stage0 = rms_stage_off(N, R, slice);
    const uint32_t stage_bytes = (uint32_t)R * slice * (RES ? 2u : 1u);
    const long long groups = (a.rows + R - 1) / R;
    const long long step = (long long)num_clusters();
    const long long first = (long long)cluster_id();
    const size_t row_bytes = (size_t)a.hidden * sizeof(T);
    const size_t col_off = (size_t)c.rank * slice;
    const unsigned char* xb = static_cast<const unsigned char*>(a.x);
    const unsigned char* rb = static_cast<const unsigned char*>(a.res);
    constexpr int kFull = 0, kEmpty = NS, kSum = 2 * NS;   // barrier ids

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(c.bar(kFull + s), 1);
            mbar_init(c.bar(kEmpty + s), kWarps);
        }
        mbar_init(c.bar(kSum + 0), 1);
        mbar_init(c.bar(kSum + 1), 1);
        fence_mbar_init();
    }
    {   // weight slice -> shared
        const uint4* wsrc = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(a.w) + col_off);
        uint4* wdst = c.ptr<uint4>(woff);
        for (uint32_t i = threadIdx.x; i < units; i += blockDim.x) wdst[i] = __ldg(wsrc + i);
    }
    __syncthreads();
    cluster_sync();   // barriers of every CTA initialised before any remote store completes on them

    // producer (thread 0): loads of local iteration i into stage i % NS
    auto issue = [&](long long i_local) {
        const long long g = first + i_local * step;
        if (g >= groups) return;
        const int s = (int)(i_local % NS);
        const long long r0 = g * R;
        const int nr = (int)min((long long)R, a.rows - r0);
        const uint32_t dst = stage0 + (uint32_t)s * stage_bytes;
        dsb::arm(c, kFull + s, (uint32_t)nr * slice * (RES ? 2u : 1u));
        for (int r = 0; r < nr; ++r) {
            const size_t src = (size_t)(r0 + r) * row_bytes + col_off;
            bulk_load_g2s(c.sa + dst + (uint32_t)r * slice, xb + src, slice, c.bar(kFull + s));
            if (RES) bulk_load_g2s(c.sa + dst + ((uint32_t)R + r) * slice, rb + src, slice, c.bar(kFull + s));
        }
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < NS; ++i) issue(i);

    const uint4* wp = c.ptr<const uint4>(woff);
    long long i = 0;
    for (long long g = first; g < groups; g += step, ++i) {
        const int s = (int)(i % NS);
        const uint32_t par = (uint32_t)(i & 1);
        const long long row0 = g * R + (long long)warp * K;
        c.deadline = globaltimer() + c.wait_limit;
        // expect this iteration's partials: N CTAs x R rows x 4 bytes
        if (threadIdx.x == 0) dsb::arm(c, kSum + (int)par, (uint32_t)N * R * 4u);
        dsb::wait(c, kFull + s);
        // ---- my K row slices -> registers (packed), sums of squares
        uint4 xp[K][UPL];
        float ss[K];
        {
            const uint4* xs = c.ptr<const uint4>(stage0 + (uint32_t)s * stage_bytes);
            const uint4* rs = xs + (size_t)R * (slice >> 4);
#pragma unroll
            for (int k = 0; k < K; ++k) {
                ss[k] = 0.f;
                const bool valid = row0 + k < a.rows;
#pragma unroll
                for (int j = 0; j < UPL; ++j) {
                    const uint32_t u = lane + 32u * j;
                    if (valid && u < units) {
                        const uint32_t idx = (warp * K + k) * units + u;
                        float f[E::kPer16];
                        E::unpack(xs[idx], f);
                        if (RES) {
                            float r[E::kPer16];
                            E::unpack(rs[idx], r);
#pragma unroll
                            for (int e = 0; e < E::kPer16; ++e) f[e] += r[e];
                            xp[k][j] = E::pack(f);   // h rounded to the element type (the pre-norm output)
                            E::unpack(xp[k][j], f);
                        } else {
                            xp[k][j] = xs[idx];
                        }
#pragma unroll
                        for (int e = 0; e < E::kPer16; ++e) ss[k] = fmaf(f[e], f[e], ss[k]);
                    } else {
                        xp[k][j] = make_uint4(0, 0, 0, 0);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(c.bar(kEmpty + s));   // this warp no longer needs the stage
        if (threadIdx.x == 0) {   // refill the stage for iteration i + NS once every warp released it
            const uint32_t epar = (c.phase >> (kEmpty + s)) & 1u;
            c.phase ^= 1u << (kEmpty + s);
            if (!c.dead && !mbar_wait_parity_until(c.bar(kEmpty + s), epar, c.deadline)) {
                c.dead = true;
                dsb::report(c, DSMEM_ERR_BIT_TIMEOUT);
            }
            issue(i + NS);
        }
        // ---- cluster AllReduce of the K partial sums: replicated push with st.async into slot[par][b][w*K..]
#pragma unroll
        for (int k = 0; k < K; ++k)
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], off);
        if (lane == 0) {
            const uint32_t dst = slots + ((par * N + c.rank) * R + warp * K) * 4u;
            for (uint32_t q = 0; q < (uint32_t)N; ++q) st_async_partials<K>(q, c.sa + dst, ss, c.bar(kSum + (int)par));
        }
        dsb::wait(c, kSum + (int)par);
        float scale[K];
        {
            const float* sl = c.ptr<const float>(slots + par * N * R * 4u);
#pragma unroll
            for (int k = 0; k < K; ++k) {
                float tot = 0.f;
#pragma unroll
                for (int q = 0; q < N; ++q) tot += sl[q * R + warp * K + k];
                scale[k] = rsqrtf(tot / (float)a.hidden + a.eps);
            }
        }
        // ---- normalise and store
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const long long row = row0 + k;
            if (row >= a.rows) continue;
            uint4* yo = reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.y) + (size_t)row * row_bytes + col_off);
            uint4* po = RES && a.pre != nullptr
                            ? reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.pre) + (size_t)row * row_bytes + col_off)
                            : nullptr;
#pragma unroll
            for (int j = 0; j < UPL; ++j) {
                const uint32_t u = lane + 32u * j;
                if (u < units) {
                    if (RES && po != nullptr) __stcs(po + u, xp[k][j]);
                    float f[E::kPer16], w[E::kPer16];
                    E::unpack(xp[k][j], f);
                    E::unpack(wp[u], w);
#pragma unroll
                    for (int e = 0; e < E::kPer16; ++e) f[e] = f[e] * scale[k] * w[e];
                    __stcs(yo + u, E::pack(f));
                }
            }
        }
    }
    cluster_sync();   // no CTA leaves while a peer may still store into its slots
}

struct RmsKey {
    const void* fn;
    int dev;
    uint32_t smem;
    bool operator<(const RmsKey& o) const {
        return fn < o.fn || (fn == o.fn && (dev < o.dev || (dev == o.dev && smem < o.smem)));
    }
};
std::mutex g_mu;
std::map<RmsKey, int> g_occ;
unsigned* g_err[64] = {};

template <int N, typename T, bool RES>
const void* rms_fn(int upl) {
    switch (upl) {
        case 1: return reinterpret_cast<const void*>(&rmsnorm_cluster_kernel<N, T, RES, 1>);
        case 2: return reinterpret_cast<const void*>(&rmsnorm_cluster_kernel<N, T, RES, 2>);
        case 4: return reinterpret_cast<const void*>(&rmsnorm_cluster_kernel<N, T, RES, 4>);
    }
    return nullptr;
}

template <typename T, bool RES>
const void* pick(int n, int upl) {
    switch (n) {
        case 1: return rms_fn<1, T, RES>(upl);
        case 2: return rms_fn<2, T, RES>(upl);
        case 4: return rms_fn<4, T, RES>(upl);
        case 8: return rms_fn<8, T, RES>(upl);
        case 16: return rms_fn<16, T, RES>(upl);
    }
    return nullptr;
}

dsmem_status rms_launch(int dtype, const void* x, const void* res, const void* w, void* y, void* pre, float eps,
                        long long rows, int hidden, int cluster_size, int max_clusters, cudaStream_t stream) {
    if (x == nullptr || w == nullptr || y == nullptr || rows < 0 || hidden <= 0 || !(eps >= 0.f))
        return DSMEM_ERR_INVALID_ARGUMENT;
    if (dtype != DSMEM_BF16 && dtype != DSMEM_F32) return DSMEM_ERR_ILLEGAL_CONFIG;
    const int n = cluster_size;
    if (!(n == 1 || n == 2 || n == 4 || n == 8 || n == 16)) return DSMEM_ERR_INVALID_ARGUMENT;
    const size_t eb = dtype == DSMEM_BF16 ? 2 : 4;
    if ((size_t)hidden % n) return DSMEM_ERR_ILLEGAL_CONFIG;
    const size_t slice = (size_t)hidden / n * eb;
    if (slice % 16 || slice / 16 > (size_t)kMaxUnitsPerLane * 32) return DSMEM_ERR_ILLEGAL_CONFIG;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(res) | reinterpret_cast<uintptr_t>(pre);
    if (al & 15u) return DSMEM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DSMEM_OK;
    const bool has_res = res != nullptr;
    const uint32_t units = (uint32_t)(slice / 16);
    const int upl = units <= 32 ? 1 : units <= 64 ? 2 : 4;
    const int r = kWarps * rms_k(upl);
    const uint32_t smem = rms_smem(n, r, (uint32_t)slice, has_res);
    if (smem > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    const void* fn = dtype == DSMEM_BF16
                         ? (has_res ? pick<__nv_bfloat16, true>(n, upl) : pick<__nv_bfloat16, false>(n, upl))
                         : (has_res ? pick<float, true>(n, upl) : pick<float, false>(n, upl));
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreadsRms, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int resident = 0;
    RmsArgs a{};
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_err[dev] == nullptr) {
            if (cudaMalloc(&g_err[dev], sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(g_err[dev], 0, sizeof(unsigned));
        }
        const RmsKey key{fn, dev, smem};
        auto it = g_occ.find(key);
        if (it == g_occ.end()) {
            if (n > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                return DSMEM_ERR_CUDA;
            if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return DSMEM_ERR_CUDA;
            if (cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared) != cudaSuccess)
                return DSMEM_ERR_CUDA;
            cfg.gridDim = dim3((unsigned)n, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&resident, fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
            g_occ[key] = resident;
        } else {
            resident = it->second;
        }
        a.err = g_err[dev];
    }
    if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;
    const long long groups = (rows + r - 1) / r;
    long long clusters = std::min<long long>(groups, resident);
    if (max_clusters > 0) clusters = std::min<long long>(clusters, max_clusters);
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    a.x = x;
    a.res = res;
    a.w = w;
    a.y = y;
    a.pre = pre;
    a.wait_limit_ns = 1000000000ull;
    a.rows = rows;
    a.hidden = hidden;
    a.eps = eps;
    a.slice_bytes = (uint32_t)slice;
    a.smem_bytes = smem;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

}  // namespace

extern "C" {

dsmem_status dsmem_rmsnorm_launch(dsmem_dtype dtype, const void* x, const void* w, float eps, long long rows,
                                  int hidden, int cluster_size, void* y, dsmem_stream_t stream) {
    return rms_launch(dtype, x, nullptr, w, y, nullptr, eps, rows, hidden, cluster_size, 0,
                      reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_rmsnorm_residual_launch(dsmem_dtype dtype, const void* x, const void* residual, const void* w,
                                           float eps, long long rows, int hidden, int cluster_size, void* pre_norm,
                                           void* y, dsmem_stream_t stream) {
    if (residual == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    return rms_launch(dtype, x, residual, w, y, pre_norm, eps, rows, hidden, cluster_size, 0,
                      reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_rmsnorm_check(int device, unsigned* error_bits) {
    unsigned v = 0;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (device < 0 || device >= 64) return DSMEM_ERR_INVALID_ARGUMENT;
        if (g_err[device] != nullptr) {
            if (cudaMemcpy(&v, g_err[device], sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(g_err[device], 0, sizeof v);
        }
    }
    if (error_bits) *error_bits = v;
    return DSMEM_OK;
}

}  // extern "C"
