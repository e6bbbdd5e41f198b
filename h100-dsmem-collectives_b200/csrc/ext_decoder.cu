// ext_decoder.cu -- Llama-2-7B-shaped decoder layer, one decode step, cluster-fused, sm_100a.
//
// Reference: kernels/fused_decoder_layer__llama2_7b__clusterfusion.cu:101-268, 291-922 (attention block,
// cluster_reduce between stages) and the layer maths of
// roofline/harness/workloads/clusterfusion_llama2_7b_decoder.py:160-180 (reference_fp32, with the FFN tail):
//   x = inp + res; xn = RMSNorm(x) w_rms; qkv = xn Wqkv^T; q, k = NEOX RoPE(q, k); append k, v to the cache;
//   a = softmax(q K^T / sqrt(D)) V over the cache and the new token; o = a Wo^T; h = x + o;
//   hn = RMSNorm(h) w_post; out = (SiLU(hn Wg^T) * hn Wu^T) Wd^T.
// B200 design: seven stream-ordered launches, every stage HBM-bound (weights read once per step, the KV
// cache once per sequence):
//   1. cluster RMSNorm of x = inp + res (ext_rmsnorm.cu: x and xn written once);
//   2. QKV projection: one cluster per 128-feature tile, the cluster's N CTAs split K; each warp streams
//      16 weight rows with 16-byte loads straight into mma.sync m16n8k16 A fragments (bf16, fp32
//      accumulate; the activation K-slice sits in shared memory in fragment order, so the k order
//      within a 32-wide block is permuted identically on both operands); the N partial tiles meet by
//      DSMEM loads (reduce-scatter by feature pairs (i, i+64)), whose owner applies RoPE and writes q
//      (fp32) and the new k, v into the cache;
//   3. decode attention: one cluster per (sequence, head), the cluster's CTAs split the keys and stream
//      them through a 4-stage shared-memory ring of 32-key K/V tiles (16-byte cp.async); groups of 8
//      lanes take one key of a tile at a time (16 dims a lane), online softmax in base 2; then the
//      partial (max, sum, acc) of the 32 groups meet in shared memory and the N CTAs' in DSMEM;
//   4. O projection (as 2) with the epilogue h = x + o;
//   5. cluster RMSNorm of h;
//   6. gate/up projection (as 2; a tile holds gate rows j and up rows j of the same 64 j) with the
//      epilogue SiLU(gate) * up;
//   7. down projection (as 2).
// Tensor cores run through the legacy mma.sync path (the B operand is only 8-16 tokens wide, so the
// projections stay HBM-bound on it).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "f32x2.cuh"

namespace {

using namespace dsmem;
using namespace dsb2;
using bf16 = __nv_bfloat16;

constexpr int kHeadDim = 128;
constexpr int kTile = 128;           // output features per cluster tile
constexpr int kProjThreads = 256;    // 8 warps x 16 feature rows
constexpr int kAttnThreads = 256;    // 32 groups of 8 lanes
constexpr uint32_t kArea = 128;      // barrier area / finish flag at the start of the dynamic window

enum Epi : int { kEpiQKV = 0, kEpiO = 1, kEpiGateUp = 2, kEpiDown = 3 };

struct ProjArgs {
    const bf16* W;        // [rows][K] (nn.Linear layout)
    const bf16* act;      // [B][K]
    int K;
    int B;
    int ffn;              // gate/up: up rows start at ffn
    int H;                // heads (QKV)
    long long cap;        // cache capacity in tokens (QKV)
    long long S;          // cached tokens before this step: the new token goes to index S
    float* q;             // QKV: [B][H][D] fp32, RoPE applied
    bf16* kc;             // QKV: caches [B][cap][H][D]
    bf16* vc;
    bf16* knew;           // QKV: [B][H][D] or nullptr
    bf16* vnew;
    const float* cosv;    // [D]
    const float* sinv;
    const bf16* x;        // O: the residual stream [B][hidden]
    bf16* o_out;          // O: attention-block output [B][hidden] or nullptr
    bf16* h_out;          // O: h = x + o
    bf16* out;            // gate/up: [B][ffn]; down: [B][hidden]
    int out_ld;
    uint32_t smem_bytes;
    unsigned* err;
};

__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <int EPI>
__device__ __forceinline__ long long weight_row(int tile, int lrow, int ffn) {
    if constexpr (EPI == kEpiGateUp) return lrow < 64 ? 64LL * tile + lrow : (long long)ffn + 64LL * tile + (lrow - 64);
    return (long long)kTile * tile + lrow;
}

// One cluster = one 128-feature tile; CTA `rank` of the cluster reduces K-slice `rank`.
template <int EPI, int N, int NT>
__global__ void __launch_bounds__(kProjThreads) proj_kernel(const ProjArgs a) {
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, 1000000000ull);
    dsb::flag_init(c);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tile = (int)cluster_id();
    const int Kc = a.K / N, k0 = (int)c.rank * Kc, nkb = Kc / 32;
    uint2* frag = c.ptr<uint2>(kArea);                              // B fragments of the K-slice
    const uint32_t frag_bytes = (uint32_t)nkb * 2u * NT * 32u * 8u;
    float* part = c.ptr<float>(kArea + frag_bytes);                // [128][8*NT] partial tile
    constexpr int NB = 8 * NT;

    // 1. the activation K-slice in fragment order: entry ((kb*2 + s)*NT + j)*32 + lane holds, for batch
    //    row n = lane/4 + 8j, the 4 elements k0 + 32kb + 8(lane%4) + 4s .. +3 (zeros past B)
    for (int e = threadIdx.x; e < nkb * 2 * NT * 32; e += blockDim.x) {
        const int l = e & 31, rest = e >> 5, j = rest % NT, s = (rest / NT) & 1, kb = rest / NT / 2;
        const int n = (l >> 2) + 8 * j;
        const int k = k0 + kb * 32 + 8 * (l & 3) + 4 * s;
        uint2 v = make_uint2(0u, 0u);
        if (n < a.B) v = *reinterpret_cast<const uint2*>(a.act + (size_t)n * a.K + k);
        frag[e] = v;
    }
    __syncthreads();

    // 2. this warp's 16 rows: lane (g, t) streams 16 B of rows g and g+8 per 32-wide k block; the k
    //    order inside a block is permuted the same way for A (here) and B (the fragments above)
    const int lrow0 = warp * 16 + g, lrow1 = lrow0 + 8;
    const uint4* w0 = reinterpret_cast<const uint4*>(a.W + weight_row<EPI>(tile, lrow0, a.ffn) * a.K + k0) + t;
    const uint4* w1 = reinterpret_cast<const uint4*>(a.W + weight_row<EPI>(tile, lrow1, a.ffn) * a.K + k0) + t;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const uint2* fr = frag + lane;
    // weights for kU k-blocks at a time, the next batch's loads issued before this batch's MMAs, so a lane
    // keeps 2 * kU (up to 4 * kU) 16-byte loads in flight
    constexpr int kU = 4;
    uint4 cur0[kU], cur1[kU], nxt0[kU], nxt1[kU];
    auto fetch = [&](uint4* d0, uint4* d1, int kb0) {
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (kb0 + u < nkb) {
                d0[u] = ld_stream(w0 + 4 * (kb0 + u));
                d1[u] = ld_stream(w1 + 4 * (kb0 + u));
            }
    };
    fetch(cur0, cur1, 0);
    for (int kb0 = 0; kb0 < nkb; kb0 += kU) {
        if (kb0 + kU < nkb) fetch(nxt0, nxt1, kb0 + kU);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int kb = kb0 + u;
            if (kb < nkb) {
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint2 b0 = fr[((kb * 2 + 0) * NT + j) * 32];
                    const uint2 b1 = fr[((kb * 2 + 1) * NT + j) * 32];
                    mma_bf16(acc[j], cur0[u].x, cur1[u].x, cur0[u].y, cur1[u].y, b0.x, b0.y);
                    mma_bf16(acc[j], cur0[u].z, cur1[u].z, cur0[u].w, cur1[u].w, b1.x, b1.y);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            cur0[u] = nxt0[u];
            cur1[u] = nxt1[u];
        }
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {   // D fragment: (row g, cols 2t, 2t+1), (row g+8, cols 2t, 2t+1)
        part[lrow0 * NB + 8 * j + 2 * t] = acc[j][0];
        part[lrow0 * NB + 8 * j + 2 * t + 1] = acc[j][1];
        part[lrow1 * NB + 8 * j + 2 * t] = acc[j][2];
        part[lrow1 * NB + 8 * j + 2 * t + 1] = acc[j][3];
    }
    cluster_sync();   // every CTA's partial tile is complete and visible

    // 3. reduce-scatter by feature pairs (i, i+64) over the cluster (rank order), then the epilogue
    const int npairs = 64 / N;
    const uint32_t part_sa = c.sa + kArea + frag_bytes;
    for (int e = threadIdx.x; e < npairs * a.B; e += blockDim.x) {
        const int i = (int)c.rank * npairs + e / a.B, n = e % a.B;
        float lo = 0.f, hi = 0.f;
#pragma unroll
        for (int r = 0; r < N; ++r) {
            lo += ld_cluster_f32(mapa(part_sa + (uint32_t)(i * NB + n) * 4u, (uint32_t)r));
            hi += ld_cluster_f32(mapa(part_sa + (uint32_t)((i + 64) * NB + n) * 4u, (uint32_t)r));
        }
        if constexpr (EPI == kEpiQKV) {
            const int which = tile / a.H, head = tile % a.H;   // 0 q, 1 k, 2 v
            float o0 = lo, o1 = hi;
            if (which < 2) {   // NEOX rotation of the pair (i, i+64)
                o0 = lo * a.cosv[i] - hi * a.sinv[i];
                o1 = hi * a.cosv[i + 64] + lo * a.sinv[i + 64];
            }
            const size_t hd = ((size_t)n * a.H + head) * kHeadDim;
            if (which == 0) {
                a.q[hd + i] = o0;
                a.q[hd + i + 64] = o1;
            } else {
                bf16* cache = which == 1 ? a.kc : a.vc;
                bf16* fresh = which == 1 ? a.knew : a.vnew;
                const size_t ci = (((size_t)n * a.cap + a.S) * a.H + head) * kHeadDim;
                cache[ci + i] = __float2bfloat16_rn(o0);
                cache[ci + i + 64] = __float2bfloat16_rn(o1);
                if (fresh != nullptr) {
                    fresh[hd + i] = __float2bfloat16_rn(o0);
                    fresh[hd + i + 64] = __float2bfloat16_rn(o1);
                }
            }
        } else if constexpr (EPI == kEpiO) {
            const size_t f = (size_t)kTile * tile + i, row = (size_t)n * a.out_ld;
            const float x0 = __bfloat162float(a.x[row + f]), x1 = __bfloat162float(a.x[row + f + 64]);
            a.h_out[row + f] = __float2bfloat16_rn(x0 + lo);
            a.h_out[row + f + 64] = __float2bfloat16_rn(x1 + hi);
            if (a.o_out != nullptr) {
                a.o_out[row + f] = __float2bfloat16_rn(lo);
                a.o_out[row + f + 64] = __float2bfloat16_rn(hi);
            }
        } else if constexpr (EPI == kEpiGateUp) {
            const float silu = lo / (1.0f + expf(-lo));
            a.out[(size_t)n * a.out_ld + 64 * tile + i] = __float2bfloat16_rn(silu * hi);
        } else {
            const size_t f = (size_t)kTile * tile + i, row = (size_t)n * a.out_ld;
            a.out[row + f] = __float2bfloat16_rn(lo);
            a.out[row + f + 64] = __float2bfloat16_rn(hi);
        }
    }
    dsb::finish(c);   // peers have finished reading my partial tile
}

struct AttnArgs {
    const float* q;       // [B][H][D], RoPE applied
    const bf16* kc;       // [B][cap][H][D]
    const bf16* vc;
    bf16* a_out;          // [B][H][D]
    long long cap;
    long long L;          // keys: the S cached tokens and the new one
    int H;
    float scale_log2;     // log2(e) / sqrt(D)
    uint32_t smem_bytes;
    unsigned* err;
};

constexpr int kKeyTile = 32;                       // keys per shared-memory tile
constexpr int kAttnStages = 4;                     // tiles in flight
constexpr uint32_t kTileBytes = kKeyTile * kHeadDim * 2u;   // one K (or V) tile, 8 KiB
constexpr int kAttnGroups = kAttnThreads / 8;      // 32 groups of 8 lanes, one key each per step
// shared memory: [kArea) flag | stages x (K tile, V tile) | group partials (m, l, acc[128]) | CTA partial
constexpr uint32_t kAttnStageOff = kArea;
constexpr uint32_t kAttnGroupOff = kAttnStageOff + kAttnStages * 2u * kTileBytes;
constexpr uint32_t kAttnCtaOff = kAttnGroupOff + (uint32_t)kAttnGroups * (2 + kHeadDim) * 4u;
constexpr uint32_t kAttnSmem = kAttnCtaOff + (2 + kHeadDim) * 4u;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int K>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(K) : "memory");
}

// One cluster = one (sequence, head); CTA r of N takes keys [r*L/N, (r+1)*L/N). The CTA streams its keys
// through kAttnStages shared-memory tiles of 32 keys (16-byte cp.async, so the loads of several tiles are
// in flight while one is consumed); 32 groups of 8 lanes each take one key of a tile per step, a lane owning
// 16 of the 128 dimensions; online softmax in base 2. Then the 32 groups' (max, sum, acc) meet in shared
// memory and the N CTAs' in DSMEM.
template <int N>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, 1000000000ull);
    dsb::flag_init(c);
    const int cid = (int)cluster_id(), b = cid / a.H, head = cid % a.H;
    const int lane = threadIdx.x & 31, sub = lane & 7, grp = threadIdx.x >> 3;
    const unsigned gmask = 0xFFu << (lane & 24);   // the 8 lanes of this group
    const long long lo = (long long)c.rank * a.L / N, hi = (long long)(c.rank + 1) * a.L / N;
    const int tiles = (int)((hi - lo + kKeyTile - 1) / kKeyTile);
    const size_t tok_stride = (size_t)a.H * kHeadDim;   // elements between consecutive keys
    const bf16* kbase = a.kc + (size_t)b * a.cap * tok_stride + (size_t)head * kHeadDim;
    const bf16* vbase = a.vc + (size_t)b * a.cap * tok_stride + (size_t)head * kHeadDim;
    // tile t: 32 keys x 256 B for K and for V = 1024 16-byte chunks, 4 per thread
    auto issue = [&](int t) {
        const int st = t % kAttnStages;
        const uint32_t kdst = c.sa + kAttnStageOff + (uint32_t)st * 2u * kTileBytes;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int chunk = threadIdx.x + u * kAttnThreads;   // 0..511: key = chunk / 16, piece = chunk % 16
            const int key = chunk >> 4, piece = chunk & 15;
            const long long s = lo + (long long)t * kKeyTile + key;
            if (s < hi) {
                const size_t off = (size_t)s * tok_stride + (size_t)piece * 8;
                cp_async16(kdst + (uint32_t)chunk * 16u, kbase + off);
                cp_async16(kdst + kTileBytes + (uint32_t)chunk * 16u, vbase + off);
            }
        }
    };
#pragma unroll
    for (int t = 0; t < kAttnStages - 1; ++t) {
        if (t < tiles) issue(t);
        cp_async_commit();
    }
    f2x q2[8];   // this lane's 16 query dimensions, pre-scaled for exp2
    {
        const float* qp = a.q + ((size_t)b * a.H + head) * kHeadDim + 16 * sub;
#pragma unroll
        for (int e = 0; e < 8; ++e) q2[e] = f2_make(qp[2 * e] * a.scale_log2, qp[2 * e + 1] * a.scale_log2);
    }
    float m = -INFINITY, l = 0.f;
    f2x acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0ull;
    for (int t = 0; t < tiles; ++t) {
        if (t + kAttnStages - 1 < tiles) issue(t + kAttnStages - 1);
        cp_async_commit();
        cp_async_wait<kAttnStages - 1>();   // tile t landed (this thread's copies)
        __syncthreads();                      // ... and every thread's
        const unsigned char* kt = c.ptr<const unsigned char>(kAttnStageOff + (uint32_t)(t % kAttnStages) * 2u * kTileBytes);
        const unsigned char* vt = kt + kTileBytes;
        const long long s = lo + (long long)t * kKeyTile + grp;   // this group's key in the tile
        const bool valid = s < hi;
        const uint4* kr = reinterpret_cast<const uint4*>(kt + grp * 256 + sub * 32);
        const uint4* vr = reinterpret_cast<const uint4*>(vt + grp * 256 + sub * 32);
        f2x dot2 = 0ull;
        if (valid) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                f2x kf[4];
                RmsElem<bf16>::unpack(kr[u], kf);
#pragma unroll
                for (int e = 0; e < 4; ++e) dot2 = f2_fma(kf[e], q2[4 * u + e], dot2);
            }
        }
        const float2 d2 = f2_split(dot2);
        float logit = d2.x + d2.y;
        logit += __shfl_xor_sync(gmask, logit, 1);
        logit += __shfl_xor_sync(gmask, logit, 2);
        logit += __shfl_xor_sync(gmask, logit, 4);
        if (valid) {
            const float mn = fmaxf(m, logit);
            const float corr = exp2f(m - mn), p = exp2f(logit - mn);
            l = l * corr + p;
            m = mn;
            const f2x c2 = f2_make(corr, corr), p2 = f2_make(p, p);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                f2x vf[4];
                RmsElem<bf16>::unpack(vr[u], vf);
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[4 * u + e] = f2_fma(acc[4 * u + e], c2, f2_mul(p2, vf[e]));
            }
        }
        __syncthreads();   // the stage is free for the tile issued next iteration
    }
    cp_async_wait<0>();
    // the 32 groups of this CTA: (max, sum, acc) in shared memory, combined per dimension
    float* gst = c.ptr<float>(kAttnGroupOff);   // per group: m, l, acc[128]
    float* cta = c.ptr<float>(kAttnCtaOff);     // M, L, A[128] of this CTA
    if (sub == 0) {
        gst[grp * (2 + kHeadDim)] = m;
        gst[grp * (2 + kHeadDim) + 1] = l;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float2 v = f2_split(acc[e]);
        gst[grp * (2 + kHeadDim) + 2 + 16 * sub + 2 * e] = v.x;
        gst[grp * (2 + kHeadDim) + 2 + 16 * sub + 2 * e + 1] = v.y;
    }
    __syncthreads();
    if (threadIdx.x < kHeadDim) {
        const int d = threadIdx.x;
        float M = -INFINITY;
        for (int g2 = 0; g2 < kAttnGroups; ++g2) M = fmaxf(M, gst[g2 * (2 + kHeadDim)]);
        float Ls = 0.f, A = 0.f;
        if (M != -INFINITY)
            for (int g2 = 0; g2 < kAttnGroups; ++g2) {
                const float f = exp2f(gst[g2 * (2 + kHeadDim)] - M);   // 0 for a group without keys (-inf)
                Ls += gst[g2 * (2 + kHeadDim) + 1] * f;
                A += gst[g2 * (2 + kHeadDim) + 2 + d] * f;
            }
        cta[2 + d] = A;
        if (d == 0) {
            cta[0] = M;
            cta[1] = Ls;
        }
    }
    cluster_sync();   // every CTA's (M, L, A) visible
    const uint32_t cta_sa = c.sa + kAttnCtaOff;
    const int dpr = kHeadDim / N;   // dims finished by this CTA
    if (threadIdx.x < dpr) {
        const int d = (int)c.rank * dpr + threadIdx.x;
        float Mr[N], Mx = -INFINITY;
#pragma unroll
        for (int r = 0; r < N; ++r) {
            Mr[r] = ld_cluster_f32(mapa(cta_sa, (uint32_t)r));
            Mx = fmaxf(Mx, Mr[r]);
        }
        float den = 0.f, num = 0.f;
#pragma unroll
        for (int r = 0; r < N; ++r) {
            if (Mr[r] == -INFINITY) continue;
            const float f = exp2f(Mr[r] - Mx);
            den += ld_cluster_f32(mapa(cta_sa + 4u, (uint32_t)r)) * f;
            num += ld_cluster_f32(mapa(cta_sa + (uint32_t)(2 + d) * 4u, (uint32_t)r)) * f;
        }
        a.a_out[((size_t)b * a.H + head) * kHeadDim + d] = __float2bfloat16_rn(num / den);
    }
    dsb::finish(c);
}

std::mutex g_dec_mu;
unsigned* g_dec_err[64] = {};

template <int EPI, int N>
const void* proj_fn(int nt) {
    return nt == 1 ? reinterpret_cast<const void*>(&proj_kernel<EPI, N, 1>)
                   : reinterpret_cast<const void*>(&proj_kernel<EPI, N, 2>);
}
template <int EPI>
const void* proj_fn_n(int n, int nt) {
    return n == 4 ? proj_fn<EPI, 4>(nt) : proj_fn<EPI, 8>(nt);
}

cudaError_t launch_cluster(const void* fn, int n, long long clusters, uint32_t smem, cudaStream_t s, void* arg) {
    {
        std::lock_guard<std::mutex> lock(g_dec_mu);
        static std::map<std::pair<const void*, uint32_t>, bool> done;
        if (!done[{fn, smem}]) {
            cudaError_t r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (r != cudaSuccess) return r;
            done[{fn, smem}] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    cfg.blockDim = dim3(kProjThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {arg};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

dsmem_status proj(int epi, int n, ProjArgs& a, long long tiles, cudaStream_t s) {
    const int nt = a.B <= 8 ? 1 : 2;
    const int nkb = a.K / n / 32;
    a.smem_bytes = kArea + (uint32_t)nkb * 2u * nt * 32u * 8u + (uint32_t)kTile * 8u * nt * 4u;
    if (a.smem_bytes > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    const void* fn = epi == kEpiQKV ? proj_fn_n<kEpiQKV>(n, nt)
                   : epi == kEpiO ? proj_fn_n<kEpiO>(n, nt)
                   : epi == kEpiGateUp ? proj_fn_n<kEpiGateUp>(n, nt)
                                       : proj_fn_n<kEpiDown>(n, nt);
    return launch_cluster(fn, n, tiles, a.smem_bytes, s, &a) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

}  // namespace

extern "C" {

size_t dsmem_decoder_workspace_bytes(int batch, int hidden, int ffn) {
    const size_t bh = (size_t)std::max(batch, 0) * (size_t)std::max(hidden, 0);
    // x, xn, a, hn (bf16), q (fp32), act (bf16 [B][ffn]); each region 256-B aligned
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    return 4 * al(bh * 2) + al(bh * 4) + al((size_t)std::max(batch, 0) * (size_t)std::max(ffn, 0) * 2);
}

dsmem_status dsmem_decoder_layer_launch(const dsmem_decoder_params* p, dsmem_stream_t stream) {
    if (p == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    const int B = p->batch, hid = p->hidden, H = p->heads, ffn = p->ffn, n = p->cluster_size;
    if (B < 1 || B > 16 || p->head_dim != kHeadDim || H < 1 || hid != H * kHeadDim || ffn < 64) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (n != 4 && n != 8) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (hid % (32 * n) != 0 || ffn % (32 * n) != 0 || ffn % 64 != 0 || hid % kTile != 0) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (p->seq_len < 0 || p->seq_len >= p->cache_capacity) return DSMEM_ERR_INVALID_ARGUMENT;
    const void* ptrs[] = {p->inp, p->res, p->w_rms, p->wqkv, p->wo, p->w_post, p->wgu, p->wd,
                          p->kcache, p->vcache, p->cos, p->sin, p->workspace, p->out, p->h_out};
    for (const void* q : ptrs)
        if (q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u)) return DSMEM_ERR_INVALID_ARGUMENT;
    if (p->workspace_bytes < dsmem_decoder_workspace_bytes(B, hid, ffn)) return DSMEM_ERR_SCRATCH_LIMIT;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    unsigned* err = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_dec_mu);
        if (g_dec_err[dev] == nullptr) {
            if (cudaMalloc(&g_dec_err[dev], 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(g_dec_err[dev], 0, 4 * sizeof(unsigned));
        }
        err = g_dec_err[dev];
    }
    auto s = reinterpret_cast<cudaStream_t>(stream);
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t bh = (size_t)B * hid;
    unsigned char* ws = static_cast<unsigned char*>(p->workspace);
    bf16* x = reinterpret_cast<bf16*>(ws);
    bf16* xn = reinterpret_cast<bf16*>(ws + al(bh * 2));
    bf16* att = reinterpret_cast<bf16*>(ws + 2 * al(bh * 2));
    bf16* hn = reinterpret_cast<bf16*>(ws + 3 * al(bh * 2));
    float* q = reinterpret_cast<float*>(ws + 4 * al(bh * 2));
    bf16* act = reinterpret_cast<bf16*>(ws + 4 * al(bh * 2) + al(bh * 4));
    dsmem_status st;

    // 1. x = inp + res, xn = RMSNorm(x) w_rms
    st = dsmem_rmsnorm_residual_launch(DSMEM_BF16, p->inp, p->res, p->w_rms, p->eps, B, hid, 8, x, xn, stream);
    if (st != DSMEM_OK) return st;
    // 2. QKV + RoPE + cache append
    ProjArgs a{};
    a.W = static_cast<const bf16*>(p->wqkv);
    a.act = xn;
    a.K = hid;
    a.B = B;
    a.H = H;
    a.cap = p->cache_capacity;
    a.S = p->seq_len;
    a.q = q;
    a.kc = static_cast<bf16*>(p->kcache);
    a.vc = static_cast<bf16*>(p->vcache);
    a.knew = static_cast<bf16*>(p->k_new);
    a.vnew = static_cast<bf16*>(p->v_new);
    a.cosv = p->cos;
    a.sinv = p->sin;
    a.err = err;
    if ((st = proj(kEpiQKV, n, a, 3LL * hid / kTile, s)) != DSMEM_OK) return st;
    // 3. attention over the S cached tokens and the new one
    {
        AttnArgs t{};
        t.q = q;
        t.kc = static_cast<const bf16*>(p->kcache);
        t.vc = static_cast<const bf16*>(p->vcache);
        t.a_out = att;
        t.cap = p->cache_capacity;
        t.L = p->seq_len + 1;
        t.H = H;
        t.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)kHeadDim));
        t.smem_bytes = kAttnSmem;
        t.err = err;
        const void* fn = n == 4 ? reinterpret_cast<const void*>(&attn_kernel<4>)
                                : reinterpret_cast<const void*>(&attn_kernel<8>);
        if (launch_cluster(fn, n, (long long)B * H, t.smem_bytes, s, &t) != cudaSuccess) return DSMEM_ERR_CUDA;
    }
    // 4. o = a Wo^T, h = x + o
    a = ProjArgs{};
    a.W = static_cast<const bf16*>(p->wo);
    a.act = att;
    a.K = hid;
    a.B = B;
    a.x = x;
    a.o_out = static_cast<bf16*>(p->o_out);
    a.h_out = static_cast<bf16*>(p->h_out);
    a.out_ld = hid;
    a.err = err;
    if ((st = proj(kEpiO, n, a, hid / kTile, s)) != DSMEM_OK) return st;
    // 5. hn = RMSNorm(h) w_post
    st = dsmem_rmsnorm_launch(DSMEM_BF16, p->h_out, p->w_post, p->eps, B, hid, 8, hn, stream);
    if (st != DSMEM_OK) return st;
    // 6. act = SiLU(hn Wg^T) * (hn Wu^T)
    a = ProjArgs{};
    a.W = static_cast<const bf16*>(p->wgu);
    a.act = hn;
    a.K = hid;
    a.B = B;
    a.ffn = ffn;
    a.out = act;
    a.out_ld = ffn;
    a.err = err;
    if ((st = proj(kEpiGateUp, n, a, ffn / 64, s)) != DSMEM_OK) return st;
    // 7. out = act Wd^T
    a = ProjArgs{};
    a.W = static_cast<const bf16*>(p->wd);
    a.act = act;
    a.K = ffn;
    a.B = B;
    a.out = static_cast<bf16*>(p->out);
    a.out_ld = hid;
    a.err = err;
    return proj(kEpiDown, n, a, hid / kTile, s);
}

dsmem_status dsmem_decoder_check(int device, unsigned* error_bits) {
    unsigned v = 0;
    {
        std::lock_guard<std::mutex> lock(g_dec_mu);
        if (device < 0 || device >= 64) return DSMEM_ERR_INVALID_ARGUMENT;
        if (g_dec_err[device] != nullptr) {
            if (cudaMemcpy(&v, g_dec_err[device], sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return DSMEM_ERR_CUDA;
            cudaMemset(g_dec_err[device], 0, 4 * sizeof(unsigned));
        }
    }
    if (error_bits) *error_bits = v;
    return DSMEM_OK;
}

}  // extern "C"
