// ext_decoder.cu -- Llama-2-7B-shaped decoder layer, one decode step, cluster-fused, sm_100a.
//
// Reference: kernels/fused_decoder_layer__llama2_7b__clusterfusion.cu:101-268, 291-922 (attention block,
// cluster_reduce between stages) and the layer maths of
// roofline/harness/workloads/clusterfusion_llama2_7b_decoder.py:160-180 (reference_fp32, with the FFN tail):
//   x = inp + res; xn = RMSNorm(x) w_rms; qkv = xn Wqkv^T; q, k = NEOX RoPE(q, k); append k, v to the cache;
//   a = softmax(q K^T / sqrt(D)) V over the cache and the new token; o = a Wo^T; h = x + o;
//   hn = RMSNorm(h) w_post; out = (SiLU(hn Wg^T) * hn Wu^T) Wd^T.
// B200 design: five stream-ordered launches, every stage HBM-bound (weights read once per step, the KV
// cache once per sequence):
//   1-2. QKV projection on the tcgen05 tensor cores, with the RMSNorm of x = inp + res fused into its
//      prologue (each CTA normalises its K-slice of the batch rows: partial sums of squares meet over
//      the cluster in DSMEM; cluster 0 writes x for the residual): persistent clusters, each with up to 8 tiles of 128
//      output features; the cluster's N CTAs split K. Per CTA a TMA producer streams 128-row weight chunks
//      (128-byte swizzle) through a 64 KiB ring, one thread issues tcgen05.mma kind::f16 (M = 128 weight
//      rows, N = 16 batch rows, K = 16; fp32 accumulators in TMEM, 16 columns per tile), and four warps
//      read the accumulators back (tcgen05.ld) into partial tiles; the N partial tiles meet by DSMEM loads
//      (reduce-scatter by feature pairs (i, i+64)), whose owner applies RoPE and writes q (fp32) and the
//      new k, v into the cache;
//   3. decode attention: one cluster per (sequence, head), the cluster's CTAs split the keys; a producer
//      warp streams them as 64-token K and V tiles of the head (one TMA load each) through a 3-stage ring
//      with full/empty mbarriers; groups of 8 lanes take two keys of a tile (16 dims a lane), online
//      softmax in base 2; then the partial (max, sum, acc) of the 32 groups meet in shared memory and the
//      N CTAs' in DSMEM;
//   4. O projection (as 2) with the epilogue h = x + o;
//   5-6. gate/up projection (as 2, with the RMSNorm of h fused into its prologue; a tile holds gate rows
//      j and up rows j of the same 64 j) with the epilogue SiLU(gate) * up;
//   7. down projection (as 2).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "f32x2.cuh"
#include "smem_attr.cuh"
#include "tmap.cuh"

namespace {

using namespace dsmem;
using namespace dsb2;
using bf16 = __nv_bfloat16;

constexpr int kHeadDim = 128;
constexpr int kTile = 128;           // output features per cluster tile
constexpr int kAttnThreads = 256;    // 32 groups of 8 lanes
constexpr uint32_t kArea = 128;      // barrier area / finish flag at the start of the dynamic window

enum Epi : int { kEpiQKV = 0, kEpiO = 1, kEpiGateUp = 2, kEpiDown = 3 };

struct ProjArgs {
    // tcgen05 path: the weight tile as {K, rows, 2 halves} (box {32, 64, 2}: one 32-wide K chunk of the
    // tile's two 64-row halves) and the activations as {K, B} (box {32, 16}: rows past B read as zero),
    // both with the 64-byte swizzle of the UMMA K-major operand layout
    alignas(64) CUtensorMap tmw;
    alignas(64) CUtensorMap tma;
    int w_row0_step;      // first weight row of tile t = t * w_row0_step (the second half follows by map)
    int tiles;            // 128-feature tiles of the projection
    int chunk;            // K chunk width: 64 (128-byte swizzle) or 32 (64-byte swizzle) elements
    // Fused RMSNorm prologue (nrm_x != nullptr): the activations are RMSNorm(h) * nrm_w with
    // h = nrm_x (+ nrm_res) rounded to bf16, over the K = hidden features of each row; cluster 0 also
    // writes h to nrm_h when given. act / tma are then unused.
    const bf16* nrm_x;
    const bf16* nrm_res;
    const bf16* nrm_w;
    bf16* nrm_h;
    float nrm_eps;
    uint32_t tmem_cols;   // TMEM columns each CTA allocates (a power of two >= 32, 16 per tile)
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

// Epilogue of one feature pair (i, i + 64) of tile `tile` for batch row n: lo, hi are the cluster sums.
template <int EPI>
__device__ __forceinline__ void proj_epilogue(const ProjArgs& a, int tile, int i, int n, float lo, float hi) {
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

// --------------------------------------------------------------------------------------------------
// tcgen05 projection: persistent clusters; cluster q takes the 128-feature tiles q, q + C, q + 2C, ..
// (at most kTcMaxTiles), CTA `rank` reduces its share of K (whole chunks, split as evenly as they allow)
// for every one of them on the 5th-generation tensor cores. Per CTA, 4 warps:
//   warp 0 lane 0  loads the activation K-slice once (one TMA load per K chunk, 16 rows: rows past B read
//                  as zero), then streams the weight rows of all its tiles, K chunks of 128 rows (one TMA
//                  load per chunk), through a 64 KiB ring without a break between tiles;
//   warp 1         allocates TMEM (16 fp32 columns per tile); its lane 0 issues, per chunk, tcgen05.mma
//                  kind::f16 (M = 128 weight rows, N = 16 activation rows, K = 16 per instruction; bf16 in,
//                  fp32 accumulate into the tile's TMEM columns) and frees the stage with tcgen05.commit;
//   warps 0-3      after the last MMA, read every tile's 128 x 16 accumulator back (tcgen05.ld 32x32b, one
//                  TMEM lane quarter per warp) into partial tiles in the (now idle) ring; then one cluster
//                  barrier, then per tile the reduce-scatter by feature pairs (i, i + 64) over the cluster
//                  (DSMEM loads, rank order) and the projection's epilogue (proj_epilogue).
// Operands are K-major with the swizzle that matches the chunk's row length: 64-element chunks (128-byte
// rows, 128-byte swizzle, 1024-byte 8-row atoms) when they divide K, else 32-element chunks (64-byte
// rows and swizzle); TMA writes exactly these layouts, and K step k of a chunk starts 32 * k bytes in.
// Measured on B200 (Llama-2-7B layer, batch 1, ncu): a 64 KiB ring beat 96 KiB, and 128-byte rows beat
// 64-byte rows by about 10 % (fewer, longer DRAM bursts per weight row).
constexpr int kTcThreads = 128;
constexpr int kTcMaxStages = 12;                          // barrier ids reserved for ring stages
constexpr uint32_t kTcRing = 64u * 1024u;                 // weight ring bytes (measured best: 96 KiB was slower)
constexpr int kTcMaxTiles = 8;                            // partial tiles (8 KiB each) reuse the ring
constexpr uint32_t kTcPart = 128u * 16u * 4u;
constexpr uint32_t kTcArea = 1024;  // barriers: full 0..11, act 12, done 13, TMEM word 14, empty 16..27,
                                    // partial sums 28; bytes [256, 768): the fused RMSNorm's partial sums of
                                    // squares [N][16], [768, 832): its row scales
constexpr int kTcFull = 0, kTcAct = 12, kTcDone = 13, kTcEmpty = 16;
constexpr uint32_t kTcTmemWord = 112;
constexpr uint32_t kTcSsq = 256, kTcScl = 768;
constexpr int kTcSsqBar = 28;
static_assert(8 * (kTcDone + 2) <= (int)dsb::kFlagOff && 8 * kTcEmpty > (int)dsb::kFlagOff &&
                  8 * (kTcEmpty + kTcMaxStages) <= (int)kTcArea && kTcMaxTiles <= 8,
              "barrier ids overlap the flag word");
static_assert(kTcMaxTiles * kTcPart <= kTcRing, "the partial tiles fit in the ring");
static_assert(kTcRing / (128u * 32u * 2u) <= (uint32_t)kTcMaxStages, "ring stages have barrier ids");
// K chunk of `cw` (64 or 32) elements: 128 weight rows of cw * 2 bytes, 16 activation rows of cw * 2 bytes.
__host__ __device__ constexpr uint32_t tc_chunk_w(int cw) { return 128u * (uint32_t)cw * 2u; }
__host__ __device__ constexpr uint32_t tc_chunk_a(int cw) { return 16u * (uint32_t)cw * 2u; }
__host__ __device__ constexpr uint32_t tc_smem(int chunks, int cw) {
    return kTcArea + 1024u + (uint32_t)chunks * tc_chunk_a(cw) + kTcRing;
}

// UMMA shared-memory descriptor of a K-major operand whose rows are `row_bytes` (128 or 64) long with the
// matching swizzle: 8-row atoms 8 * row_bytes apart.
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t saddr, uint32_t row_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu)                // start address (16-byte units)
           | ((uint64_t)1u << 16)                            // leading byte offset (unused by swizzled K-major)
           | ((uint64_t)((8u * row_bytes) >> 4) << 32)       // stride byte offset between 8-row atoms
           | ((uint64_t)1u << 46)                            // descriptor version of sm_100
           | ((uint64_t)(row_bytes == 128u ? 2u : 4u) << 61);   // layout: 128- or 64-byte swizzle
}
// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, N = 16, M = 128.
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kTcIdesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Bounded wait by one thread for barrier i to finish the phase of parity `par`.
__device__ __forceinline__ void tc_wait(dsb::Ctx& c, int i, uint32_t par) {
    if (c.dead) return;
    if (mbar_try_wait_parity(c.bar(i), par)) return;
    if (!mbar_wait_parity_until(c.bar(i), par, c.deadline)) {
        c.dead = true;
        dsb::report_timeout(c, i);
    }
}

template <int EPI, int N>
__global__ void __launch_bounds__(kTcThreads) proj_tc_kernel(const __grid_constant__ ProjArgs a) {
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, 1000000000ull);
    dsb::flag_init(c);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = (int)cluster_id(), C = (int)num_clusters();
    const int nt = a.tiles > q ? min(kTcMaxTiles, (a.tiles - q + C - 1) / C) : 0;   // this cluster's tiles
    // this CTA's K chunks: the K / cw chunks split as evenly as whole chunks allow
    const int cw = a.chunk, tch = a.K / cw;
    const int ch0 = (int)c.rank * tch / N, nch = ((int)c.rank + 1) * tch / N - ch0;
    const uint32_t cwb = tc_chunk_w(cw), cab = tc_chunk_a(cw), rowb = (uint32_t)cw * 2u;
    const uint32_t act0 = ((c.sa + kTcArea + 1023u) & ~1023u) - c.sa;   // 1024-aligned (swizzle atoms)
    const uint32_t ring0 = act0 + (uint32_t)((tch + N - 1) / N) * cab;  // 1024-aligned as well
    const int nst = (int)(kTcRing / cwb);
    constexpr int NB = 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(c.bar(kTcFull + s), 1);
            mbar_init(c.bar(kTcEmpty + s), 1);
        }
        mbar_init(c.bar(kTcAct), 1);
        mbar_init(c.bar(kTcDone), 1);
        mbar_init(c.bar(kTcSsqBar), 1);
        if (a.nrm_x != nullptr) dsb::arm(c, kTcSsqBar, (uint32_t)N * (uint32_t)a.B * 4u);   // every peer's partials
        fence_mbar_init();
        prefetch_tmap(&a.tmw);
        if (a.nrm_x == nullptr) prefetch_tmap(&a.tma);
    }
    if (warp == 1) {   // TMEM: 16 fp32 columns per tile
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(c.sa + kTcTmemWord),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *c.ptr<volatile uint32_t>(kTcTmemWord);
    c.deadline = globaltimer() + c.wait_limit;

    const bool fused = a.nrm_x != nullptr;
    const int total = nt * nch;   // weight chunks of this CTA over all its tiles: chunk g = tile g / nch
    // Issue weight chunk g into its stage (after the stage's previous chunk was consumed). Producer lane.
    auto issue = [&](int g) {
        const int s = g % nst, j = g / nch, i = g % nch;
        if (g >= nst) {
            c.deadline = globaltimer() + c.wait_limit;
            tc_wait(c, kTcEmpty + s, (uint32_t)((g / nst - 1) & 1));
        }
        if (c.dead) return;
        dsb::arm(c, kTcFull + s, cwb);
        tma_load_3d(c.sa + ring0 + (uint32_t)s * cwb, &a.tmw, (ch0 + i) * cw, (q + j * C) * a.w_row0_step, 0,
                    c.bar(kTcFull + s));
    };
    int g_issued = 0;
    if (fused) {
        // ------------------------------------------------------------------ fused RMSNorm prologue
        // Every thread arrives at the cluster barrier before any bulk load is issued (an arrive issued after
        // them waits for their bytes), then the first ring's worth of weight chunks goes out, so the loads
        // overlap the prologue; the partial sums travel by st.async onto each peer's barrier.
        cluster_arrive();
        if (warp == 0 && lane == 0)
            for (; g_issued < min(nst, total); ++g_issued) issue(g_issued);
        const int k0 = ch0 * cw, kl = nch * cw, units = kl / 8;   // this CTA's K range, 8-element units
        // h of unit u of row r: 8 bf16 values, x (+ res) rounded to bf16
        auto load_h = [&](int r, int u, f2x* f) {
            const size_t off = (size_t)r * a.K + k0 + 8 * u;
            RmsElem<bf16>::unpack(*reinterpret_cast<const uint4*>(a.nrm_x + off), f);
            if (a.nrm_res != nullptr) {
                f2x rr[4];
                RmsElem<bf16>::unpack(*reinterpret_cast<const uint4*>(a.nrm_res + off), rr);
#pragma unroll
                for (int e = 0; e < 4; ++e) f[e] = f2_add(f[e], rr[e]);
                RmsElem<bf16>::unpack(RmsElem<bf16>::pack(f), f);
            }
        };
        // pass 1: h of every (row, unit) into its swizzled place in the operand (rows past B zero), and
        // each row's partial sum of squares over this CTA's K range
        const uint32_t sw_mask = cw == 64 ? 7u : 3u;
        auto slot = [&](int r, int u) {   // shared-memory offset of unit u of row r in the operand
            const int i = u / (cw / 8), uc = u % (cw / 8);
            const uint32_t swz = (uint32_t)uc ^ (cw == 64 ? ((uint32_t)r & sw_mask) : (((uint32_t)r >> 1) & sw_mask));
            return act0 + (uint32_t)i * cab + (uint32_t)r * rowb + 16u * swz;
        };
        // the weight units of pass 2 (units tid and tid + 128), loaded now so their latency overlaps pass 1
        uint4 wreg[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            const int u = threadIdx.x + h2 * kTcThreads;
            wreg[h2] = u < units ? *reinterpret_cast<const uint4*>(a.nrm_w + k0 + 8 * u) : make_uint4(0u, 0u, 0u, 0u);
        }
        float part_ss[4];   // this warp's rows w, w + 4, w + 8, w + 12
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int r = warp + 4 * rr;
            f2x acc = 0ull;
#pragma unroll 2
            for (int u = lane; u < units; u += 32) {
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (r < a.B) {
                    f2x f[4];
                    load_h(r, u, f);
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc = f2_fma(f[e], f[e], acc);
                    v = RmsElem<bf16>::pack(f);
                    if (q == 0 && a.nrm_h != nullptr) *reinterpret_cast<uint4*>(a.nrm_h + (size_t)r * a.K + k0 + 8 * u) = v;
                }
                *c.ptr<uint4>(slot(r, u)) = v;
            }
            const float2 a2 = f2_split(acc);
            float v = a2.x + a2.y;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            part_ss[rr] = v;
        }
        cluster_wait();   // every peer's barriers initialised (and its arrive released them)
        // lane p < N sends this warp's row partials into slot [rank][r] of CTA p
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int r = warp + 4 * rr;
            if (r < a.B && lane < N) {
                const uint32_t dst = mapa(c.sa + kTcSsq + 4u * ((uint32_t)c.rank * 16u + (uint32_t)r), (uint32_t)lane);
                asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst),
                             "r"(__float_as_uint(part_ss[rr])), "r"(mapa(c.bar(kTcSsqBar), (uint32_t)lane))
                             : "memory");
            }
        }
        c.deadline = globaltimer() + c.wait_limit;
        tc_wait(c, kTcSsqBar, 0u);   // every peer's partials of every row
        float* scl = c.ptr<float>(kTcScl);
        if (threadIdx.x < a.B) {
            const float* ssq = c.ptr<const float>(kTcSsq);
            float t = 0.f;
            for (int p2 = 0; p2 < N; ++p2) t += ssq[p2 * 16 + threadIdx.x];   // rank order
            scl[threadIdx.x] = rsqrtf(fmaf(t, 1.0f / (float)a.K, a.nrm_eps));
        }
        __syncthreads();
        // pass 2: y = (h * scale) * w in place, w of a unit shared by the rows
        for (int u = threadIdx.x, h2 = 0; u < units; u += kTcThreads, ++h2) {
            f2x w[4];
            RmsElem<bf16>::unpack(h2 < 2 ? wreg[h2 & 1] : *reinterpret_cast<const uint4*>(a.nrm_w + k0 + 8 * u), w);
            for (int r = 0; r < a.B; ++r) {
                uint4* pv = c.ptr<uint4>(slot(r, u));
                f2x f[4];
                RmsElem<bf16>::unpack(*pv, f);
                const f2x scale2 = f2_make(scl[r], scl[r]);
#pragma unroll
                for (int e = 0; e < 4; ++e) f[e] = f2_mul(f2_mul(f[e], scale2), w[e]);
                *pv = RmsElem<bf16>::pack(f);
            }
        }
        fence_proxy_async_smem();   // the operand is read by tcgen05.mma (async proxy)
        __syncthreads();
    }

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (!fused) {
            dsb::arm(c, kTcAct, (uint32_t)nch * cab);
            for (int i = 0; i < nch; ++i)
                tma_load_2d(c.sa + act0 + (uint32_t)i * cab, &a.tma, (ch0 + i) * cw, 0, c.bar(kTcAct));
        }
        for (int g = g_issued; g < total && !c.dead; ++g) issue(g);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------------ MMA issuer
        if (!fused) tc_wait(c, kTcAct, 0u);
        int g = 0;
        for (int j = 0; j < nt && !c.dead; ++j) {
            const uint32_t d = tmem + 16u * (uint32_t)j;   // the tile's accumulator columns
            for (int i = 0; i < nch; ++i, ++g) {
                const int s = g % nst;
                c.deadline = globaltimer() + c.wait_limit;
                tc_wait(c, kTcFull + s, (uint32_t)((g / nst) & 1));
                if (c.dead) break;
                tc_fence_after();
                const uint32_t wa = c.sa + ring0 + (uint32_t)s * cwb, aa = c.sa + act0 + (uint32_t)i * cab;
                for (int k = 0; k < cw / 16; ++k)   // K steps of 16 elements = 32 bytes into the swizzled rows
                    umma_bf16(d, umma_desc_kmajor(wa + 32u * k, rowb), umma_desc_kmajor(aa + 32u * k, rowb),
                              (i | k) != 0 ? 1u : 0u);
                umma_commit(c.bar(kTcEmpty + s));   // the stage is free once these MMAs have read it
            }
        }
        umma_commit(c.bar(kTcDone));   // every MMA of this thread complete -> accumulators final
    }
    __syncwarp();

    // ---------------------------------------------------------------------- accumulators -> partial tiles
    c.deadline = globaltimer() + c.wait_limit;
    tc_wait(c, kTcDone, 0u);
    tc_fence_after();
    const int row = 32 * warp + lane;   // TMEM lane = weight row of the tile = output feature
    for (int j = 0; j < nt; ++j) {
        uint32_t r[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(tmem + ((uint32_t)(32 * warp) << 16) + 16u * (uint32_t)j));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float* part = c.ptr<float>(ring0 + (uint32_t)j * kTcPart);
#pragma unroll
        // a CTA without K chunks (K < N chunks) issued no MMA: its partial sums are zero
        for (int e = 0; e < 16; ++e) part[row * NB + e] = (c.dead || nch == 0) ? 0.f : __uint_as_float(r[e]);
    }
    tc_fence_before();
    cluster_sync();   // every CTA's partial tiles complete and visible; every TMEM read done
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");

    // ---------------------------------------------------------------------- reduce-scatter + epilogue
    const int npairs = 64 / N;
    for (int j = 0; j < nt; ++j) {
        const uint32_t part_sa = c.sa + ring0 + (uint32_t)j * kTcPart;
        for (int e = threadIdx.x; e < npairs * a.B; e += blockDim.x) {
            const int i = (int)c.rank * npairs + e / a.B, n = e % a.B;
            float lo = 0.f, hi = 0.f;
#pragma unroll
            for (int r = 0; r < N; ++r) {
                lo += ld_cluster_f32(mapa(part_sa + (uint32_t)(i * NB + n) * 4u, (uint32_t)r));
                hi += ld_cluster_f32(mapa(part_sa + (uint32_t)((i + 64) * NB + n) * 4u, (uint32_t)r));
            }
            proj_epilogue<EPI>(a, q + j * C, i, n, lo, hi);
        }
    }
    dsb::finish(c);   // peers have finished reading my partial tiles
}

struct AttnArgs {
    // the K and V caches as {D, H, cap, B} (box {D, 1, kKeyTile, 1}: one head of kKeyTile consecutive tokens)
    alignas(64) CUtensorMap tmk;
    alignas(64) CUtensorMap tmv;
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

constexpr int kKeyTile = 64;                       // keys per shared-memory tile (two per group)
constexpr int kAttnStages = 3;                     // tiles in flight
constexpr uint32_t kTileBytes = kKeyTile * kHeadDim * 2u;   // one K (or V) tile, 16 KiB
constexpr int kAttnGroups = kAttnThreads / 8;      // 32 groups of 8 lanes, two keys each per tile
constexpr int kAttnCompute = kAttnThreads / 32;    // compute warps; one more warp loads the tiles
// shared memory: [kArea) barriers (full 0..2, empty 3..5) + flag | stages x (K tile, V tile) | group
// partials (m, l, acc[128]) | CTA partial
constexpr uint32_t kAttnStageOff = kArea;
constexpr uint32_t kAttnGroupOff = kAttnStageOff + kAttnStages * 2u * kTileBytes;
constexpr uint32_t kAttnCtaOff = kAttnGroupOff + (uint32_t)kAttnGroups * (2 + kHeadDim) * 4u;
constexpr uint32_t kAttnSmem = kAttnCtaOff + (2 + kHeadDim) * 4u;
constexpr int kAttnFull = 0, kAttnEmpty = kAttnStages;
static_assert(8 * 2 * kAttnStages <= (int)dsb::kFlagOff, "barrier ids overlap the flag word");

// One cluster = one (sequence, head); CTA r of N takes keys [r*L/N, (r+1)*L/N). A producer warp streams the
// CTA's keys as tiles of 64 tokens of this head, one TMA load for K and one for V per tile (tokens past the
// cache read as zero), through kAttnStages shared-memory stages with full/empty mbarriers; 32 groups of 8
// lanes take two keys of a tile each, a lane owning 16 of the 128 dimensions; online softmax in base 2.
// Then the 32 groups' (max, sum, acc) meet in shared memory and the N CTAs' in DSMEM.
template <int N>
__global__ void __launch_bounds__(kAttnThreads + 32) attn_kernel(const __grid_constant__ AttnArgs a) {
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, 1000000000ull);
    dsb::flag_init(c);
    const int cid = (int)cluster_id(), b = cid / a.H, head = cid % a.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane & 7, grp = threadIdx.x >> 3;
    const unsigned gmask = 0xFFu << (lane & 24);   // the 8 lanes of this group
    const long long lo = (long long)c.rank * a.L / N, hi = (long long)(c.rank + 1) * a.L / N;
    const int tiles = (int)((hi - lo + kKeyTile - 1) / kKeyTile);
    if (threadIdx.x == 0) {
        for (int st = 0; st < kAttnStages; ++st) {
            mbar_init(c.bar(kAttnFull + st), 1);
            mbar_init(c.bar(kAttnEmpty + st), kAttnCompute);
        }
        fence_mbar_init();
    }
    __syncthreads();
    c.deadline = globaltimer() + c.wait_limit;
    float m = -INFINITY, l = 0.f;
    f2x acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0ull;
    if (warp == kAttnCompute) {
        // ------------------------------------------------------------------ producer warp (lane 0)
        if (lane == 0) {
            prefetch_tmap(&a.tmk);
            prefetch_tmap(&a.tmv);
            for (int t = 0; t < tiles; ++t) {
                const int st = t % kAttnStages;
                if (t >= kAttnStages) {
                    c.deadline = globaltimer() + c.wait_limit;
                    tc_wait(c, kAttnEmpty + st, (uint32_t)((t / kAttnStages - 1) & 1));
                }
                if (c.dead) break;
                const uint32_t dst = c.sa + kAttnStageOff + (uint32_t)st * 2u * kTileBytes;
                const int tok = (int)(lo + (long long)t * kKeyTile);
                dsb::arm(c, kAttnFull + st, 2u * kTileBytes);
                tma_load_4d(dst, &a.tmk, 0, head, tok, b, c.bar(kAttnFull + st));
                tma_load_4d(dst + kTileBytes, &a.tmv, 0, head, tok, b, c.bar(kAttnFull + st));
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ compute warps
        f2x q2[8];   // this lane's 16 query dimensions, pre-scaled for exp2
        {
            const float* qp = a.q + ((size_t)b * a.H + head) * kHeadDim + 16 * sub;
#pragma unroll
            for (int e = 0; e < 8; ++e) q2[e] = f2_make(qp[2 * e] * a.scale_log2, qp[2 * e + 1] * a.scale_log2);
        }
        for (int t = 0; t < tiles; ++t) {
            const int st = t % kAttnStages;
            c.deadline = globaltimer() + c.wait_limit;
            tc_wait(c, kAttnFull + st, (uint32_t)((t / kAttnStages) & 1));
            const unsigned char* kt = c.ptr<const unsigned char>(kAttnStageOff + (uint32_t)st * 2u * kTileBytes);
            const unsigned char* vt = kt + kTileBytes;
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                const int key = grp + h2 * kAttnGroups;   // this group's keys in the tile
                const long long s = lo + (long long)t * kKeyTile + key;
                const bool valid = s < hi;
                const uint4* kr = reinterpret_cast<const uint4*>(kt + key * 256 + sub * 32);
                const uint4* vr = reinterpret_cast<const uint4*>(vt + key * 256 + sub * 32);
                f2x dot2 = 0ull;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    f2x kf[4];
                    RmsElem<bf16>::unpack(kr[u], kf);
#pragma unroll
                    for (int e = 0; e < 4; ++e) dot2 = f2_fma(kf[e], q2[4 * u + e], dot2);
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
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(c.bar(kAttnEmpty + st));   // this warp is done with the stage
        }
    }
    __syncthreads();
    // the 32 groups of this CTA: (max, sum, acc) in shared memory, combined per dimension
    float* gst = c.ptr<float>(kAttnGroupOff);   // per group: m, l, acc[128]
    float* cta = c.ptr<float>(kAttnCtaOff);     // M, L, A[128] of this CTA
    if (warp < kAttnCompute) {
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

cudaError_t launch_cluster(const void* fn, int n, long long clusters, uint32_t smem, cudaStream_t s, void* arg,
                           int threads) {
    int dev = 0;
    cudaError_t r = cudaGetDevice(&dev);
    if (r != cudaSuccess || (r = dsb_attr::ensure_smem(fn, dev, smem)) != cudaSuccess) return r;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {arg};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Same block shape as the tcgen05 projection kernels and no TMEM: the occupancy query runs on it, because
// the query counts one CTA per SM for kernels that allocate TMEM (it cannot see how many columns they take),
// while two of these CTAs (at most 2 x 128 of the SM's 512 columns) share an SM.
__global__ void __launch_bounds__(kTcThreads) tc_occupancy_probe() {}

// Co-resident clusters of a tcgen05 projection kernel of `smem` bytes (cached per cluster size, device and
// shared memory).
cudaError_t tc_resident(const void* /*fn*/, int n, uint32_t smem, int* out) {
    const void* fn = reinterpret_cast<const void*>(&tc_occupancy_probe);
    int dev = 0;
    cudaError_t r = cudaGetDevice(&dev);
    if (r != cudaSuccess) return r;
    std::lock_guard<std::mutex> lock(g_dec_mu);
    static std::map<std::tuple<int, int, uint32_t>, int> cache;
    auto key = std::make_tuple(n, dev, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return (*out = it->second), cudaSuccess;
    if ((r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess) return r;
    // the largest shared-memory carveout, so that two CTAs share an SM (the default carveout fits one)
    if ((r = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared)) !=
        cudaSuccess)
        return r;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)n, 1, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int res = 0;
    if ((r = cudaOccupancyMaxActiveClusters(&res, fn, &cfg)) != cudaSuccess) return r;
    cache[key] = res;
    *out = res;
    return cudaSuccess;
}

template <int EPI>
const void* proj_tc_fn(int n) {
    return n == 4 ? reinterpret_cast<const void*>(&proj_tc_kernel<EPI, 4>)
                  : reinterpret_cast<const void*>(&proj_tc_kernel<EPI, 8>);
}

// Projection of a.act [B][K] by the weight rows of `tiles` 128-feature tiles on the tcgen05 kernel.
// w_rows: rows of a.W; the tile's second 64 rows follow its first 64 by `half_rows` rows (64, or ffn for
// the gate/up tiles, whose first half is gate rows and second half up rows), and tile t starts at row
// t * row_step.
dsmem_status proj(int epi, int n, ProjArgs& a, long long tiles, cudaStream_t s, long long w_rows, long long half_rows,
                  int row_step) {
    const cuuint64_t K = (cuuint64_t)a.K;
    // K chunks of 64 elements (128-byte rows, 128-byte swizzle) when they divide K, else 32 (64-byte)
    const int cw = a.K % 64 == 0 ? 64 : 32;
    const CUtensorMapSwizzle sw = cw == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    {   // weights: {K, rows reachable from a tile's first half, 2 halves}, box {cw, 64, 2}
        const cuuint64_t dims[3] = {K, (cuuint64_t)(w_rows - half_rows), 2};
        const cuuint64_t strides[2] = {K * 2, (cuuint64_t)half_rows * K * 2};
        const cuuint32_t box[3] = {(cuuint32_t)cw, 64, 2};
        if (!dsb_tmap::encode(&a.tmw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.W, dims, strides, box, sw))
            return DSMEM_ERR_CUDA;
    }
    if (a.nrm_x == nullptr) {   // activations: {K, B}, box {cw, 16} (else the kernel computes them)
        const cuuint64_t dims[2] = {K, (cuuint64_t)a.B};
        const cuuint64_t strides[1] = {K * 2};
        const cuuint32_t box[2] = {(cuuint32_t)cw, 16};
        if (!dsb_tmap::encode(&a.tma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.act, dims, strides, box, sw))
            return DSMEM_ERR_CUDA;
    }
    a.chunk = cw;
    a.w_row0_step = row_step;
    a.tiles = (int)tiles;
    a.smem_bytes = tc_smem((a.K / cw + n - 1) / n, cw);
    if (a.smem_bytes > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    const void* fn = epi == kEpiQKV ? proj_tc_fn<kEpiQKV>(n)
                   : epi == kEpiO ? proj_tc_fn<kEpiO>(n)
                   : epi == kEpiGateUp ? proj_tc_fn<kEpiGateUp>(n)
                                       : proj_tc_fn<kEpiDown>(n);
    // persistent clusters: as many as are co-resident, each with at most kTcMaxTiles tiles
    int resident = 0;
    if (tc_resident(fn, n, a.smem_bytes, &resident) != cudaSuccess || resident < 1) return DSMEM_ERR_CUDA;
    const long long clusters = std::max<long long>(std::min<long long>(tiles, resident),
                                                   (tiles + kTcMaxTiles - 1) / kTcMaxTiles);
    const long long per = (tiles + clusters - 1) / clusters;
    uint32_t cols = 32;
    while (cols < 16u * (uint32_t)per) cols *= 2;
    a.tmem_cols = cols;
    return launch_cluster(fn, n, clusters, a.smem_bytes, s, &a, kTcThreads) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

}  // namespace

extern "C" {

size_t dsmem_decoder_workspace_bytes(int batch, int hidden, int ffn) {
    const size_t bh = (size_t)std::max(batch, 0) * (size_t)std::max(hidden, 0);
    // x, (spare), a, (spare) (bf16 [B][hidden]), q (fp32), act (bf16 [B][ffn]); each region 256-B aligned
    // (the two spare regions held the normalised rows before the RMSNorms moved into the projections)
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
    bf16* att = reinterpret_cast<bf16*>(ws + 2 * al(bh * 2));
    float* q = reinterpret_cast<float*>(ws + 4 * al(bh * 2));
    bf16* act = reinterpret_cast<bf16*>(ws + 4 * al(bh * 2) + al(bh * 4));
    dsmem_status st;

    // 1-2. x = inp + res, xn = RMSNorm(x) w_rms (fused prologue; cluster 0 writes x), QKV + RoPE + cache append
    ProjArgs a{};
    a.W = static_cast<const bf16*>(p->wqkv);
    a.nrm_x = static_cast<const bf16*>(p->inp);
    a.nrm_res = static_cast<const bf16*>(p->res);
    a.nrm_w = static_cast<const bf16*>(p->w_rms);
    a.nrm_h = x;
    a.nrm_eps = p->eps;
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
    if ((st = proj(kEpiQKV, n, a, 3LL * hid / kTile, s, 3LL * hid, 64, kTile)) != DSMEM_OK) return st;
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
        {   // caches {D, H, cap, B}, box {D, 1, kKeyTile, 1}
            const cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)H, (cuuint64_t)p->cache_capacity, (cuuint64_t)B};
            const cuuint64_t strides[3] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)H * kHeadDim * 2,
                                           (cuuint64_t)p->cache_capacity * H * kHeadDim * 2};
            const cuuint32_t box[4] = {(cuuint32_t)kHeadDim, 1, (cuuint32_t)kKeyTile, 1};
            if (!dsb_tmap::encode(&t.tmk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, p->kcache, dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
                !dsb_tmap::encode(&t.tmv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, p->vcache, dims, strides, box,
                                  CU_TENSOR_MAP_SWIZZLE_NONE))
                return DSMEM_ERR_CUDA;
        }
        t.err = err;
        // The attention's cluster size follows the number of (sequence, head) pairs, not the projections':
        // few pairs need the keys of each split 8 ways to fill the GPU, many pairs stream longer key ranges
        // per CTA with less merging (measured, Llama-2-7B at S = 4096: batch 1 -> 8, 4 and 16 -> 2).
        const int pairs = B * H;
        const int na = pairs <= 48 ? 8 : pairs <= 96 ? 4 : 2;
        const void* fn = na == 2 ? reinterpret_cast<const void*>(&attn_kernel<2>)
                       : na == 4 ? reinterpret_cast<const void*>(&attn_kernel<4>)
                                 : reinterpret_cast<const void*>(&attn_kernel<8>);
        if (launch_cluster(fn, na, (long long)B * H, t.smem_bytes, s, &t, kAttnThreads + 32) != cudaSuccess)
            return DSMEM_ERR_CUDA;
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
    if ((st = proj(kEpiO, n, a, hid / kTile, s, hid, 64, kTile)) != DSMEM_OK) return st;
    // 5-6. hn = RMSNorm(h) w_post (fused prologue), act = SiLU(hn Wg^T) * (hn Wu^T)
    a = ProjArgs{};
    a.W = static_cast<const bf16*>(p->wgu);
    a.nrm_x = static_cast<const bf16*>(p->h_out);
    a.nrm_w = static_cast<const bf16*>(p->w_post);
    a.nrm_eps = p->eps;
    a.K = hid;
    a.B = B;
    a.ffn = ffn;
    a.out = act;
    a.out_ld = ffn;
    a.err = err;
    if ((st = proj(kEpiGateUp, n, a, ffn / 64, s, 2LL * ffn, ffn, 64)) != DSMEM_OK) return st;
    // 7. out = act Wd^T
    a = ProjArgs{};
    a.W = static_cast<const bf16*>(p->wd);
    a.act = act;
    a.K = ffn;
    a.B = B;
    a.out = static_cast<bf16*>(p->out);
    a.out_ld = hid;
    a.err = err;
    return proj(kEpiDown, n, a, hid / kTile, s, hid, 64, kTile);
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
