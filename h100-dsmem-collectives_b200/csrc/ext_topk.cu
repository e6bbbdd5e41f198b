// ext_topk.cu -- exact top-k index selection over rows of fp32 logits: a cluster per row, radix select with a
// DSMEM histogram AllReduce (sm_100a).
//
// Reference: kernels/topk_filtered_cluster8__llm_sampling__hpcops.cu (hpc-ops src/topk/topk_filtered.cu,
// topk_filtered_cluster8_exact_kernel): per row of `length` scores, the indices of the k largest, by radix select
// over a cluster of 8 CTAs that each scan a contiguous segment:
//   (i)   coarse 2048-bin histogram of an order-preserving key of the fp16-rounded score (sign, 5 exponent and
//         5 mantissa bits: a monotone projection, so a larger coarse key means a larger score),
//   (ii)  AllReduce(sum) of the histogram over the cluster (cluster_allreduce_histogram: each CTA owns 2048/N
//         bins; pull reduce-scatter + push all-gather between two cluster barriers),
//   (iii) the threshold bin tau with count(key > tau) < k <= count(key >= tau),
//   (iv)  up to three fine rounds over the fp32 key bits [21..31], [10..20], [0..9] of the candidates still tied,
//   (v)   rank 0 gathers the selected indices and boundary candidates through DSMEM and writes the row.
// The hpc-ops sources are an absent submodule here (the excerpt needs its headers), so this is a restatement of
// the published radix-select method with the reference's key projection, digit split and AllReduce placement.
//
// B200 design (one launch; persistent clusters of N CTAs, 512 threads, one row at a time per cluster):
//   * CTA b stages its segment of the row in shared memory once (one bulk copy of the 16-byte-aligned interior,
//     plain loads for the up to 3 + 3 ragged end elements: rows of odd length are not 16-byte aligned), and
//     every later pass (histograms, counts, output) reads shared memory;
//   * each histogram round is a two-shot AllReduce in shared memory: CTA b bulk-copies bins [j*B, (j+1)*B) of
//     its histogram into slot b of CTA j (B = 2048/N), CTA j sums the N slots of its bins and bulk-copies the
//     totals into every CTA's row histogram at the same offset; each shot completes on the receiver's mbarrier,
//     so a round has no cluster barrier, and buffer reuse across rounds and rows follows from the shots' order
//     (a peer's next reduce-scatter comes after it received this CTA's all-gather, i.e. after this CTA summed
//     its slots; its next all-gather comes after this CTA's next reduce-scatter, i.e. after this CTA read the
//     row histogram);
//   * every CTA derives the same threshold from the same histogram, so no CTA gathers for another: after the
//     rounds, each CTA counts its strictly selected elements and its exact ties, one st.async exchange of those
//     two counts gives every CTA its output offset and its share of the ties (in rank order), and each CTA
//     writes its own indices straight to the output row (warp-range ballot compaction, one block scan);
//   * the fine rounds run on the key relative to the coarse bin's exact key range (the floats rounding to the
//     bin's fp16 values lie strictly between the neighbouring fp16 values), so for finite bins two rounds of
//     11 + at most 10 bits resolve the cut instead of the reference's three absolute rounds.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "smem_attr.cuh"

namespace {

using namespace dsmem;

constexpr int kThreadsTk = 512;
constexpr int kWarpsTk = kThreadsTk / 32;
constexpr int kBins = 2048;
// barrier ids (8 bytes each in [0, 128)): segment load 0, reduce-scatter 1, all-gather 2, counts 3; byte 120 holds
// the end-of-kernel flag word of dsb::finish
constexpr int kLoadBar = 0, kRsBar = 1, kAgBar = 2, kCntBar = 3;
constexpr uint32_t kHistOff = 128;                      // this CTA's histogram of the round: kBins u32
constexpr uint32_t kSlotOff = kHistOff + kBins * 4;     // reduce-scatter slots: N x B u32 (= kBins u32)
constexpr uint32_t kRowHistOff = kSlotOff + kBins * 4;  // the cluster's histogram of the round: kBins u32
constexpr uint32_t kCntOff = kRowHistOff + kBins * 4;   // count exchange: 16 x 2 u32
constexpr uint32_t kScratchOff = kCntOff + 16 * 8;      // block scans: 64 u32
constexpr uint32_t kSegOff = kScratchOff + 64 * 4;      // the segment (16-byte aligned)
static_assert(kSegOff % 16 == 0, "segment alignment");

struct TkArgs {
    const float* x;
    int* out;
    unsigned* err;
    unsigned long long wait_limit_ns;
    long long rows;
    int n, k;
    int seg;          // elements per CTA segment (a multiple of 4)
    uint32_t smem_bytes;
};

// Order-preserving keys: a larger key means a larger float (NaN above +inf, -NaN below -inf).
__device__ __forceinline__ uint32_t key32(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint32_t coarse_key(float v) {   // 11 bits of the fp16-rounded value's key
    const uint32_t h = (uint32_t)__half_as_ushort(__float2half_rn(v));
    const uint32_t k16 = (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
    return k16 >> 5;
}

// The fp16 value whose coarse 16-bit key is k16 (the inverse of the key transform of coarse_key).
__device__ __forceinline__ float half16_value(uint32_t k16) {
    const uint32_t h = (k16 & 0x8000u) ? (k16 & 0x7FFFu) : (~k16 & 0xFFFFu);
    return __half2float(__ushort_as_half((unsigned short)h));
}

__device__ __forceinline__ void wait_bar(dsb::Ctx& c, int i) { dsb::wait(c, i); }

// Block-wide: the largest bin d with sum(hist[d..]) >= r, the count strictly above it and r' = r - above.
// Every thread returns the same values. Thread t owns bins [4t, 4t + 4).
struct Cut {
    uint32_t d, above, r, in_bin;
};
__device__ Cut find_cut(const dsb::Ctx& c, const uint32_t* hist, uint32_t r) {
    uint32_t* scr = c.ptr<uint32_t>(kScratchOff);
    const uint32_t t = threadIdx.x, lane = t & 31u, w = t >> 5;
    const uint4 h = reinterpret_cast<const uint4*>(hist)[t];
    const uint32_t s = h.x + h.y + h.z + h.w;
    uint32_t v = s;   // suffix sum over lanes >= lane
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_down_sync(0xffffffffu, v, off);
        if (lane + off < 32) v += y;
    }
    if (lane == 0) scr[w] = v;
    __syncthreads();
    uint32_t hi = 0;   // bins above this warp
    for (uint32_t q = w + 1; q < (uint32_t)kWarpsTk; ++q) hi += scr[q];
    const uint32_t above_t = hi + (v - s);   // bins above this thread's four
    if (above_t < r && r <= above_t + s) {
        uint32_t acc = above_t;
        const uint32_t hb[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
        for (int j = 3; j >= 0; --j) {
            if (acc + hb[j] >= r) {
                scr[32] = 4u * t + (uint32_t)j;
                scr[33] = acc;
                scr[34] = hb[j];
                break;
            }
            acc += hb[j];
        }
    }
    __syncthreads();
    Cut cut;
    cut.d = scr[32];
    cut.above = scr[33];
    cut.in_bin = scr[34];
    cut.r = r - cut.above;
    __syncthreads();   // scratch free for the next scan
    return cut;
}

template <int N>
__global__ void __launch_bounds__(kThreadsTk, 1) topk_cluster_kernel(const __grid_constant__ TkArgs a) {
    constexpr uint32_t B = kBins / N;   // bins owned per CTA
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(c.bar(i), 1);
        fence_mbar_init();
    }
    __syncthreads();
    cluster_sync();   // every CTA's barriers initialised before any remote copy
    uint32_t* hist = c.ptr<uint32_t>(kHistOff);
    const uint32_t* slots = c.ptr<const uint32_t>(kSlotOff);
    uint32_t* rowh = c.ptr<uint32_t>(kRowHistOff);
    float* segbuf = c.ptr<float>(kSegOff);
    const int n = a.n, k = a.k;
    const int start = (int)c.rank * a.seg;
    const int L = max(0, min(a.seg, n - start));   // this CTA's elements of every row
    const long long nclu = (long long)num_clusters(), cq = (long long)cluster_id();

    // One histogram AllReduce: hist (this CTA) -> rowh (the cluster's), two shots over DSMEM.
    auto allreduce = [&]() {
        fence_proxy_async_smem();   // the histogram's generic writes before the bulk copies read it
        __syncthreads();
        if (tid == 0) {
            dsb::arm(c, kRsBar, (N - 1) * B * 4u);
            for (uint32_t j = 1; j < (uint32_t)N; ++j) {
                const uint32_t dst = (c.rank + j) % N;
                bulk_push(dst, c.sa + kSlotOff + c.rank * B * 4u, c.sa + kHistOff + dst * B * 4u, B * 4u,
                          c.bar(kRsBar));
            }
        }
        wait_bar(c, kRsBar);
        for (uint32_t i = tid; i < B; i += kThreadsTk) {
            uint32_t s = hist[c.rank * B + i];
#pragma unroll
            for (int q = 0; q < N; ++q)
                if ((uint32_t)q != c.rank) s += slots[q * B + i];
            rowh[c.rank * B + i] = s;
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            dsb::arm(c, kAgBar, (N - 1) * B * 4u);
            for (uint32_t j = 1; j < (uint32_t)N; ++j) {
                const uint32_t dst = (c.rank + j) % N;
                bulk_push(dst, c.sa + kRowHistOff + c.rank * B * 4u, c.sa + kRowHistOff + c.rank * B * 4u, B * 4u,
                          c.bar(kAgBar));
            }
        }
        wait_bar(c, kAgBar);
    };
    auto clear_hist = [&]() {
        reinterpret_cast<uint4*>(hist)[tid] = make_uint4(0u, 0u, 0u, 0u);   // kBins / 4 == kThreadsTk
    };

    for (long long row = cq; row < a.rows; row += nclu) {
        c.deadline = globaltimer() + c.wait_limit;
        c.unit = (uint32_t)(row / nclu);
        // ---- stage the segment: elements [g0, g0 + L) of the flattened array at smem index (g0 & 3) + i
        const long long g0 = row * (long long)n + start, g1 = g0 + L;
        const long long c0 = (g0 + 3) & ~3LL, c1 = g1 & ~3LL;
        const long long a0 = c0 < g1 ? c0 : g1, a1 = c1 > a0 ? c1 : a0;   // the 16-byte-aligned interior
        const uint32_t off = (uint32_t)(g0 & 3);
        float* seg = segbuf + off;
        if (tid == 0) {
            const uint32_t bytes = (uint32_t)(a1 - a0) * 4u;
            dsb::arm(c, kLoadBar, bytes);
            if (bytes) bulk_load_g2s(c.sa + kSegOff + (uint32_t)(a0 - (g0 & ~3LL)) * 4u, a.x + a0, bytes, c.bar(kLoadBar));
        }
        if (tid < (uint32_t)(a0 - g0)) seg[tid] = a.x[g0 + tid];                              // ragged head
        if (tid < (uint32_t)(g1 - a1)) seg[(a1 - g0) + tid] = a.x[a1 + tid];                  // ragged tail
        clear_hist();
        __syncthreads();
        wait_bar(c, kLoadBar);

        // ---- coarse round
        for (int e = (int)tid; e < L; e += kThreadsTk) atomicAdd(&hist[coarse_key(seg[e])], 1u);
        allreduce();
        const Cut cc = find_cut(c, rowh, (uint32_t)k);
        const uint32_t tau = cc.d;
        bool full = cc.r == cc.in_bin;   // the whole cut bin is selected
        // Fine rounds over the candidates (coarse key == tau) on u = key32 - base: the floats that round to the
        // bin's fp16 values lie strictly between the fp16 values just below and just above the bin, so when
        // those are finite and the key span fits 21 bits, u < 2^21 and two digits cover it (the top 11 bits of
        // the span, then the rest); otherwise three absolute digits of key32 (bits 21..31, 10..20, 0..9).
        uint32_t base = 0;
        int shifts[3] = {21, 10, 0}, nfine = 3;
        uint32_t masks[3] = {0x7FFu, 0x7FFu, 0x3FFu};
        {
            const uint32_t kb = tau << 5;
            bool ok = kb > 0u && kb + 32u <= 0xFFFFu;
            float lo = 0.f, hi = 0.f;
            if (ok) {
                lo = half16_value(kb - 1u);
                hi = half16_value(kb + 32u);
                ok = !isnan(lo) && !isnan(hi);
            }
            if (ok) {
                const uint32_t klo = key32(lo) + 1u, span = key32(hi) - klo;   // u in [0, span)
                const int bits = span <= 1u ? 1 : 32 - __clz(span - 1u);        // bits of span - 1
                if (bits <= 21) {
                    base = klo;
                    const int s1 = bits > 11 ? bits - 11 : 0;
                    shifts[0] = s1, masks[0] = 0x7FFu, shifts[1] = 0, masks[1] = (1u << s1) - 1u;
                    nfine = s1 > 0 ? 2 : 1;
                }
            }
        }
        int shift = 32;   // no fine digit yet; else the chosen prefix is (u >> shift) == prefix
        uint32_t prefix = 0, r = cc.r;
        for (int fr = 0; fr < nfine && !full; ++fr) {
            __syncthreads();   // every thread read rowh before the next reduce-scatter
            clear_hist();
            __syncthreads();
            const int sh = shifts[fr];
            for (int e = (int)tid; e < L; e += kThreadsTk) {
                const float v = seg[e];
                if (coarse_key(v) != tau) continue;
                const uint32_t u = key32(v) - base;
                if (shift < 32 && (u >> shift) != prefix) continue;
                atomicAdd(&hist[(u >> sh) & masks[fr]], 1u);
            }
            allreduce();
            const Cut fc = find_cut(c, rowh, r);
            prefix = (shift == 32 ? 0u : (prefix << (shift - sh))) | fc.d;   // = the chosen u's top bits above sh
            shift = sh;
            r = fc.r;
            full = fc.r == fc.in_bin;
        }
        // selection: coarse > tau; or coarse == tau and (no fine round, or u's prefix > prefix, or == prefix and
        // (full, or among the first r exact ties in rank/index order))
        auto cls = [&](float v) -> int {   // 2 selected, 1 exact tie still to share, 0 not
            const uint32_t ck = coarse_key(v);
            if (ck != tau) return ck > tau ? 2 : 0;
            if (shift == 32) return 2;   // no fine round: full bin
            const uint32_t p = (key32(v) - base) >> shift;
            if (p != prefix) return p > prefix ? 2 : 0;
            return full ? 2 : 1;
        };
        // ---- output: warp w owns elements [w * Lw, (w + 1) * Lw) of the segment, 32 at a time. Pass A counts
        // the strictly selected and the tied elements per warp; one block scan gives every warp its offsets;
        // pass B writes with in-warp ballots (no block barrier per element tile).
        const int Lw = ((L + kWarpsTk - 1) / kWarpsTk + 31) & ~31;
        const uint32_t lane = tid & 31u, w = tid >> 5, lt = (1u << lane) - 1u;
        const int e0 = (int)w * Lw, e1 = min(L, e0 + Lw);
        uint32_t wsel = 0, wtie = 0;
        for (int e = e0 + (int)lane; e - (int)lane < e1; e += 32) {
            const int sv = e < e1 ? cls(seg[e]) : 0;
            wsel += __popc(__ballot_sync(0xffffffffu, sv == 2));
            wtie += __popc(__ballot_sync(0xffffffffu, sv == 1));
        }
        uint32_t* scr = c.ptr<uint32_t>(kScratchOff);
        if (lane == 0) scr[w] = wsel, scr[16 + w] = wtie;
        __syncthreads();
        uint32_t sel_pre = 0, tie_pre = 0, sel_all = 0, tie_all = 0;
        for (uint32_t q = 0; q < (uint32_t)kWarpsTk; ++q) {
            const uint32_t sq = scr[q], tq = scr[16 + q];
            sel_pre += q < w ? sq : 0u;
            tie_pre += q < w ? tq : 0u;
            sel_all += sq;
            tie_all += tq;
        }
        if (tid == 0) {   // exchange (selected, ties) with every CTA of the cluster, this one included
            dsb::arm(c, kCntBar, N * 8u);
            const unsigned long long pk = ((unsigned long long)tie_all << 32) | sel_all;
            for (uint32_t q = 0; q < (uint32_t)N; ++q) {
                const uint32_t rd = mapa(c.sa + kCntOff + c.rank * 8u, q), rb = mapa(c.bar(kCntBar), q);
                asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(rd),
                             "l"(pk), "r"(rb)
                             : "memory");
            }
        }
        wait_bar(c, kCntBar);
        // Exact ties (after the last fine round, when the cut bin is not taken whole) go to the ranks in order:
        // rank q takes min(its ties, r - ties of lower ranks). Rank q's indices follow those of lower ranks;
        // within a rank the strictly selected come first, then its taken ties.
        const uint32_t* cnt = c.ptr<const uint32_t>(kCntOff);
        const bool share = shift != 32 && !full;
        uint32_t out_off = 0, ties_before = 0, take = 0;
        for (uint32_t q = 0; q <= c.rank; ++q) {
            const uint32_t tq = cnt[2 * q + 1];
            const uint32_t tk = share ? (uint32_t)max(0, min((int)tq, (int)r - (int)ties_before)) : 0u;
            if (q < c.rank) out_off += cnt[2 * q] + tk;
            else take = tk;
            ties_before += tq;
        }
        int* orow = a.out + row * (long long)k;
        uint32_t sel_run = sel_pre, tie_run = tie_pre;
        for (int e = e0 + (int)lane; e - (int)lane < e1; e += 32) {
            const int sv = e < e1 ? cls(seg[e]) : 0;
            const uint32_t bs = __ballot_sync(0xffffffffu, sv == 2), bt = __ballot_sync(0xffffffffu, sv == 1);
            uint32_t slot = 0xFFFFFFFFu;
            if (sv == 2) slot = out_off + sel_run + __popc(bs & lt);
            if (sv == 1) {
                const uint32_t tr = tie_run + __popc(bt & lt);
                if (tr < take) slot = out_off + sel_all + tr;
            }
            if (sv != 0 && slot != 0xFFFFFFFFu) {
                if (slot < (uint32_t)k) orow[slot] = start + e;
                else dsb::report(c, DSMEM_ERR_BIT_BOUNDS);
            }
            sel_run += __popc(bs);
            tie_run += __popc(bt);
        }
        __syncthreads();   // the segment, the scratch and the count slots are free for the next row
    }
    dsb::finish(c);
}

std::mutex g_mu;
std::map<std::tuple<const void*, int, uint32_t>, int> g_occ;
unsigned* g_err[64] = {};

const void* tk_fn(int n) {
    switch (n) {
        case 2: return reinterpret_cast<const void*>(&topk_cluster_kernel<2>);
        case 4: return reinterpret_cast<const void*>(&topk_cluster_kernel<4>);
        case 8: return reinterpret_cast<const void*>(&topk_cluster_kernel<8>);
        case 16: return reinterpret_cast<const void*>(&topk_cluster_kernel<16>);
    }
    return nullptr;
}

}  // namespace

extern "C" {

dsmem_status dsmem_topk_launch(const float* logits, long long rows, int n, int k, int* out_indices, int cluster_size,
                               dsmem_stream_t stream) {
    if (logits == nullptr || out_indices == nullptr || rows < 0 || n <= 0 || k < 1 || k > n)
        return DSMEM_ERR_INVALID_ARGUMENT;
    // 16-byte aligned logits: the segments' aligned interiors are bulk-copied
    if ((reinterpret_cast<uintptr_t>(logits) & 15u) || (reinterpret_cast<uintptr_t>(out_indices) & 3u))
        return DSMEM_ERR_INVALID_ARGUMENT;
    const void* fn = tk_fn(cluster_size);
    if (fn == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DSMEM_OK;
    const int N = cluster_size;
    const int seg = ((n + N - 1) / N + 3) / 4 * 4;
    const uint64_t smem = (uint64_t)kSegOff + ((uint64_t)seg + 4) * 4;   // + 3 elements of alignment offset
    if (smem > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)N;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreadsTk, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int resident = 0;
    TkArgs a{};
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_err[dev] == nullptr) {
            if (cudaMalloc(&g_err[dev], 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
            if (cudaMemset(g_err[dev], 0, 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
        }
        if (dsb_attr::ensure_smem(fn, dev, (uint32_t)smem, N > 8) != cudaSuccess) return DSMEM_ERR_CUDA;
        const auto key = std::make_tuple(fn, dev, (uint32_t)smem);
        auto it = g_occ.find(key);
        if (it == g_occ.end()) {
            cfg.gridDim = dim3((unsigned)N, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&resident, fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
            g_occ[key] = resident;
        } else {
            resident = it->second;
        }
        a.err = g_err[dev];
    }
    if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;
    const long long clusters = std::min<long long>(rows, resident);
    cfg.gridDim = dim3((unsigned)(clusters * N), 1, 1);
    a.x = logits;
    a.out = out_indices;
    a.wait_limit_ns = 1000000000ull;
    a.rows = rows;
    a.n = n;
    a.k = k;
    a.seg = seg;
    a.smem_bytes = (uint32_t)smem;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

dsmem_status dsmem_topk_check(int device, unsigned* error_bits) {
    unsigned v = 0;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (device < 0 || device >= 64) return DSMEM_ERR_INVALID_ARGUMENT;
        if (g_err[device] != nullptr) {
            if (cudaMemcpy(&v, g_err[device], sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return DSMEM_ERR_CUDA;
            if (cudaMemset(g_err[device], 0, 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
        }
    }
    if (error_bits) *error_bits = v;
    return DSMEM_OK;
}

}  // extern "C"
