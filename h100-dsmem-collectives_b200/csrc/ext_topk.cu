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
//   * every CTA derives the same threshold from the same histogram, so no CTA gathers for another: one scan
//     after the coarse round appends the strictly selected elements and the cut bin's candidates to two
//     shared-memory index lists (warp-aggregated appends), the fine rounds read only the candidates, one
//     st.async exchange of the per-CTA counts gives every CTA its output offset and its share of exact ties
//     (in rank order), and each CTA writes its own indices straight to the output row. Coarse keys are
//     computed two at a time (packed fp16x2 conversion). The segment is scanned twice in all (histogram,
//     lists); a candidate list that overflows, or k above the list capacity, rescans the segment instead;
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
constexpr uint32_t kScratchOff = kCntOff + 16 * 8;      // block scans and list counters: 64 u32
constexpr uint32_t kListCap = 4096;                     // entries of each index list
constexpr uint32_t kSelOff = kScratchOff + 64 * 4;      // indices of the strictly selected elements
constexpr uint32_t kCandOff = kSelOff + kListCap * 4;   // indices of the cut bin's candidates
constexpr uint32_t kSegOff = kCandOff + kListCap * 4;   // the segment (16-byte aligned)
constexpr int kCtrSel = 48, kCtrCand = 49, kCtrOut = 50, kCtrTie = 51;   // scratch words
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

// Order-preserving keys: a larger key means a larger float. NaN keys do not depend on the payload (+NaN the
// largest key, -NaN the smallest), so every NaN is an exact tie with every other NaN of its sign: on B200 the
// payload a NaN shows was not the same in every pass of the kernel, and the passes must agree.
__device__ __forceinline__ uint32_t key32(float v) {
    const uint32_t b = __float_as_uint(v);
    if (isnan(v)) return (b >> 31) ? 0u : 0xFFFFFFFFu;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
// Coarse keys (11 bits of the order-preserving key of the fp16-rounded value), two at a time: one packed
// fp16x2 conversion, the key transform on both 16-bit lanes (sign set: all bits flipped; clear: top bit set),
// then the top 11 bits of each lane. NaN inputs are binned explicitly (+NaN in the top bin, -NaN in the
// bottom one, as their fp32 keys order them): the NaN payload a conversion produces depends on the instruction
// (packed or single), and every pass must bin a value the same way.
__device__ __forceinline__ void coarse_key2(float lo, float hi, uint32_t& ck_lo, uint32_t& ck_hi) {
    const __half2 hv = __floats2half2_rn(lo, hi);   // .x (low lane) = lo
    const uint32_t x = *reinterpret_cast<const uint32_t*>(&hv);
    const uint32_t sgn = (x >> 15) & 0x00010001u;
    const uint32_t key = x ^ ((sgn * 0x7FFFu) | 0x80008000u);
    ck_lo = (key >> 5) & 0x7FFu;
    ck_hi = (key >> 21) & 0x7FFu;
    if (isnan(lo)) ck_lo = (__float_as_uint(lo) >> 31) ? 0u : 0x7FFu;
    if (isnan(hi)) ck_hi = (__float_as_uint(hi) >> 31) ? 0u : 0x7FFu;
}
__device__ __forceinline__ uint32_t coarse_key(float v) {
    uint32_t a, b;
    coarse_key2(v, v, a, b);
    return a;
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
        uint32_t* scr = c.ptr<uint32_t>(kScratchOff);
        if (tid < 4) scr[kCtrSel + tid] = 0u;
        __syncthreads();
        wait_bar(c, kLoadBar);

        // ---- coarse round: the segment as 16-byte units u of the aligned buffer, element 4u + j - off
        const int nu = (int)((off + (uint32_t)L + 3u) >> 2);
        const float4* seg4 = reinterpret_cast<const float4*>(segbuf);
        for (int u = (int)tid; u < nu; u += kThreadsTk) {
            const float4 v = seg4[u];
            uint32_t ck[4];
            coarse_key2(v.x, v.y, ck[0], ck[1]);
            coarse_key2(v.z, v.w, ck[2], ck[3]);
            const int i0 = 4 * u - (int)off;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (i0 + j >= 0 && i0 + j < L) atomicAdd(&hist[ck[j]], 1u);
        }
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
        // ---- one scan: the strictly selected (coarse > tau, or >= tau when the cut bin is taken whole) and
        // the cut bin's candidates go to two index lists (warp-aggregated appends). A candidate list that
        // overflows, or k above the list capacity, falls back to rescanning the segment below.
        const bool lists = (uint32_t)k <= kListCap;
        uint32_t* sel_list = c.ptr<uint32_t>(kSelOff);
        uint32_t* cand_list = c.ptr<uint32_t>(kCandOff);
        const uint32_t lane = tid & 31u, w = tid >> 5, lt = (1u << lane) - 1u;
        auto append = [&](bool flag, int ctr, uint32_t* list, int e) {
            const uint32_t b = __ballot_sync(0xffffffffu, flag);
            if (b == 0u) return;
            const int leader = __ffs(b) - 1;
            uint32_t pos0 = 0;
            if ((int)lane == leader) pos0 = atomicAdd(&scr[ctr], (uint32_t)__popc(b));
            pos0 = __shfl_sync(0xffffffffu, pos0, leader);
            if (flag) {
                const uint32_t pos = pos0 + __popc(b & lt);
                if (pos < kListCap) list[pos] = (uint32_t)e;
            }
        };
        if (lists) {
            for (int ub = 0; ub < nu; ub += kThreadsTk) {   // uniform trip count: the appends use full-warp ballots
                const int u = ub + (int)tid;
                uint32_t ck[4] = {0u, 0u, 0u, 0u};
                if (u < nu) {
                    const float4 v = seg4[u];
                    coarse_key2(v.x, v.y, ck[0], ck[1]);
                    coarse_key2(v.z, v.w, ck[2], ck[3]);
                }
                const int i0 = 4 * u - (int)off;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const bool valid = u < nu && i0 + j >= 0 && i0 + j < L;
                    append(valid && (ck[j] > tau || (full && ck[j] == tau)), kCtrSel, sel_list, i0 + j);
                    append(valid && !full && ck[j] == tau, kCtrCand, cand_list, i0 + j);
                }
            }
        }
        __syncthreads();
        const uint32_t nsel = scr[kCtrSel], ncand = scr[kCtrCand];
        const bool use_lists = lists && ncand <= kListCap;   // uniform in the CTA (the peers may differ)

        int shift = 32;   // no fine digit yet; else the chosen prefix is (u >> shift) == prefix
        uint32_t prefix = 0, r = cc.r;
        for (int fr = 0; fr < nfine && !full; ++fr) {
            __syncthreads();   // every thread read rowh before the next reduce-scatter
            clear_hist();
            __syncthreads();
            const int sh = shifts[fr];
            auto add = [&](float v) {
                const uint32_t u = key32(v) - base;
                if (shift < 32 && (u >> shift) != prefix) return;
                atomicAdd(&hist[(u >> sh) & masks[fr]], 1u);
            };
            if (use_lists) {
                for (uint32_t i = tid; i < ncand; i += kThreadsTk) add(seg[cand_list[i]]);
            } else {
                for (int e = (int)tid; e < L; e += kThreadsTk) {
                    const float v = seg[e];
                    if (coarse_key(v) == tau) add(v);
                }
            }
            allreduce();
            const Cut fc = find_cut(c, rowh, r);
            prefix = (shift == 32 ? 0u : (prefix << (shift - sh))) | fc.d;   // = the chosen u's top bits above sh
            shift = sh;
            r = fc.r;
            full = fc.r == fc.in_bin;
        }
        // selection: coarse > tau; or coarse == tau and (no fine round, or u's prefix > prefix, or == prefix and
        // (full, or among the first r exact ties in rank order))
        auto cls = [&](float v) -> int {   // 2 selected, 1 exact tie still to share, 0 not
            const uint32_t ck = coarse_key(v);
            if (ck != tau) return ck > tau ? 2 : 0;
            if (shift == 32) return 2;   // no fine round: full bin
            const uint32_t p = (key32(v) - base) >> shift;
            if (p != prefix) return p > prefix ? 2 : 0;
            return full ? 2 : 1;
        };
        // ---- counts. Lists: the selected list plus the candidates' classes. Otherwise warp w counts elements
        // [w * Lw, (w + 1) * Lw) of the segment (pass A of the rescan path; pass B below writes them).
        const int Lw = ((L + kWarpsTk - 1) / kWarpsTk + 31) & ~31;
        const int e0 = (int)w * Lw, e1 = min(L, e0 + Lw);
        uint32_t wsel = 0, wtie = 0;
        if (use_lists) {
            for (uint32_t i = tid; i < ncand; i += kThreadsTk) {
                const int sv = cls(seg[cand_list[i]]);
                wsel += sv == 2;
                wtie += sv == 1;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                wsel += __shfl_xor_sync(0xffffffffu, wsel, o);
                wtie += __shfl_xor_sync(0xffffffffu, wtie, o);
            }
        } else {
            for (int e = e0 + (int)lane; e - (int)lane < e1; e += 32) {
                const int sv = e < e1 ? cls(seg[e]) : 0;
                wsel += __popc(__ballot_sync(0xffffffffu, sv == 2));
                wtie += __popc(__ballot_sync(0xffffffffu, sv == 1));
            }
        }
        if (lane == 0) scr[w] = wsel, scr[16 + w] = wtie;
        __syncthreads();
        uint32_t sel_pre = 0, tie_pre = 0, sel_all = use_lists ? nsel : 0u, tie_all = 0;
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
        auto put = [&](uint32_t slot, int e) {
            if (slot < (uint32_t)k) orow[slot] = start + e;
            else dsb::report(c, DSMEM_ERR_BIT_BOUNDS);
        };
        if (use_lists) {
            for (uint32_t i = tid; i < nsel; i += kThreadsTk) put(out_off + i, (int)sel_list[i]);
            for (uint32_t i = tid; i < ncand; i += kThreadsTk) {
                const int e = (int)cand_list[i];
                const int sv = cls(seg[e]);
                if (sv == 2) put(out_off + nsel + atomicAdd(&scr[kCtrOut], 1u), e);
                if (sv == 1) {
                    const uint32_t tr = atomicAdd(&scr[kCtrTie], 1u);
                    if (tr < take) put(out_off + sel_all + tr, e);
                }
            }
        } else {   // pass B: in-warp ballots over the warp's range
            uint32_t sel_run = sel_pre, tie_run = tie_pre;
            for (int e = e0 + (int)lane; e - (int)lane < e1; e += 32) {
                const int sv = e < e1 ? cls(seg[e]) : 0;
                const uint32_t bs = __ballot_sync(0xffffffffu, sv == 2), bt = __ballot_sync(0xffffffffu, sv == 1);
                if (sv == 2) put(out_off + sel_run + __popc(bs & lt), e);
                if (sv == 1) {
                    const uint32_t tr = tie_run + __popc(bt & lt);
                    if (tr < take) put(out_off + sel_all + tr, e);
                }
                sel_run += __popc(bs);
                tie_run += __popc(bt);
            }
        }
        __syncthreads();   // the segment, the scratch and the count slots are free for the next row
    }
    // No cluster barrier at the end: every remote write into this CTA (histogram shots, counts) completed on a
    // barrier it waited for, and its own last bulk copies (the all-gather shot) had landed before any peer sent
    // the counts this CTA waited for. A CTA whose wait gave up lingers instead.
    if (__syncthreads_or(c.dead ? 1 : 0)) {
        const unsigned long long until = globaltimer() + dsb::kSettleNs;
        while (globaltimer() < until) {
        }
    }
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

dsmem_status dsmem_topk_query(int n, int cluster_size, size_t* smem_bytes) {
    if (n <= 0 || tk_fn(cluster_size) == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    const int seg = ((n + cluster_size - 1) / cluster_size + 3) / 4 * 4;
    const uint64_t smem = (uint64_t)kSegOff + ((uint64_t)seg + 4) * 4;   // + 3 elements of alignment offset
    if (smem > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    if (smem_bytes) *smem_bytes = (size_t)smem;
    return DSMEM_OK;
}

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
    size_t smem = 0;
    const dsmem_status qs = dsmem_topk_query(n, N, &smem);
    if (qs != DSMEM_OK) return qs;
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
