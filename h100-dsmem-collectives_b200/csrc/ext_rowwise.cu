// ext_rowwise.cu -- row-wise reduction-reuse workloads for sm_100a: a row per cluster, one DSMEM exchange per row.
//
// Reference kernels (the clustered variants of kernels/*__reduction_reuse__credit.cu; fp32, rows x cols):
//   rowwise_quant__reduction_reuse__credit.cu:104-155           q = clamp(rint(x * 127/amax)), scale = amax/127
//   lars_momentum__reduction_reuse__credit.cu:126-185            u = mu m + g + wd w, w' = w - lr trust u, m' = u
//   layernorm_backward__reduction_reuse__credit.cu:119-186       dx of LayerNorm (two statistic stages)
//   pearson_backward__reduction_reuse__credit.cu:158-227         dx, dy of the Pearson correlation (one 5-scalar stage)
//   softmax_logits_backward__reduction_reuse__credit.cu:164-237  dx of softmax (max, sum, dot: three stages)
//   weighted_var_backward__reduction_reuse__credit.cu:135-221    dx of the weighted variance (three stages)
// There, P CTAs share a row, CTA b stages column slice b in shared memory, and every row statistic is an
// AllReduce over the cluster by the direct replicated push with two cluster barriers per statistic stage.
//
// B200 design:
//   * one exchange per row for every workload. Each CTA reduces its slice to a small mergeable record and the
//     cluster merges the N records: a maximum; plain sums; count (or weight), mean and centred sums for the
//     variance statistics, merged by the pairwise update of Chan, Golub & LeVeque (1979); a max-shifted sum of
//     exponentials for the softmax, merged by the online-softmax rescaling (Milakov & Gimelshein 2018). The
//     reference's later stages follow algebraically from the merged record (sum dyg*xhat = inv_std * sum
//     dyg*(x - mean), sum w(x-m)^2 and sum dy(x-m) shifted to the global mean), so a row costs one DSMEM
//     round trip instead of 1-3 rounds of two cluster barriers;
//   * the exchange is the replicated push by st.async: lane q < N of the row team's first warp stores the record
//     into slot[set][b][row] of CTA q (itself included), the bytes completing on CTA q's mbarrier of the set;
//     no cluster barrier per row. Every lane merges the N records with the same butterfly of symmetric merges,
//     so every CTA (and lane) of the cluster derives bit-identical row statistics;
//   * persistent clusters; rows go in groups of R = 8 / tw (a team of tw warps per row); cluster q of C takes
//     groups q, q + C, ..; a producer warp streams each group's row slices with one bulk copy per row and input
//     into a ring of shared-memory stages (full/empty mbarriers): every input is read from HBM once and from
//     shared memory twice (statistics, outputs). (Re-reading the rows through the L2 for the output pass, to
//     free a stage right after its statistics, measured about 2x slower.)
//   * the teams run one group ahead: group i+1's records go out before group i's outputs are computed, so
//     the exchange hides behind the output pass;
//   * outputs leave with 16-byte streaming stores (int8: 4-byte); rows whose columns are not a multiple of 4
//     (or unaligned arrays) take plain per-element copies and stores through the same pipeline.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <type_traits>

#include "../../include/dsmem_b200.h"
#include "../collectives/dsmem_b200_algos.cuh"
#include "smem_attr.cuh"

namespace {

using namespace dsmem;

constexpr int kWarps = 8;                       // row-team warps
constexpr int kThreadsRw = (kWarps + 1) * 32;   // + the producer warp
constexpr int kProducer = kWarps;
constexpr int kMaxStages = 8;
constexpr int kMaxAhead = 1;                    // groups whose records go out before a group's outputs
constexpr int kMaxSets = 2 * kMaxAhead + 2;     // exchange slot sets (the reuse argument is at the consumer loop)
constexpr int kMaxKP = 8;                       // record floats (padded to 1, 2, 4 or 8)
// barrier ids (8 bytes each, [0, 256) of shared memory): full[s] 0..7, column vector 8, empty[s] 16..23,
// exchange[set] 24..31; byte 120 (id 15) holds the end-of-kernel flag word of dsb::finish
constexpr int kFull = 0, kColBar = 8, kEmpty = 16, kExch = 24;
constexpr uint32_t kBarBytes = 256;
constexpr uint32_t kRedOff = kBarBytes;                       // team scratch: 8 warps x 8 floats
constexpr uint32_t kSlotsOff = kRedOff + kWarps * kMaxKP * 4;  // 512
static_assert(8 * kColBar < (int)dsb::kFlagOff && 8 * kEmpty > (int)dsb::kFlagOff, "barrier ids overlap the flag");
static_assert(kExch + kMaxSets <= (int)kBarBytes / 8 && kEmpty + kMaxStages <= kExch, "barrier ids overlap");

struct RwArgs {
    const float* in[3];   // per-element inputs (row-major rows x cols)
    const float* col;     // per-column input (LayerNorm gamma) or null
    const float* rowin;   // per-row input (Pearson upstream gradient) or null
    void* out[2];         // per-element outputs
    float* rowout;        // per-row output (quantisation scales) or null
    unsigned* err;
    unsigned long long wait_limit_ns;
    long long rows;
    int cols;
    int slice;            // elements per CTA column slice (a multiple of 4)
    int tw;               // warps per row team (1, 2, 4, 8); rows per group R = 8 / tw
    int stages;           // ring stages (1..8)
    int ahead;            // groups whose records go out before a group's outputs (0 or 1, <= stages - 1)
    int sets;             // exchange slot sets: 2 * ahead + 2
    int vec;              // cols % 4 == 0 and 16-B aligned arrays: bulk copies and vector stores
    uint32_t smem_bytes;
    uint32_t col_off, stage_off, stage_bytes;
    float p[5];           // workload parameters
};

__host__ __device__ constexpr uint32_t align128(uint32_t v) { return (v + 127u) & ~127u; }
__host__ __device__ constexpr uint32_t rw_slots_bytes(int sets, int n, int r, int kp) {
    return (uint32_t)sets * n * r * kp * 4u;
}

// Bounded wait by the calling thread for barrier i to finish the phase of parity `par`.
__device__ __forceinline__ void wait_par(dsb::Ctx& c, int i, uint32_t par) {
    if (c.dead) return;
    if (mbar_try_wait_parity(c.bar(i), par)) return;
    if (!mbar_wait_parity_until(c.bar(i), par, c.deadline)) {
        c.dead = true;
        if ((threadIdx.x & 31) == 0) dsb::report_timeout(c, i);
    }
}

// A row team: tw warps (tw * 32 threads) on one row of a group.
struct Team {
    uint32_t warp, lane, team, tw, tt, TT;
    dsb::Ctx* c;
    __device__ __forceinline__ void bar() const {
        if (tw > 1) asm volatile("bar.sync %0, %1;" ::"r"(1u + team), "r"(tw * 32u) : "memory");
    }
    // Team-wide sum of K values; every thread gets the same totals (warp butterfly, then the team's warps in
    // order).
    template <int K>
    __device__ __forceinline__ void sum(float (&v)[K]) const {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int k = 0; k < K; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
        if (tw == 1) return;
        float* red = c->ptr<float>(kRedOff);
        if (lane == 0)
#pragma unroll
            for (int k = 0; k < K; ++k) red[warp * kMaxKP + k] = v[k];
        bar();
        const uint32_t w0 = team * tw;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            float t = red[w0 * kMaxKP + k];
            for (uint32_t w = 1; w < tw; ++w) t += red[(w0 + w) * kMaxKP + k];
            v[k] = t;
        }
        bar();   // scratch free for the next reduction
    }
    __device__ __forceinline__ float max(float v) const {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (tw == 1) return v;
        float* red = c->ptr<float>(kRedOff);
        if (lane == 0) red[warp * kMaxKP] = v;
        bar();
        const uint32_t w0 = team * tw;
        float t = red[w0 * kMaxKP];
        for (uint32_t w = 1; w < tw; ++w) t = fmaxf(t, red[(w0 + w) * kMaxKP]);
        bar();
        return t;
    }
};

// Shared-memory row slices of one row (one per input) and the column slice; L valid elements.
template <int KIN>
struct Slices {
    const float* s[KIN];
    const float* col;
    int L;
    __device__ __forceinline__ float4 ld(int a, int u) const { return reinterpret_cast<const float4*>(s[a])[u]; }
    __device__ __forceinline__ float4 ldc(int u) const { return reinterpret_cast<const float4*>(col)[u]; }
};
__device__ __forceinline__ float f4(const float4& v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

// Runs f(u, n) over this thread's 4-element units u of an L-element slice (n valid elements in the unit).
template <class F>
__device__ __forceinline__ void for_units(const Team& tm, int L, F&& f) {
    for (int u = (int)tm.tt; 4 * u < L; u += (int)tm.TT) f(u, min(4, L - 4 * u));
}

// ------------------------------------------------------------------------------------------- workloads
// Each workload: kIn staged inputs, kOut per-element outputs, a record of kK floats (padded to kKP), local()
// (the CTA's record of its slice; every team thread gets it), ident(), merge() (symmetric: merge(a, b) and
// merge(b, a) are bitwise equal), Par finalize() and out() (outputs of 4 elements).

// rowwise_quant__reduction_reuse__credit.cu:129-153: amax = max |x| (identity 0, NaN ignored by fmaxf),
// inv_scale = 127/amax (0 for an all-zero row), q = clamp(nearbyint(x * inv_scale), -127, 127), scale = amax/127
// written by CTA rank 0.
struct WQuant {
    static constexpr int kIn = 1, kOut = 1, kK = 1, kKP = 1;
    static constexpr bool kCol = false, kRowIn = false, kRowOut = true, kI8 = true;
    struct Par {
        float inv, scale;
    };
    static __device__ void ident(float (&r)[kKP]) { r[0] = 0.f; }
    static __device__ void local(const Team& tm, const Slices<kIn>& sl, float (&r)[kKP]) {
        float m = 0.f;
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 v = sl.ld(0, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) m = fmaxf(m, fabsf(f4(v, j)));
        });
        r[0] = tm.max(m);
    }
    static __device__ void merge(float (&a)[kKP], const float (&b)[kKP]) { a[0] = fmaxf(a[0], b[0]); }
    static __device__ Par finalize(const float (&t)[kKP], const RwArgs&, float) {
        const float amax = t[0];
        return Par{amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f, __fdiv_rn(amax, 127.0f)};
    }
    static __device__ float row_out(const Par& p) { return p.scale; }
    static __device__ void out(const Par& p, const float4 (&v)[kIn], const float4&, float4 (&o)[kOut]) {
        auto q = [&](float x) { return fminf(127.0f, fmaxf(-127.0f, rintf(__fmul_rn(x, p.inv)))); };
        o[0] = make_float4(q(v[0].x), q(v[0].y), q(v[0].z), q(v[0].w));
    }
};

// lars_momentum__reduction_reuse__credit.cu:160-184 (update_value :120-124): u = mu*m + g + wd*w,
// trust = eta*||w|| / (||u|| + eps), w' = w - lr*trust*u, m' = u. Record {sum w^2, sum u^2}.
// p = {mu, wd, lr, eta, eps}.
struct WLars {
    static constexpr int kIn = 3, kOut = 2, kK = 2, kKP = 2;
    static constexpr bool kCol = false, kRowIn = false, kRowOut = false, kI8 = false;
    struct Par {
        float mu, wd, step;
    };
    static __device__ __forceinline__ float upd(const RwArgs& a, float w, float g, float m) {
        return a.p[0] * m + g + a.p[1] * w;
    }
    static __device__ void ident(float (&r)[kKP]) { r[0] = r[1] = 0.f; }
    static __device__ void local(const Team& tm, const Slices<kIn>& sl, float (&r)[kKP], const RwArgs& a) {
        float s[2] = {0.f, 0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 w = sl.ld(0, u), g = sl.ld(1, u), m = sl.ld(2, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) {
                    const float wj = f4(w, j), uj = upd(a, wj, f4(g, j), f4(m, j));
                    s[0] = fmaf(wj, wj, s[0]);
                    s[1] = fmaf(uj, uj, s[1]);
                }
        });
        tm.sum<2>(s);
        r[0] = s[0];
        r[1] = s[1];
    }
    static __device__ void merge(float (&a)[kKP], const float (&b)[kKP]) {
        a[0] += b[0];
        a[1] += b[1];
    }
    static __device__ Par finalize(const float (&t)[kKP], const RwArgs& a, float) {
        const float trust = a.p[3] * sqrtf(t[0]) / (sqrtf(t[1]) + a.p[4]);
        return Par{a.p[0], a.p[1], a.p[2] * trust};
    }
    static __device__ void out(const Par& p, const float4 (&v)[kIn], const float4&, float4 (&o)[kOut]) {
        auto one = [&](float w, float g, float m, float& wo, float& mo) {
            const float u = p.mu * m + g + p.wd * w;
            wo = w - p.step * u;
            mo = u;
        };
        one(v[0].x, v[1].x, v[2].x, o[0].x, o[1].x);
        one(v[0].y, v[1].y, v[2].y, o[0].y, o[1].y);
        one(v[0].z, v[1].z, v[2].z, o[0].z, o[1].z);
        one(v[0].w, v[1].w, v[2].w, o[0].w, o[1].w);
    }
};

// Count-weighted merge of (n, mean, centred sums) records (Chan, Golub & LeVeque 1979), written so that
// merge(a, b) == merge(b, a) bitwise. Returns the merged mean; da, db = the parts' means minus it.
__device__ __forceinline__ float chan_mean(float na, float ma, float nb, float mb, float n) {
    return n > 0.f ? (na * ma + nb * mb) / n : 0.f;
}

// layernorm_backward__reduction_reuse__credit.cu:146-185: mean = sum x / cols, var = max(sum x^2/cols - mean^2, 0),
// inv_std = rsqrt(var + eps), xhat = (x - mean) inv_std, dyg = dy gamma,
// dx = (dyg - mean(dyg) - xhat mean(dyg xhat)) inv_std. Record {n, mean, sum (x-mean)^2, sum dyg,
// sum dyg (x-mean)} of the slice; sum dyg xhat = inv_std * sum dyg (x - mean). p = {eps}.
struct WLnBwd {
    static constexpr int kIn = 2, kOut = 1, kK = 5, kKP = 8;
    static constexpr bool kCol = true, kRowIn = false, kRowOut = false, kI8 = false;
    struct Par {
        float mean, inv_std, mdyg, mdx;
    };
    static __device__ void ident(float (&r)[kKP]) {
#pragma unroll
        for (int k = 0; k < kKP; ++k) r[k] = 0.f;
    }
    static __device__ void local(const Team& tm, const Slices<kIn>& sl, float (&r)[kKP], const RwArgs&) {
        float s1[1] = {0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 x = sl.ld(0, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) s1[0] += f4(x, j);
        });
        tm.sum<1>(s1);
        const float cnt = (float)sl.L, mean = sl.L > 0 ? s1[0] / cnt : 0.f;
        float s[3] = {0.f, 0.f, 0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 x = sl.ld(0, u), dy = sl.ld(1, u), g = sl.ldc(u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) {
                    const float d = f4(x, j) - mean, dyg = f4(dy, j) * f4(g, j);
                    s[0] = fmaf(d, d, s[0]);
                    s[1] += dyg;
                    s[2] = fmaf(dyg, d, s[2]);
                }
        });
        tm.sum<3>(s);
        r[0] = cnt, r[1] = mean, r[2] = s[0], r[3] = s[1], r[4] = s[2];
        r[5] = r[6] = r[7] = 0.f;
    }
    static __device__ void merge(float (&a)[kKP], const float (&b)[kKP]) {
        const float n = a[0] + b[0], m = chan_mean(a[0], a[1], b[0], b[1], n);
        const float da = a[1] - m, db = b[1] - m;
        const float m2 = (a[2] + b[2]) + (a[0] * da * da + b[0] * db * db);
        const float c = (a[4] + b[4]) + (da * a[3] + db * b[3]);
        a[0] = n, a[1] = m, a[2] = m2, a[3] = a[3] + b[3], a[4] = c;
    }
    static __device__ Par finalize(const float (&t)[kKP], const RwArgs& a, float) {
        const float inv_cols = 1.0f / (float)a.cols;
        const float var = fmaxf(t[2] * inv_cols, 0.f);
        const float inv_std = rsqrtf(var + a.p[0]);
        return Par{t[1], inv_std, t[3] * inv_cols, t[4] * inv_std * inv_cols};
    }
    static __device__ void out(const Par& p, const float4 (&v)[kIn], const float4& g, float4 (&o)[kOut]) {
        auto one = [&](float x, float dy, float gm) {
            const float xhat = (x - p.mean) * p.inv_std;
            return (dy * gm - p.mdyg - xhat * p.mdx) * p.inv_std;
        };
        o[0] = make_float4(one(v[0].x, v[1].x, g.x), one(v[0].y, v[1].y, g.y), one(v[0].z, v[1].z, g.z),
                           one(v[0].w, v[1].w, g.w));
    }
};

// pearson_backward__reduction_reuse__credit.cu:187-226: var_x = sum (x - mean_x)^2, var_y likewise,
// cov = sum (x - mean_x)(y - mean_y) (sums, not means), inv_x = rsqrt(var_x + eps), inv_y likewise,
// dx = g ((y - my) inv_x inv_y - (x - mx) cov inv_x^3 inv_y), dy = g ((x - mx) inv_x inv_y - (y - my) cov inv_x
// inv_y^3), g = grad[row]. Record {n, mean_x, mean_y, M2x, M2y, Cxy}. p = {eps}.
struct WPearson {
    static constexpr int kIn = 2, kOut = 2, kK = 6, kKP = 8;
    static constexpr bool kCol = false, kRowIn = true, kRowOut = false, kI8 = false;
    struct Par {
        float mx, my, inv_xy, cx, cy, g;
    };
    static __device__ void ident(float (&r)[kKP]) {
#pragma unroll
        for (int k = 0; k < kKP; ++k) r[k] = 0.f;
    }
    static __device__ void local(const Team& tm, const Slices<kIn>& sl, float (&r)[kKP], const RwArgs&) {
        float s1[2] = {0.f, 0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 x = sl.ld(0, u), y = sl.ld(1, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) s1[0] += f4(x, j), s1[1] += f4(y, j);
        });
        tm.sum<2>(s1);
        const float cnt = (float)sl.L;
        const float mx = sl.L > 0 ? s1[0] / cnt : 0.f, my = sl.L > 0 ? s1[1] / cnt : 0.f;
        float s[3] = {0.f, 0.f, 0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 x = sl.ld(0, u), y = sl.ld(1, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) {
                    const float dx = f4(x, j) - mx, dy = f4(y, j) - my;
                    s[0] = fmaf(dx, dx, s[0]);
                    s[1] = fmaf(dy, dy, s[1]);
                    s[2] = fmaf(dx, dy, s[2]);
                }
        });
        tm.sum<3>(s);
        r[0] = cnt, r[1] = mx, r[2] = my, r[3] = s[0], r[4] = s[1], r[5] = s[2];
        r[6] = r[7] = 0.f;
    }
    static __device__ void merge(float (&a)[kKP], const float (&b)[kKP]) {
        const float n = a[0] + b[0];
        const float mx = chan_mean(a[0], a[1], b[0], b[1], n), my = chan_mean(a[0], a[2], b[0], b[2], n);
        const float dxa = a[1] - mx, dxb = b[1] - mx, dya = a[2] - my, dyb = b[2] - my;
        const float m2x = (a[3] + b[3]) + (a[0] * dxa * dxa + b[0] * dxb * dxb);
        const float m2y = (a[4] + b[4]) + (a[0] * dya * dya + b[0] * dyb * dyb);
        const float cxy = (a[5] + b[5]) + (a[0] * dxa * dya + b[0] * dxb * dyb);
        a[0] = n, a[1] = mx, a[2] = my, a[3] = m2x, a[4] = m2y, a[5] = cxy;
    }
    static __device__ Par finalize(const float (&t)[kKP], const RwArgs& a, float g) {
        const float inv_x = rsqrtf(fmaxf(t[3], 0.f) + a.p[0]), inv_y = rsqrtf(fmaxf(t[4], 0.f) + a.p[0]);
        const float inv_xy = inv_x * inv_y, cov = t[5];
        return Par{t[1], t[2], inv_xy, cov * inv_x * inv_x * inv_x * inv_y, cov * inv_x * inv_y * inv_y * inv_y, g};
    }
    static __device__ void out(const Par& p, const float4 (&v)[kIn], const float4&, float4 (&o)[kOut]) {
        auto one = [&](float x, float y, float& ox, float& oy) {
            const float xc = x - p.mx, yc = y - p.my;
            ox = p.g * (yc * p.inv_xy - xc * p.cx);
            oy = p.g * (xc * p.inv_xy - yc * p.cy);
        };
        one(v[0].x, v[1].x, o[0].x, o[1].x);
        one(v[0].y, v[1].y, o[0].y, o[1].y);
        one(v[0].z, v[1].z, o[0].z, o[1].z);
        one(v[0].w, v[1].w, o[0].w, o[1].w);
    }
};

// softmax_logits_backward__reduction_reuse__credit.cu:199-236: m = max z, Z = sum exp(z - m), p = exp(z - m)/Z,
// dot = sum p dy, dx = p (dy - dot). Record {m_b, sum exp(z - m_b), sum exp(z - m_b) dy} of the slice, merged by
// rescaling both sums to the larger maximum.
struct WSoftmaxBwd {
    static constexpr int kIn = 2, kOut = 1, kK = 3, kKP = 4;
    static constexpr bool kCol = false, kRowIn = false, kRowOut = false, kI8 = false;
    struct Par {
        float m, inv_sum, dot;
    };
    static __device__ void ident(float (&r)[kKP]) { r[0] = -INFINITY, r[1] = r[2] = r[3] = 0.f; }
    static __device__ void local(const Team& tm, const Slices<kIn>& sl, float (&r)[kKP], const RwArgs&) {
        float m = -INFINITY;
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 z = sl.ld(0, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) m = fmaxf(m, f4(z, j));
        });
        m = tm.max(m);
        float s[2] = {0.f, 0.f};
        if (m != -INFINITY) {
            for_units(tm, sl.L, [&](int u, int n) {
                const float4 z = sl.ld(0, u), dy = sl.ld(1, u);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < n) {
                        const float e = expf(f4(z, j) - m);
                        s[0] += e;
                        s[1] = fmaf(e, f4(dy, j), s[1]);
                    }
            });
        }
        tm.sum<2>(s);
        r[0] = m, r[1] = s[0], r[2] = s[1], r[3] = 0.f;
    }
    static __device__ void merge(float (&a)[kKP], const float (&b)[kKP]) {
        const float m = fmaxf(a[0], b[0]);
        const float fa = a[0] == -INFINITY ? 0.f : expf(a[0] - m), fb = b[0] == -INFINITY ? 0.f : expf(b[0] - m);
        a[1] = a[1] * fa + b[1] * fb;
        a[2] = a[2] * fa + b[2] * fb;
        a[0] = m;
    }
    static __device__ Par finalize(const float (&t)[kKP], const RwArgs&, float) {
        const float inv_sum = 1.0f / t[1];
        return Par{t[0], inv_sum, t[2] * inv_sum};
    }
    static __device__ void out(const Par& p, const float4 (&v)[kIn], const float4&, float4 (&o)[kOut]) {
        auto one = [&](float z, float dy) { return expf(z - p.m) * p.inv_sum * (dy - p.dot); };
        o[0] = make_float4(one(v[0].x, v[1].x), one(v[0].y, v[1].y), one(v[0].z, v[1].z), one(v[0].w, v[1].w));
    }
};

// weighted_var_backward__reduction_reuse__credit.cu:166-220 (backward_value :119-130): inv_sum_w = 1/(sum w + eps),
// mean = sum wx * inv_sum_w, var = max(sum w (x - mean)^2 * inv_sum_w, 0), inv_std = rsqrt(var + eps),
// dx = inv_std (dy - w inv_sum_w sum dy - w (x - mean) inv_std^2 inv_sum_w sum dy (x - mean)).
// Record {W, m, sum w (x - m)^2, sum dy, sum dy (x - m)} with m the slice's weighted mean (weights are
// non-negative variance weights); the reference's eps-shifted mean follows from it exactly. p = {eps}.
struct WWvarBwd {
    static constexpr int kIn = 3, kOut = 1, kK = 5, kKP = 8;
    static constexpr bool kCol = false, kRowIn = false, kRowOut = false, kI8 = false;
    struct Par {
        float mean, inv_sum_w, inv_std, sdy, sdyc;
    };
    static __device__ void ident(float (&r)[kKP]) {
#pragma unroll
        for (int k = 0; k < kKP; ++k) r[k] = 0.f;
    }
    static __device__ void local(const Team& tm, const Slices<kIn>& sl, float (&r)[kKP], const RwArgs&) {
        float s1[2] = {0.f, 0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 x = sl.ld(0, u), w = sl.ld(1, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) {
                    s1[0] += f4(w, j);
                    s1[1] = fmaf(f4(w, j), f4(x, j), s1[1]);
                }
        });
        tm.sum<2>(s1);
        const float W = s1[0], m = W != 0.f ? s1[1] / W : 0.f;
        float s[3] = {0.f, 0.f, 0.f};
        for_units(tm, sl.L, [&](int u, int n) {
            const float4 x = sl.ld(0, u), w = sl.ld(1, u), dy = sl.ld(2, u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < n) {
                    const float d = f4(x, j) - m;
                    s[0] = fmaf(f4(w, j) * d, d, s[0]);
                    s[1] += f4(dy, j);
                    s[2] = fmaf(f4(dy, j), d, s[2]);
                }
        });
        tm.sum<3>(s);
        r[0] = W, r[1] = m, r[2] = s[0], r[3] = s[1], r[4] = s[2];
        r[5] = r[6] = r[7] = 0.f;
    }
    static __device__ void merge(float (&a)[kKP], const float (&b)[kKP]) {
        const float W = a[0] + b[0], m = W != 0.f ? (a[0] * a[1] + b[0] * b[1]) / W : 0.f;
        const float da = a[1] - m, db = b[1] - m;
        const float m2 = (a[2] + b[2]) + (a[0] * da * da + b[0] * db * db);
        const float c = (a[4] + b[4]) + (da * a[3] + db * b[3]);
        a[0] = W, a[1] = m, a[2] = m2, a[3] = a[3] + b[3], a[4] = c;
    }
    static __device__ Par finalize(const float (&t)[kKP], const RwArgs& a, float) {
        const float eps = a.p[0];
        const float inv_sum_w = 1.0f / (t[0] + eps);
        const float mean = t[1] * t[0] * inv_sum_w;   // = sum wx / (sum w + eps)
        const float d = t[1] - mean;
        const float var = fmaxf((t[2] + t[0] * d * d) * inv_sum_w, 0.f);
        return Par{mean, inv_sum_w, rsqrtf(var + eps), t[3], t[4] + d * t[3]};
    }
    static __device__ void out(const Par& p, const float4 (&v)[kIn], const float4&, float4 (&o)[kOut]) {
        const float inv_var = p.inv_std * p.inv_std;
        auto one = [&](float x, float w, float dy) {
            const float c = x - p.mean;
            return p.inv_std * (dy - w * p.inv_sum_w * p.sdy - w * c * inv_var * p.inv_sum_w * p.sdyc);
        };
        o[0] = make_float4(one(v[0].x, v[1].x, v[2].x), one(v[0].y, v[1].y, v[2].y), one(v[0].z, v[1].z, v[2].z),
                           one(v[0].w, v[1].w, v[2].w));
    }
};

// WQuant::local has no RwArgs parameter; give every workload the same call shape.
template <class W>
__device__ __forceinline__ void local_of(const Team& tm, const Slices<W::kIn>& sl, float (&r)[W::kKP], const RwArgs& a) {
    if constexpr (std::is_same<W, WQuant>::value)
        W::local(tm, sl, r);
    else
        W::local(tm, sl, r, a);
}

// st.async of a record of KP floats into CTA q's slot, completing on CTA q's barrier.
template <int KP>
__device__ __forceinline__ void push_rec(uint32_t rd, uint32_t rbar, const float (&r)[KP]) {
    if constexpr (KP == 1) {
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(rd),
                     "r"(__float_as_uint(r[0])), "r"(rbar)
                     : "memory");
    } else if constexpr (KP == 2) {
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1,%2}, [%3];" ::"r"(rd),
                     "f"(r[0]), "f"(r[1]), "r"(rbar)
                     : "memory");
    } else {
#pragma unroll
        for (int j = 0; j < KP; j += 4)
            asm volatile(
                "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1,%2,%3,%4}, [%5];" ::"r"(rd + 4u * j),
                "f"(r[j]), "f"(r[j + 1]), "f"(r[j + 2]), "f"(r[j + 3]), "r"(rbar)
                : "memory");
    }
}

template <class W, int N>
__global__ void __launch_bounds__(kThreadsRw, 2) rowwise_kernel(const __grid_constant__ RwArgs a) {
    constexpr int KP = W::kKP, KIN = W::kIn;
    static_assert(W::kK <= KP && KP <= kMaxKP && (KP == 1 || KP == 2 || KP % 4 == 0), "record padding");
    dsb::Ctx c;
    dsb::ctx_init(c, a.smem_bytes, a.err, a.wait_limit_ns);
    dsb::flag_init(c);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const int tw = a.tw, R = kWarps / tw, nst = a.stages, nsets = a.sets;
    const int slice = a.slice, cols = a.cols;
    const int start = (int)c.rank * slice;
    const int L = max(0, min(slice, cols - start));   // this CTA's columns of every row
    const uint32_t arrivals = a.vec ? 1u : 32u;      // plain copies: every producer lane arrives
    const uint32_t row_bytes = (uint32_t)slice * 4u;
    const long long nclu = (long long)num_clusters(), cq = (long long)cluster_id();
    const long long groups = (a.rows + R - 1) / R;
    const long long iters = groups > cq ? (groups - cq + nclu - 1) / nclu : 0;
    auto group_row0 = [&](long long i) { return (cq + i * nclu) * R; };
    // stage s, input k, row r of the group
    auto slice_off = [&](int s, int k, int r) {
        return a.stage_off + (uint32_t)s * a.stage_bytes + ((uint32_t)k * R + (uint32_t)r) * row_bytes;
    };
    if (warp == kProducer && lane == 0) {
        for (int s = 0; s < nst; ++s) mbar_init(c.bar(kFull + s), arrivals);
        mbar_init(c.bar(kColBar), arrivals);
        fence_mbar_init();
    } else if (warp == 0) {
        if (lane < (uint32_t)nst) mbar_init(c.bar(kEmpty + (int)lane), kWarps);
        if (lane < (uint32_t)a.sets) mbar_init(c.bar(kExch + (int)lane), 1);
        fence_mbar_init();
    }
    __syncthreads();
    // every CTA's barriers initialised (released cluster-wide) before a peer's record can land on them; the
    // producer waits only after its loop, so the first loads overlap the rendezvous
    cluster_arrive();
    c.deadline = globaltimer() + c.wait_limit;

    if (warp == kProducer) {
        // ------------------------------------------------------------------------------ producer warp
        if (W::kCol) {
            const float* src = a.col + start;
            const uint32_t dst = a.col_off;
            if (a.vec) {
                if (lane == 0) {
                    dsb::arm(c, kColBar, (uint32_t)L * 4u);
                    if (L > 0) bulk_load_g2s(c.sa + dst, src, (uint32_t)L * 4u, c.bar(kColBar));
                }
            } else {
                for (int e = (int)lane; e < L; e += 32) c.ptr<float>(dst)[e] = src[e];
                mbar_arrive(c.bar(kColBar));
            }
        }
        for (long long i = 0; i < iters; ++i) {
            c.deadline = globaltimer() + c.wait_limit;
            const int s = (int)(i % nst);
            const long long round = i / nst;
            if (round > 0) wait_par(c, kEmpty + s, (uint32_t)((round - 1) & 1));
            __syncwarp();
            const long long r0 = group_row0(i);
            const int nrows = (int)max(0LL, min((long long)R, a.rows - r0));
            if (a.vec) {
                if (lane == 0) {
                    dsb::arm(c, kFull + s, (uint32_t)(nrows * KIN * L) * 4u);
                    if (L > 0)
                        for (int r = 0; r < nrows; ++r)
#pragma unroll
                            for (int k = 0; k < KIN; ++k)
                                bulk_load_g2s(c.sa + slice_off(s, k, r), a.in[k] + (size_t)(r0 + r) * cols + start,
                                              (uint32_t)L * 4u, c.bar(kFull + s));
                }
            } else {
                for (int r = 0; r < nrows; ++r)
#pragma unroll
                    for (int k = 0; k < KIN; ++k) {
                        const float* src = a.in[k] + (size_t)(r0 + r) * cols + start;
                        float* dst = c.ptr<float>(slice_off(s, k, r));
                        for (int e = (int)lane; e < L; e += 32) dst[e] = src[e];
                    }
                mbar_arrive(c.bar(kFull + s));   // each lane releases its own copies
            }
        }
        __syncwarp();
        cluster_wait();
    } else {
        cluster_wait();
        // ------------------------------------------------------------------------------ row teams
        Team tm;
        tm.warp = warp, tm.lane = lane, tm.tw = (uint32_t)tw, tm.team = warp / (uint32_t)tw;
        tm.tt = (warp % (uint32_t)tw) * 32u + lane, tm.TT = (uint32_t)tw * 32u, tm.c = &c;
        const uint32_t rec_bytes = (uint32_t)(N * R * KP) * 4u;
        auto slot_off = [&](int set, int rank, int r) {
            return kSlotsOff + ((uint32_t)((set * N + rank) * R + r) * KP) * 4u;
        };
        auto slices = [&](int s) {
            Slices<KIN> sl;
#pragma unroll
            for (int k = 0; k < KIN; ++k) sl.s[k] = c.ptr<const float>(slice_off(s, k, (int)tm.team));
            sl.col = c.ptr<const float>(a.col_off);
            sl.L = L;
            return sl;
        };
        if (W::kCol) wait_par(c, kColBar, 0);
        // statistics of group i: the team's record of its row goes to every CTA of the cluster
        auto stats = [&](long long i) {
            const int s = (int)(i % nst), set = (int)(i % nsets);
            wait_par(c, kFull + s, (uint32_t)((i / nst) & 1));
            const long long row = group_row0(i) + tm.team;
            Slices<KIN> sl = slices(s);
            if (row >= a.rows) sl.L = 0;   // a row past the end sends the identity record
            float r[KP];
            W::ident(r);
            local_of<W>(tm, sl, r, a);
            if (warp == 0 && lane == 0) dsb::arm(c, kExch + set, rec_bytes);
            if (tm.tt < (uint32_t)N) {
                const uint32_t q = tm.tt;
                push_rec<KP>(mapa(c.sa + slot_off(set, (int)c.rank, (int)tm.team), q), mapa(c.bar(kExch + set), q), r);
            }
        };
        // outputs of group i: merge the N records of the team's row, then the output pass over the stage
        auto outputs = [&](long long i) {
            const int s = (int)(i % nst), set = (int)(i % nsets);
            wait_par(c, kExch + set, (uint32_t)((i / nsets) & 1));
            float t[KP];
            W::ident(t);
            if (lane < (uint32_t)N) {
                const float* src = c.ptr<const float>(slot_off(set, (int)lane, (int)tm.team));
#pragma unroll
                for (int k = 0; k < KP; ++k) t[k] = src[k];
            }
#pragma unroll
            for (int off = N / 2; off > 0; off >>= 1) {
                float o[KP];
#pragma unroll
                for (int k = 0; k < KP; ++k) o[k] = __shfl_xor_sync(0xffffffffu, t[k], off);
                W::merge(t, o);
            }
#pragma unroll
            for (int k = 0; k < KP; ++k) t[k] = __shfl_sync(0xffffffffu, t[k], 0);
            const long long row = group_row0(i) + tm.team;
            if (row < a.rows) {
                const float rin = W::kRowIn ? a.rowin[row] : 0.f;
                const typename W::Par p = W::finalize(t, a, rin);
                if constexpr (W::kRowOut) {
                    if (c.rank == 0 && tm.tt == 0) a.rowout[row] = W::row_out(p);
                }
                const Slices<KIN> sl = slices(s);
                const size_t base = (size_t)row * cols + start;
                for_units(tm, L, [&](int u, int n) {
                    float4 v[KIN], o[W::kOut];
#pragma unroll
                    for (int k = 0; k < KIN; ++k) v[k] = sl.ld(k, u);
                    const float4 cv = W::kCol ? sl.ldc(u) : make_float4(0.f, 0.f, 0.f, 0.f);
                    W::out(p, v, cv, o);
                    if constexpr (W::kI8) {
                        signed char* dst = static_cast<signed char*>(a.out[0]) + base + 4 * u;
                        if (n == 4 && a.vec) {
                            const uint32_t w = ((uint32_t)(uint8_t)(signed char)o[0].x) |
                                               ((uint32_t)(uint8_t)(signed char)o[0].y << 8) |
                                               ((uint32_t)(uint8_t)(signed char)o[0].z << 16) |
                                               ((uint32_t)(uint8_t)(signed char)o[0].w << 24);
                            __stcs(reinterpret_cast<unsigned*>(dst), w);
                        } else {
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                if (j < n) dst[j] = (signed char)f4(o[0], j);
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < W::kOut; ++k) {
                            float* dst = static_cast<float*>(a.out[k]) + base + 4 * u;
                            if (n == 4 && a.vec) {
                                __stcs(reinterpret_cast<float4*>(dst), o[k]);
                            } else {
#pragma unroll
                                for (int j = 0; j < 4; ++j)
                                    if (j < n) dst[j] = f4(o[k], j);
                            }
                        }
                    }
                });
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(c.bar(kEmpty + s));   // the stage's rows are consumed
        };
        // Teams run D = a.ahead groups ahead (D <= 1 and D <= stages - 1): iteration i sends group i+D's
        // records, then computes group i's outputs, so an exchange is in flight while a group's outputs are
        // written. Progress: group i+D's stage is loaded once group i+D-stages is consumed, and D <= stages - 1
        // puts that in an earlier iteration. (Deeper look-ahead measured slower on B200: the stages held for
        // pending outputs are stages not loading.) Slot-set reuse: a team sends exchange e only after its outputs(e-D-1), i.e. after its wait for e-D-1,
        // which needed every team of every CTA to send e-D-1; each of those sent it only after reading exchange
        // e-2D-2 (its outputs(e-2D-2)). So when e's records reach a CTA, that CTA's exchange e-2D-2 is complete
        // and read, only e-2D-1 .. e-1 may still be in use, and 2D+2 sets keep them apart (the barrier of e's
        // set has finished the phase of e-2D-2 for the same reason).
        const long long D = a.ahead;
        for (long long j = 0; j < D && j < iters; ++j) {
            c.deadline = globaltimer() + c.wait_limit;
            stats(j);
        }
        for (long long i = 0; i < iters; ++i) {
            c.deadline = globaltimer() + c.wait_limit;
            c.unit = (uint32_t)i;
            if (i + D < iters) stats(i + D);
            outputs(i);
        }
    }
    dsb::finish(c);   // no CTA leaves while a peer may still store into its slots
}

// ------------------------------------------------------------------------------------------- host side
struct RwKey {
    const void* fn;
    int dev;
    uint32_t smem;
    bool operator<(const RwKey& o) const {
        return fn < o.fn || (fn == o.fn && (dev < o.dev || (dev == o.dev && smem < o.smem)));
    }
};
std::mutex g_mu;
std::map<RwKey, int> g_occ;
unsigned* g_err[64] = {};

template <class W>
const void* rw_fn(int n) {
    switch (n) {
        case 1: return reinterpret_cast<const void*>(&rowwise_kernel<W, 1>);
        case 2: return reinterpret_cast<const void*>(&rowwise_kernel<W, 2>);
        case 4: return reinterpret_cast<const void*>(&rowwise_kernel<W, 4>);
        case 8: return reinterpret_cast<const void*>(&rowwise_kernel<W, 8>);
        case 16: return reinterpret_cast<const void*>(&rowwise_kernel<W, 16>);
    }
    return nullptr;
}

constexpr uint32_t kSmemPerSm = 233472;   // 228 KiB of shared memory per SM (1 KiB reserved per CTA)

// Launch geometry of a workload: slice, team width, ring depth and the shared-memory layout: at most 4
// 16-byte units per lane per pass (the team width grows with the slice), two CTAs per SM with at least two
// stages each when they fit (else one CTA with as many stages as fit), one group of look-ahead when there are
// two or more stages.
template <class W>
dsmem_status rw_plan(int cols, int n, RwArgs& a) {
    const int slice = ((cols + n - 1) / n + 3) / 4 * 4;
    const int units = slice / 4;
    int tw = 1;
    while (tw < kWarps && units > tw * 32 * 4) tw *= 2;
    const int R = kWarps / tw;
    const uint32_t row_bytes = (uint32_t)slice * 4u;
    const uint32_t stage_bytes = (uint32_t)W::kIn * R * row_bytes;
    const int sets = 2 * kMaxAhead + 2;
    const uint32_t col_off = align128(kSlotsOff + rw_slots_bytes(sets, n, R, W::kKP));
    const uint32_t stage_off = align128(col_off + (W::kCol ? row_bytes : 0u));
    auto smem = [&](int st) { return stage_off + (uint32_t)st * stage_bytes; };
    int st = kMaxStages;
    while (st > 2 && 2u * (smem(st) + 1024u) > kSmemPerSm) --st;
    if (2u * (smem(st) + 1024u) > kSmemPerSm) {
        st = kMaxStages;
        while (st > 1 && smem(st) > dsb::kSmemLimit) --st;
        if (smem(st) > dsb::kSmemLimit) return DSMEM_ERR_SMEM_LIMIT;
    }
    a.slice = slice;
    a.tw = tw;
    a.stages = st;
    a.ahead = std::min(kMaxAhead, st - 1);
    a.sets = sets;
    a.col_off = col_off;
    a.stage_off = stage_off;
    a.stage_bytes = stage_bytes;
    a.smem_bytes = smem(st);
    return DSMEM_OK;
}

template <class W>
dsmem_status rw_launch(RwArgs a, const void* const* arrays, int narrays, long long rows, int cols, int n,
                       cudaStream_t stream) {
    if (rows < 0 || cols <= 0) return DSMEM_ERR_INVALID_ARGUMENT;
    if (!(n == 1 || n == 2 || n == 4 || n == 8 || n == 16)) return DSMEM_ERR_INVALID_ARGUMENT;
    for (int k = 0; k < narrays; ++k)
        if (arrays[k] == nullptr) return DSMEM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DSMEM_OK;
    a.rows = rows;
    a.cols = cols;
    const dsmem_status ps = rw_plan<W>(cols, n, a);
    if (ps != DSMEM_OK) return ps;
    uintptr_t al = 0;
    for (int k = 0; k < narrays; ++k) al |= reinterpret_cast<uintptr_t>(arrays[k]);
    a.vec = (cols % 4 == 0 && (al & 15u) == 0) ? 1 : 0;
    const void* fn = rw_fn<W>(n);
    int dev = 0;
    if (fn == nullptr) return DSMEM_ERR_ILLEGAL_CONFIG;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSMEM_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreadsRw, 1, 1);
    cfg.dynamicSmemBytes = a.smem_bytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int resident = 0;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_err[dev] == nullptr) {   // error bits, timeout detail, cluster id, spare
            if (cudaMalloc(&g_err[dev], 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
            if (cudaMemset(g_err[dev], 0, 4 * sizeof(unsigned)) != cudaSuccess) return DSMEM_ERR_CUDA;
        }
        if (dsb_attr::ensure_smem(fn, dev, a.smem_bytes, n > 8) != cudaSuccess) return DSMEM_ERR_CUDA;
        const RwKey key{fn, dev, a.smem_bytes};
        auto it = g_occ.find(key);
        if (it == g_occ.end()) {
            cfg.gridDim = dim3((unsigned)n, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&resident, fn, &cfg) != cudaSuccess) return DSMEM_ERR_CUDA;
            g_occ[key] = resident;
        } else {
            resident = it->second;
        }
        a.err = g_err[dev];
    }
    if (resident < 1) return DSMEM_ERR_SMEM_LIMIT;
    const long long groups = (rows + (kWarps / a.tw) - 1) / (kWarps / a.tw);
    const long long clusters = std::min<long long>(groups, resident);
    cfg.gridDim = dim3((unsigned)(clusters * n), 1, 1);
    a.wait_limit_ns = 1000000000ull;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? DSMEM_OK : DSMEM_ERR_CUDA;
}

RwArgs blank() {
    RwArgs a;
    memset(&a, 0, sizeof a);
    return a;
}

}  // namespace

extern "C" {

dsmem_status dsmem_rowwise_quant_launch(const float* x, int8_t* q, float* scales, long long rows, int cols,
                                        int cluster_size, dsmem_stream_t stream) {
    RwArgs a = blank();
    a.in[0] = x;
    a.out[0] = q;
    a.rowout = scales;
    const void* arr[] = {x, q, scales};
    return rw_launch<WQuant>(a, arr, 3, rows, cols, cluster_size, reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_lars_momentum_launch(const float* weight, const float* grad, const float* momentum,
                                        float* weight_out, float* momentum_out, long long rows, int cols,
                                        float momentum_coeff, float weight_decay, float lr, float trust_coeff,
                                        float eps, int cluster_size, dsmem_stream_t stream) {
    RwArgs a = blank();
    a.in[0] = weight, a.in[1] = grad, a.in[2] = momentum;
    a.out[0] = weight_out, a.out[1] = momentum_out;
    a.p[0] = momentum_coeff, a.p[1] = weight_decay, a.p[2] = lr, a.p[3] = trust_coeff, a.p[4] = eps;
    const void* arr[] = {weight, grad, momentum, weight_out, momentum_out};
    return rw_launch<WLars>(a, arr, 5, rows, cols, cluster_size, reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_layernorm_backward_launch(const float* x, const float* dy, const float* gamma, float* dx,
                                             long long rows, int cols, float eps, int cluster_size,
                                             dsmem_stream_t stream) {
    RwArgs a = blank();
    a.in[0] = x, a.in[1] = dy;
    a.col = gamma;
    a.out[0] = dx;
    a.p[0] = eps;
    const void* arr[] = {x, dy, gamma, dx};
    return rw_launch<WLnBwd>(a, arr, 4, rows, cols, cluster_size, reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_pearson_backward_launch(const float* x, const float* y, const float* grad, float* dx, float* dy,
                                           long long rows, int cols, float eps, int cluster_size,
                                           dsmem_stream_t stream) {
    RwArgs a = blank();
    a.in[0] = x, a.in[1] = y;
    a.rowin = grad;
    a.out[0] = dx, a.out[1] = dy;
    a.p[0] = eps;
    const void* arr[] = {x, y, grad, dx, dy};
    return rw_launch<WPearson>(a, arr, 5, rows, cols, cluster_size, reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_softmax_logits_backward_launch(const float* logits, const float* dy, float* dx, long long rows,
                                                  int cols, int cluster_size, dsmem_stream_t stream) {
    RwArgs a = blank();
    a.in[0] = logits, a.in[1] = dy;
    a.out[0] = dx;
    const void* arr[] = {logits, dy, dx};
    return rw_launch<WSoftmaxBwd>(a, arr, 3, rows, cols, cluster_size, reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_weighted_var_backward_launch(const float* x, const float* weights, const float* dy, float* dx,
                                                long long rows, int cols, float eps, int cluster_size,
                                                dsmem_stream_t stream) {
    RwArgs a = blank();
    a.in[0] = x, a.in[1] = weights, a.in[2] = dy;
    a.out[0] = dx;
    a.p[0] = eps;
    const void* arr[] = {x, weights, dy, dx};
    return rw_launch<WWvarBwd>(a, arr, 4, rows, cols, cluster_size, reinterpret_cast<cudaStream_t>(stream));
}

dsmem_status dsmem_rowwise_query(int workload, int cols, int cluster_size, size_t* smem_bytes, int* rows_per_group,
                                 int* stages, int* ahead) {
    if (cols <= 0 || !(cluster_size == 1 || cluster_size == 2 || cluster_size == 4 || cluster_size == 8 ||
                       cluster_size == 16))
        return DSMEM_ERR_INVALID_ARGUMENT;
    RwArgs a = blank();
    dsmem_status s;
    switch (workload) {
        case 0: s = rw_plan<WQuant>(cols, cluster_size, a); break;
        case 1: s = rw_plan<WLars>(cols, cluster_size, a); break;
        case 2: s = rw_plan<WLnBwd>(cols, cluster_size, a); break;
        case 3: s = rw_plan<WPearson>(cols, cluster_size, a); break;
        case 4: s = rw_plan<WSoftmaxBwd>(cols, cluster_size, a); break;
        case 5: s = rw_plan<WWvarBwd>(cols, cluster_size, a); break;
        default: return DSMEM_ERR_INVALID_ARGUMENT;
    }
    if (s != DSMEM_OK) return s;
    if (smem_bytes) *smem_bytes = a.smem_bytes;
    if (rows_per_group) *rows_per_group = kWarps / a.tw;
    if (stages) *stages = a.stages;
    if (ahead) *ahead = a.ahead;
    return DSMEM_OK;
}

dsmem_status dsmem_rowwise_check(int device, unsigned* error_bits) {
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
