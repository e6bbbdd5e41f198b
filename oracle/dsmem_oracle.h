/*
 * dsmem_oracle.h -- CPU oracle for the DSMEM collective catalogue and its consumers.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library; the product (h100-dsmem-collectives_b200/) never does.
 *
 * Restates, in plain C, the host side of the reference harness collectives/harness/main.cu:
 *   fill_input()  main.cu:118-126   (patterns A and B)
 *   reference()   main.cu:129-149   (double / int64 accumulation over the layouts of
 *                                    collectives/dsmem_primitives.cuh:209-213)
 *   check()       main.cu:156-173   (exact or 1e-5*(1+|ref|)*ceil(log2 N))
 * extended to batches of independent cluster problems (cluster-major layout of include/dsmem_b200.h)
 * and to bf16 elements, plus the RMSNorm formula of roofline/harness/workloads/clusterfusion_rmsnorm.py:65.
 * Parity is pinned by golden vectors produced by the reference's own fill_input()/reference()
 * compiled from the reference sources (oracle/Makefile, target `ref`; fixtures in tests/golden/).
 */
#ifndef DSMEM_ORACLE_H
#define DSMEM_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_BF16 = 1, ORC_I32 = 2 };
/* 4..7 are B200 extensions with no reference file (rooted at rank 0): broadcast, reduce, gather, scatter. */
enum {
    ORC_ALLREDUCE = 0, ORC_ALLGATHER = 1, ORC_REDUCESCATTER = 2, ORC_ALLTOALL = 3, ORC_BROADCAST = 4, ORC_REDUCE = 5,
    ORC_GATHER = 6, ORC_SCATTER = 7
};

/* mt19937_64 (Matsumoto & Nishimura 2000), the engine of the reference's pattern B. */
typedef struct {
    uint64_t mt[312];
    int idx;
} orc_mt64;
void orc_mt64_seed(orc_mt64* g, uint64_t seed);
uint64_t orc_mt64_next(orc_mt64* g);
/* libstdc++ uniform_real_distribution<double>(lo, hi) on mt19937_64: (hi-lo)*canonical + lo, where
 * canonical = (double)g() / 2^64 (values that round to 1 become the largest double below 1). */
double orc_uniform_real(orc_mt64* g, double lo, double hi);
/* Uniform integer in [lo, hi] by Lemire's multiply-shift rejection method (ACM TOMACS 29(1), 2019)
 * on 64-bit draws, the method libstdc++'s uniform_int_distribution uses for mt19937_64. */
int64_t orc_uniform_int(orc_mt64* g, int64_t lo, int64_t hi);

/* bf16 <-> float (round to nearest even). */
uint16_t orc_f32_to_bf16(float x);
float orc_bf16_to_f32(uint16_t h);

/* Pattern A (main.cu:119): in[k] = T((k*7+3) % 17 - 8) over the whole array. */
void orc_fill_pattern_a(int dtype, void* buf, size_t n);
/* Pattern B (main.cu:121-124): mt19937_64(20261025), U(-1,1) in double, converted to the element type. */
void orc_fill_pattern_b(int dtype, void* buf, size_t n);
/* Seeded draws of the benchmark configurations: U(lo,hi) (float types) from mt19937_64(seed). */
void orc_fill_uniform_real(int dtype, void* buf, size_t n, uint64_t seed, double lo, double hi);
/* Seeded integer draws U[lo, hi] into int32 from mt19937_64(seed). */
void orc_fill_uniform_int(int32_t* buf, size_t n, uint64_t seed, int64_t lo, int64_t hi);
/* Seeded N(mean, std) draws (Box-Muller on two canonical doubles), converted to the element type. */
void orc_fill_normal(int dtype, void* buf, size_t n, uint64_t seed, double mean, double std);

/* Element counts per rank of one cluster problem. */
size_t orc_in_elems(int op, int n, size_t m);
size_t orc_out_elems(int op, int n, size_t m);

/* main.cu:129-149 for `clusters` independent problems: ref (double) has clusters*N*out_elems entries. */
void orc_reference(int op, int dtype, int n, size_t m, long long clusters, const void* in, double* ref);

/* main.cu:156-173. mode 0: exact in the element type (got == T(ref)); mode 1: |got-ref| <= tol*(1+|ref|).
 * Returns the number of bad elements; max_abs / max_rel (err/(1+|ref|)) may be NULL. */
long long orc_check(int dtype, size_t n, const void* out, const double* ref, int mode, double tol, double* max_abs,
                    double* max_rel);

/* RMSNorm oracle (clusterfusion_rmsnorm.py:65 in double): y = x * 1/sqrt(mean(x^2) + eps) * w per row;
 * x [rows][hidden], w [hidden] in dtype (F32 or BF16); y in double. If `res` is non-NULL the row is
 * h = x + res first (rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:8-9), and h (double) is
 * written to pre (if non-NULL). */
void orc_rmsnorm(int dtype, size_t rows, size_t hidden, const void* x, const void* res, const void* w, double eps,
                 double* y, double* pre);

/* Tensor-parallel AllReduce + RMSNorm oracle: h = sum over ranks of xs[k] (+ res), in double, then the
 * RMSNorm above (clusterfusion_rmsnorm.py:65) of h; xs: `ranks` arrays [rows][hidden]; y in double. */
void orc_tp_rmsnorm(int dtype, size_t ranks, size_t rows, size_t hidden, const void* const* xs, const void* res,
                    const void* w, double eps, double* y);

/* Decoder layer oracle (clusterfusion_llama2_7b_decoder.py:160-180, reference_fp32 with the FFN tail) in
 * double: bf16 inputs and weights, no intermediate rounding. Caches [batch][cap][heads][head_dim] with
 * seq_len valid tokens; the new k, v are the step's own (RoPE on q and k with cos/sin [head_dim]).
 * Outputs [batch][hidden] (k_new / v_new [batch][heads*head_dim]; any output pointer but out may be NULL). */
void orc_decoder_layer(int batch, int hidden, int heads, int head_dim, int ffn, long long seq_len, long long cap,
                       const uint16_t* inp, const uint16_t* res, const uint16_t* w_rms, const uint16_t* wqkv,
                       const uint16_t* wo, const uint16_t* w_post, const uint16_t* wgu, const uint16_t* wd,
                       const uint16_t* kc, const uint16_t* vc, const float* cosv, const float* sinv, double eps,
                       double* out, double* h_out, double* o_out, double* k_new, double* v_new);

/* Sum of `ranks` arrays of bf16/f32 (TP all-reduce input), in double. */
void orc_sum_ranks(int dtype, size_t ranks, size_t n, const void* const* xs, double* out);

/* Row-wise reduction-reuse workloads: the formulas of the clustered kernels of
 * kernels/<name>__reduction_reuse__credit.cu over fp32 [rows][cols] inputs, row statistics accumulated in
 * double in the reference's own stage order (one-pass variance where the reference uses it). */
/* rowwise_quant :129-153 -- in fp32 exactly as the kernel computes it (max is order-free, so this is bit-exact):
 * amax = max |x| (from 0, NaN ignored), inv = 127/amax (0 if amax == 0), q = clamp(nearbyint(x*inv), -127, 127),
 * scale = amax/127. */
void orc_rowwise_quant(size_t rows, size_t cols, const float* x, int8_t* q, float* scales);
/* The element formula alone (quantize_to_i8, rowwise_quant :100-105). */
int orc_quantize_i8(float value, float inv_scale);
/* lars_momentum :160-184 (update_value :120-124). */
void orc_lars_momentum(size_t rows, size_t cols, const float* w, const float* g, const float* m, double mu,
                       double wd, double lr, double eta, double eps, double* w_out, double* m_out);
double orc_lars_update(double w, double g, double m, double mu, double wd);
/* layernorm_backward :146-185. */
void orc_layernorm_backward(size_t rows, size_t cols, const float* x, const float* dy, const float* gamma,
                            double eps, double* dx);
/* pearson_backward :187-226. */
void orc_pearson_backward(size_t rows, size_t cols, const float* x, const float* y, const float* grad, double eps,
                          double* dx, double* dy);
/* softmax_logits_backward :199-236. */
void orc_softmax_logits_backward(size_t rows, size_t cols, const float* z, const float* dy, double* dx);
/* weighted_var_backward :166-220 and its element formula backward_value :119-130. */
void orc_weighted_var_backward(size_t rows, size_t cols, const float* x, const float* w, const float* dy,
                               double eps, double* dx);
double orc_wvar_backward_value(double value, double weight, double grad, double mean, double inv_sum_w,
                               double inv_std, double sum_dy, double sum_dy_centered);
/* Exact top-k (hpc-ops topk_filtered, validated in its tests against torch.topk): the k largest values of each
 * row, sorted descending, into vals[rows][k]. +NaN ranks above +inf (torch's order); -NaN below -inf (the
 * sign-respecting key order of the kernels' key transform; torch would rank it first as well). */
void orc_topk_values(size_t rows, size_t n, size_t k, const float* x, float* vals);

#ifdef __cplusplus
}
#endif
#endif
