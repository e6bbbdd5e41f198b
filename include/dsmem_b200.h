/*
 * dsmem_b200.h -- C ABI of the B200 (sm_100a) thread-block-cluster collective catalogue.
 *
 * The reference repository (lomolisso/h100-dsmem-collectives) has no library interface: each
 * algorithm is a compile-time plugin, collectives/<op>__<alg>__<src>.cu, that defines
 *     __global__ void __cluster_dims__(CLUSTER_N,1,1)
 *     collective_kernel(const ELEM_T* in, ELEM_T* out, unsigned long long* ts, unsigned* smid);
 * (contract: collectives/dsmem_primitives.cuh:205-220), compiled once per (file, CLUSTER_N, MSG_ELEMS,
 * ELEM_T) and launched by collectives/harness/main.cu:267-275 as ONE cluster per launch. This header
 * replaces that compile-time selection with run-time arguments: one call launches a batch of
 * `num_clusters` independent problems, each exactly the reference kernel's problem, on resident
 * persistent clusters. Plain pointers and sizes only; no CUDA or torch types in the signatures
 * (dsmem_stream_t is ABI-identical to cudaStream_t).
 *
 * Data layout of a batch (cluster problem c, rank b, M = elements per rank block, cluster-major):
 *   ALLREDUCE      in [c][b][M]            out[c][b][M]     (main.cu:132-136)
 *   ALLGATHER      in [c][b][M]            out[c][b][N][M]  (main.cu:137-138)
 *   REDUCESCATTER  in [c][b][N][M]         out[c][b][M]     (main.cu:139-142)
 *   ALLTOALL       in [c][b][N][M]         out[c][b][N][M]  (main.cu:143-145)
 *   BROADCAST, REDUCE in [c][b][M]         out[c][b][M]     (rooted at rank 0, no reference file)
 *   GATHER         in [c][b][M]            out[c][b][N][M]  (rooted at rank 0, no reference file)
 *   SCATTER        in [c][b][N][M]         out[c][b][M]     (rooted at rank 0, no reference file)
 * bytes_per_cta is the nccl-tests payload P of the reference sweep (main.cu:97, driver.py:156-163):
 *   ALLREDUCE (and BROADCAST, REDUCE) P = M * sizeof(T); every other op P = N * M * sizeof(T).
 */
#ifndef DSMEM_B200_H
#define DSMEM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st* dsmem_stream_t; /* == cudaStream_t */

/* Return codes. ILLEGAL_CONFIG mirrors the reference build matrix's SKIP:static_assert and
 * SMEM_LIMIT its SKIP:smem (collectives/harness/driver.py:210-230, main.cu:90-92); TIMEOUT replaces
 * the reference watchdog's DEADLOCK exit (main.cu:277-320): a device-side mbarrier wait gave up. */
typedef enum {
    DSMEM_OK = 0,
    DSMEM_ERR_ILLEGAL_CONFIG = 1,
    DSMEM_ERR_SMEM_LIMIT = 2,
    DSMEM_ERR_TIMEOUT = 3,
    DSMEM_ERR_CUDA = 4,
    DSMEM_ERR_INVALID_ARGUMENT = 5,
    DSMEM_ERR_BOUNDS = 6,
    DSMEM_ERR_NCCL = 7,
    DSMEM_ERR_SCRATCH_LIMIT = 8
} dsmem_status;

/* COLL_OP values of collectives/harness/main.cu:7-8. */
typedef enum {
    DSMEM_OP_ALLREDUCE = 0,
    DSMEM_OP_ALLGATHER = 1,
    DSMEM_OP_REDUCESCATTER = 2,
    DSMEM_OP_ALLTOALL = 3,
    /* B200 extension, no reference file: broadcast of rank 0's vector (M elements per rank in and out;
     * P = M * sizeof(T) as for allreduce), algorithms DIRECT_PUSH, DIRECT_PULL and BINOMIAL. */
    DSMEM_OP_BROADCAST = 4,
    /* B200 extensions, no reference file: the other collectives rooted at rank 0, algorithms DIRECT_PUSH,
     * DIRECT_PULL and BINOMIAL each.
     *   REDUCE   in M elements per rank, out M per rank; rank 0's out = op over the ranks' vectors (P = M *
     *            sizeof(T), as for allreduce). The other ranks' out blocks are not written.
     *   GATHER   in M per rank, out N * M per rank; rank 0's out = the ranks' vectors in rank order (P = N * M *
     *            sizeof(T), as for allgather). The other ranks' out blocks are not written.
     *   SCATTER  in N * M per rank, of which only rank 0's is read; out M per rank: rank r gets block r of rank
     *            0's input (P = N * M * sizeof(T), as for reducescatter). */
    DSMEM_OP_REDUCE = 5,
    DSMEM_OP_GATHER = 6,
    DSMEM_OP_SCATTER = 7
} dsmem_op;

/* The <alg> component of the reference file names collectives/<op>__<alg>__<src>.cu
 * (collectives/README.md:19-49). Not every algorithm exists for every op. */
typedef enum {
    DSMEM_ALG_AUTO = 0,                               /* measured table, else a built-in default */
    DSMEM_ALG_RING = 1,                               /* allreduce, allgather, reducescatter     */
    DSMEM_ALG_RECURSIVE_DOUBLING = 2,                 /* allreduce, allgather                    */
    DSMEM_ALG_SHIFT_ACCUMULATE_BULK = 3,              /* allreduce (N = 4)                       */
    DSMEM_ALG_SHIFT_ACCUMULATE_ATOMIC = 4,            /* allreduce (N = 2, 4)                    */
    DSMEM_ALG_DIRECT_REPLICATED_PUSH = 5,             /* allreduce, allgather                    */
    DSMEM_ALG_PULL_REDUCE_SCATTER_PUSH_ALLGATHER = 6, /* allreduce                               */
    DSMEM_ALG_RABENSEIFNER = 7,                       /* allreduce                               */
    DSMEM_ALG_ONE_SHOT_PULL = 8,                      /* allreduce                               */
    DSMEM_ALG_TWO_SHOT_PUSH = 9,                      /* allreduce                               */
    DSMEM_ALG_REDUCE_BCAST_BINOMIAL = 10,             /* allreduce                               */
    DSMEM_ALG_ATOMIC_ALL_PUSH = 11,                   /* allreduce                               */
    DSMEM_ALG_2D_MESH = 12,                           /* allreduce                               */
    DSMEM_ALG_DIRECT_SHIFT = 13,                      /* allgather                               */
    DSMEM_ALG_BRUCK = 14,                             /* allgather, alltoall                     */
    DSMEM_ALG_DIRECT_PULL = 15,                       /* allgather, reducescatter, alltoall, rooted */
    DSMEM_ALG_GATHER_BCAST_BINOMIAL = 16,             /* allgather                               */
    DSMEM_ALG_RECURSIVE_HALVING = 17,                 /* reducescatter                           */
    DSMEM_ALG_DIRECT_PUSH = 18,                       /* reducescatter, alltoall, rooted         */
    DSMEM_ALG_PAIRWISE_EXCHANGE = 19,                 /* alltoall (N = 2)                        */
    DSMEM_ALG_PAIRWISE_XOR = 20,                      /* alltoall                                */
    DSMEM_ALG_SHIFT = 21,                             /* alltoall                                */
    /* B200 extension, no reference file: allreduce whose reduce-scatter shot (the two-shot's first) runs
     * over DSMEM and whose all-gather goes straight into the N output rows (half the SM-to-SM bytes). */
    DSMEM_ALG_RS_PUSH_GLOBAL_AG = 22,                 /* allreduce                               */
    /* B200 extensions, no reference file: the ring (N <= 8) and recursive-doubling AllReduce schedules with
     * a buffer and an mbarrier per round instead of a barrier.cluster per round (the "DSMEM-native"
     * variants the reference defers, collectives/ROADMAP.md:38-45); same arithmetic as the originals. */
    DSMEM_ALG_RING_CREDIT = 23,                       /* allreduce (N <= 8), allgather, reducescatter */
    DSMEM_ALG_RECURSIVE_DOUBLING_CREDIT = 24,         /* allreduce, allgather                    */
    DSMEM_ALG_BINOMIAL = 25,                          /* broadcast, reduce, gather, scatter      */
    DSMEM_ALG_BRUCK_CREDIT = 26,                      /* allgather, alltoall                     */
    DSMEM_ALG_RECURSIVE_HALVING_CREDIT = 27,          /* reducescatter                           */
    /* B200 extensions, no reference file: more of the deferred mbarrier-credit forms (same rounds, partners
     * and arithmetic as the originals, no barrier.cluster between rounds). */
    DSMEM_ALG_RABENSEIFNER_CREDIT = 28,               /* allreduce                               */
    DSMEM_ALG_PAIRWISE_XOR_CREDIT = 29,               /* alltoall                                */
    DSMEM_ALG_BINOMIAL_CREDIT = 30,                   /* allreduce (reduce + broadcast), allgather (gather + broadcast) */
    DSMEM_ALG_SHIFT_ACCUMULATE_BULK_CREDIT = 31,      /* allreduce (N = 4)                       */
    DSMEM_ALG_COUNT = 32
} dsmem_alg;

/* ELEM_T of the reference (float | int, main.cu:99) plus bf16. */
typedef enum { DSMEM_F32 = 0, DSMEM_BF16 = 1, DSMEM_I32 = 2 } dsmem_dtype;

/* Error bits of the device error word (dsmem_last_error). */
#define DSMEM_ERRBIT_TIMEOUT 1u
#define DSMEM_ERRBIT_BOUNDS 2u

/*
 * Launch one collective on `num_clusters` independent cluster problems (stream-ordered, asynchronous).
 * Replaces: compiling collectives/<op>__<alg>__<src>.cu with -DCLUSTER_N -DMSG_ELEMS -DELEM_T
 * (collectives/harness/driver.py:233-239) and launching collective_kernel<<<N, 256, smem>>>
 * (collectives/harness/main.cu:267-275), once per problem.
 *   cluster_size   N in {2, 4, 8, 16} (16 is a non-portable cluster size)
 *   bytes_per_cta  P, see the header comment
 *   in, out        device pointers, 16-byte aligned, sizes per the batch layout above
 *   stamps         nullable; else [num_clusters][N][32] u64 %globaltimer slots per problem:
 *                  [0] entry, [1] exit, [2 + r] end of round r (dsmem_primitives.cuh:216-218)
 *   stream         CUDA stream (NULL = legacy default stream)
 * Returns ILLEGAL_CONFIG for (op, alg, N, P, dtype) combinations the reference rejects by static_assert,
 * SMEM_LIMIT when the algorithm's shared memory exceeds 227 KiB per CTA, CUDA on launch failure.
 * Device-side timeouts are reported by dsmem_last_error / dsmem_check, not by this call.
 */
dsmem_status dsmem_collective_launch(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                     size_t bytes_per_cta, const void* in, void* out, int num_clusters,
                                     unsigned long long* stamps, dsmem_stream_t stream);

/* As dsmem_collective_launch, plus SM ids ([num_clusters][N] u32, nullable: main.cu's smid array),
 * and an explicit cap on resident clusters (0 = as many as fit). */
dsmem_status dsmem_collective_launch_ex(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                        size_t bytes_per_cta, const void* in, void* out, long long num_clusters,
                                        unsigned long long* stamps, unsigned* smid, int max_resident_clusters,
                                        dsmem_stream_t stream);

/* The same batch on HOST buffers, synchronous: in and out are host memory (page-locked for overlap; pageable
 * works, slower), laid out as for dsmem_collective_launch; on return out holds the results. The batch streams
 * through double-buffered device staging in chunks of chunk_clusters problems (0: about 64 MiB per chunk):
 * the host-to-device copy of chunk i+1, the collective on chunk i and the device-to-host copy of chunk i-1
 * overlap on three streams. AUTO is resolved once for the whole batch. Device errors as dsmem_check. For
 * REDUCE and GATHER only rank 0's out block of each problem is copied back; the other blocks of out keep their
 * contents. The host-side counterpart of the reference harness's reference() on host arrays (main.cu:129-149). */
dsmem_status dsmem_collective_host(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                   size_t bytes_per_cta, const void* host_in, void* host_out, long long num_clusters,
                                   long long chunk_clusters);

/* Static legality and shared-memory size of a configuration (the reference build matrix's
 * classification, driver.py:210-230, and the COLLECTIVE_SMEM_BYTES tag, main.cu:104-121).
 * legal = 1 if the configuration runs; smem_bytes = dynamic shared memory per CTA. */
dsmem_status dsmem_query(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta,
                         size_t* smem_bytes, int* legal);

/* Resident clusters of one launch on the current device (cudaOccupancyMaxActiveClusters,
 * main.cu:215-222) for a legal configuration. */
dsmem_status dsmem_max_active_clusters(dsmem_op op, dsmem_alg alg, dsmem_dtype dtype, int cluster_size,
                                       size_t bytes_per_cta, int* clusters);

/* Variant selection for DSMEM_ALG_AUTO: a measured table of lines "op cluster_size bytes_per_cta dtype alg"
 * (names as in dsmem_alg_name / dsmem_op_name). A lookup takes the entry with the same op, N and dtype
 * and the largest bytes_per_cta <= the request. Replaces the "best per (op, N, payload)" selection of
 * collectives/analysis/collectives_figures.py:549. */
dsmem_status dsmem_autotune_table_load(const char* path);
/* The algorithm AUTO resolves to (after legality) for this configuration. */
dsmem_alg dsmem_autotune_pick(dsmem_op op, dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta);
/* The algorithm AUTO runs for a launch of num_clusters problems: the table's `batch` regime (throughput)
 * when num_clusters > 1, its `single` regime (latency, the reference harness's one cluster per launch)
 * otherwise, each falling back to the other and then to the built-in order. Table lines are
 * "op cluster_size bytes_per_cta dtype alg [single|batch]" (default single); the table measured on B200
 * (h100-dsmem-collectives_b200/autotune_b200.tsv, next to lib/) is loaded on first use unless
 * DSMEM_AUTOTUNE_TABLE names another file (empty: none) or dsmem_autotune_table_load ran first. */
dsmem_alg dsmem_autotune_pick_ex(dsmem_op op, dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta,
                                 long long num_clusters);

/* Read and clear the device error word of `device` (synchronises that device). The word is shared by every
 * catalogue launch on the device, from any stream or host thread: a read reports the errors of all launches
 * since the previous read. Each word is read and cleared in one atomic exchange, so a bit set while the read
 * runs is either returned or kept for the next read, never lost. */
dsmem_status dsmem_last_error(int device, unsigned* error_bits);
/* As dsmem_last_error, plus where the first timed-out wait since the last read gave up:
 * detail = 0x80000000 | barrier << 24 | cluster rank << 16 | problem-or-unit counter (low 16 bits),
 * 0 if no wait timed out; cluster = its %clusterid.x. Any pointer may be NULL. No reference
 * counterpart (the reference's hangs end in its host watchdog, collectives/harness/main.cu:277-320). */
dsmem_status dsmem_last_error_detail(int device, unsigned* error_bits, unsigned* detail, unsigned* cluster);
/* Synchronise `stream`, then map the device error word to TIMEOUT / BOUNDS (and clear it); as above, the word
 * also carries errors of launches on other streams since the last read. */
dsmem_status dsmem_check(dsmem_stream_t stream);

/* Names: "<op>", "<alg>" and the reference file stem "<op>__<alg>__<src>". */
const char* dsmem_op_name(dsmem_op op);
const char* dsmem_alg_name(dsmem_alg alg);
const char* dsmem_dtype_name(dsmem_dtype dtype);
const char* dsmem_status_string(dsmem_status status);
/* Reference file stem of (op, alg), or NULL if the pair does not exist. */
const char* dsmem_file_stem(dsmem_op op, dsmem_alg alg);
/* Parse a reference file stem (e.g. "allreduce__ring__nccl"); returns INVALID_ARGUMENT if unknown. */
dsmem_status dsmem_lookup(const char* file_stem, dsmem_op* op, dsmem_alg* alg);

/* Per-device wait limit of the batch kernels in nanoseconds of %globaltimer (default 1e9). */
dsmem_status dsmem_set_wait_limit_ns(unsigned long long ns);

/* Batches of more than one problem run on a pipelined driver where the algorithm has one (two-shot
 * AllReduce: bulk HBM loads/stores overlapped with the shots, no per-problem cluster barrier). 0 forces
 * the plain driver (load, entry barrier, collective, store, exit barrier per problem). Default 1. */
dsmem_status dsmem_set_pipelined(int enable);
/* Largest sub-vector per CTA the pipelined drivers stream at once (256 B .. 64 KiB, multiple of 16;
 * default 16 KiB). Larger problems are split into equal legal sub-vectors no larger than this. */
dsmem_status dsmem_set_pipeline_unit_bytes(size_t bytes);
/* The streamed batch driver of rs_push_global_ag (reduce-scatter over DSMEM, all-gather through the
 * outputs; warp-specialised, an input ring and a slot ring): largest sub-vector per CTA (256 B .. 64 KiB,
 * multiple of 16), input stages `depth` (2..8; 0: by cluster size) and slot stages `lag` = units of
 * reduce-scatter in flight (1 .. depth-1); depth - lag loads stream in meanwhile; fewer stages where the window
 * does not fit. Results do not depend on these. Defaults (also restored by (0, 0, 0)), measured on B200: 16 KiB
 * units, 3 input stages at cluster size 8 and 2 otherwise, 1 slot stage; launches of at most one wave
 * (clusters x N <= SM count) take 32 KiB units, 4 input stages and 3 slot stages. */
dsmem_status dsmem_set_stream_pipeline(size_t unit_bytes, int depth, int lag);

/* Failure-detection self-test: launches one 2-CTA cluster whose mbarrier is armed for 16 bytes that
 * never arrive, with a wait limit of `limit_ns`; every wait gives up after the limit and the kernel
 * exits normally. dsmem_check afterwards must report DSMEM_ERR_TIMEOUT. Replaces nothing in the
 * reference (its hangs were caught by a host watchdog, collectives/harness/main.cu:277-320). */
dsmem_status dsmem_selftest_timeout(unsigned long long limit_ns, dsmem_stream_t stream);

/*
 * Cluster-fused RMSNorm: y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w, fp32 statistics, bf16 or f32 in/out.
 * Row r is split across a cluster of `cluster_size` CTAs (1, 2, 4, 8, 16; hidden/cluster_size elements per
 * CTA, a multiple of 16 bytes and at most 2 KiB), whose partial sums of squares meet in a DSMEM AllReduce.
 * Replaces RMSNormKernel of kernels/rmsnorm__llama__clusterfusion.cu:35-108 (called as
 * clusterfusion.rmsnorm(x, w), roofline/harness/workloads/clusterfusion_rmsnorm.py:50), generalised from
 * fp16 / 64 x 8192 / cluster 2 compiled in to run-time dtype, shape and cluster size.
 * x, y: [rows][hidden] row-major, 16-byte aligned; w: [hidden].
 */
dsmem_status dsmem_rmsnorm_launch(dsmem_dtype dtype, const void* x, const void* w, float eps, long long rows,
                                  int hidden, int cluster_size, void* y, dsmem_stream_t stream);

/* As dsmem_rmsnorm_launch on h = x + residual (rounded to dtype), written to pre_norm (nullable) -- the
 * RMSNorm half of hpc-ops' fused AllReduce+RMSNorm, kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197
 * (outputPreNorm / outputNorm, :182-187 / :179-196). */
dsmem_status dsmem_rmsnorm_residual_launch(dsmem_dtype dtype, const void* x, const void* residual, const void* w,
                                           float eps, long long rows, int hidden, int cluster_size, void* pre_norm,
                                           void* y, dsmem_stream_t stream);

/* Read and clear the RMSNorm kernels' device error word of `device` (synchronous). */
dsmem_status dsmem_rmsnorm_check(int device, unsigned* error_bits);

/*
 * Row-wise reduction-reuse workloads (fp32, [rows][cols] row-major): a cluster of `cluster_size` CTAs
 * (1, 2, 4, 8, 16) per row, CTA b staging column slice b (ceil(cols / cluster_size) rounded up to 4
 * elements) in shared memory, and ONE DSMEM exchange per row of a mergeable statistics record. Each
 * replaces the clustered kernel of kernels/<name>__reduction_reuse__credit.cu, whose launch is one
 * cluster of P CTAs per row (gridDim = rows * P, slice_elems = the column slice) and whose statistics
 * take 1-3 replicated-push AllReduce stages of two cluster barriers each. Arrays 16-byte aligned with
 * cols % 4 == 0 take bulk copies and vector stores; other shapes take per-element copies (same results).
 * DSMEM_ERR_SMEM_LIMIT when one row slice of every input exceeds the 227 KiB per CTA (the reference
 * declares the same shapes invalid). Device errors (bounded waits) are read by dsmem_rowwise_check.
 */
/* rowwise_quant__reduction_reuse__credit.cu:104-155 (cluster_quant_staged_kernel): amax = max |x| of the
 * row, q = clamp(nearbyint(x * (127 / amax)), -127, 127) (0 for an all-zero row), scales[row] = amax / 127. */
dsmem_status dsmem_rowwise_quant_launch(const float* x, int8_t* q, float* scales, long long rows, int cols,
                                        int cluster_size, dsmem_stream_t stream);
/* lars_momentum__reduction_reuse__credit.cu:126-185 (cluster_lars_staged_kernel): u = momentum_coeff * m +
 * g + weight_decay * w, trust = trust_coeff * ||w|| / (||u|| + eps) over the row, w_out = w - lr * trust * u,
 * m_out = u. The reference compiles in 0.9, 0.01, 1e-3, 0.02, 1e-6 (:29-33). */
dsmem_status dsmem_lars_momentum_launch(const float* weight, const float* grad, const float* momentum,
                                        float* weight_out, float* momentum_out, long long rows, int cols,
                                        float momentum_coeff, float weight_decay, float lr, float trust_coeff,
                                        float eps, int cluster_size, dsmem_stream_t stream);
/* layernorm_backward__reduction_reuse__credit.cu:119-186 (cluster_bwd_staged_kernel): dx of LayerNorm
 * given x, dy and gamma [cols] (mean and biased variance of x over the row; eps inside the rsqrt). */
dsmem_status dsmem_layernorm_backward_launch(const float* x, const float* dy, const float* gamma, float* dx,
                                             long long rows, int cols, float eps, int cluster_size,
                                             dsmem_stream_t stream);
/* pearson_backward__reduction_reuse__credit.cu:158-227 (cluster_bwd_staged_kernel): dx, dy of the Pearson
 * correlation of rows x, y given the upstream gradient grad[rows]. */
dsmem_status dsmem_pearson_backward_launch(const float* x, const float* y, const float* grad, float* dx, float* dy,
                                           long long rows, int cols, float eps, int cluster_size,
                                           dsmem_stream_t stream);
/* softmax_logits_backward__reduction_reuse__credit.cu:164-237 (cluster_softmax_logits_bwd_staged_kernel):
 * dx = p * (dy - sum(p * dy)) with p = softmax(logits) over the row. */
dsmem_status dsmem_softmax_logits_backward_launch(const float* logits, const float* dy, float* dx, long long rows,
                                                  int cols, int cluster_size, dsmem_stream_t stream);
/* weighted_var_backward__reduction_reuse__credit.cu:135-221 (cluster_bwd_staged_kernel): dx of the weighted
 * variance (non-negative weights; the reference compiles in eps = 1e-6, :29). */
dsmem_status dsmem_weighted_var_backward_launch(const float* x, const float* weights, const float* dy, float* dx,
                                                long long rows, int cols, float eps, int cluster_size,
                                                dsmem_stream_t stream);
/* Read and clear the row-wise kernels' device error word of `device` (synchronous). */
dsmem_status dsmem_rowwise_check(int device, unsigned* error_bits);
/* Launch plan of a row-wise workload (0 quant, 1 LARS, 2 LayerNorm backward, 3 Pearson backward, 4 softmax
 * backward, 5 weighted-variance backward) at `cols` columns: dynamic shared memory per CTA, rows per group,
 * ring stages and groups of look-ahead; SMEM_LIMIT where the launch would return it. No device call. */
dsmem_status dsmem_rowwise_query(int workload, int cols, int cluster_size, size_t* smem_bytes, int* rows_per_group,
                                 int* stages, int* ahead);

/*
 * Exact top-k indices of every row of fp32 logits ([rows][n] row-major, 16-byte aligned base; any n): for
 * each row the indices (0..n-1) of its k largest values, written to out_indices[row][0..k) in an unspecified
 * order; among equal values at the cut, lower ranks' segments are taken first (+NaN ranks above +inf, -NaN
 * below -inf; all NaNs of a sign are equal). A cluster
 * of cluster_size CTAs (2, 4, 8, 16) per row; each stages a contiguous segment of ceil(n / cluster_size)
 * elements in shared memory (DSMEM_ERR_SMEM_LIMIT above about 200 KiB per segment); the radix select's
 * 2048-bin histograms meet in a two-shot DSMEM AllReduce. Replaces topk_filtered_cluster8_exact_kernel of
 * kernels/topk_filtered_cluster8__llm_sampling__hpcops.cu (hpc.topk(logits, ke, out, ...) with k = 2048 at
 * cluster 8), generalised to any k <= n and cluster size. 1 <= k <= n.
 */
dsmem_status dsmem_topk_launch(const float* logits, long long rows, int n, int k, int32_t* out_indices,
                               int cluster_size, dsmem_stream_t stream);
/* Read and clear the top-k kernel's device error word of `device` (synchronous). */
dsmem_status dsmem_topk_check(int device, unsigned* error_bits);
/* Dynamic shared memory per CTA of a top-k launch over rows of n (SMEM_LIMIT where the launch would return it).
 * No device call. */
dsmem_status dsmem_topk_query(int n, int cluster_size, size_t* smem_bytes);

/* SM-to-SM bandwidth ceiling (the DSMEM roofline denominator). Replaces the reference's microbenchmark
 * roofline/harness/ceilings/src/dsmem_bw.cu:1-40 (ops `ld` and `tma_put`, ring +1, max active clusters,
 * 96 KiB per pass): mode 0 pull (ld.shared::cluster.v4), 1 push (cp.async.bulk) to the ring neighbour,
 * 2 push to every peer (8 KiB per peer per pass, 4 KiB at cluster size 16; the fan-out pattern of the direct
 * and two-shot algorithms, which the reference did not measure). ctas_per_sm 1 is the reference's shape
 * (96 KiB tiles, 1024 threads, one CTA per SM); 4 uses 24 KiB tiles and 256 threads so clusters of 8/16
 * also occupy the SMs that one-CTA-per-SM placement leaves idle. Times `reps` launches of `passes` passes;
 * the caller fits 1/slope over several pass counts. */
dsmem_status dsmem_ceiling_dsmem_bw(int mode, int cluster_size, int ctas_per_sm, int passes, int reps,
                                    double* ms_median, long long* bytes_per_launch, int* clusters);

/*
 * Ceilings beyond DSMEM and HBM, for hierarchical rooflines (the reference's ceiling suite,
 * roofline/harness/ceilings and roofline/docs/DESIGN.md:28-48, measures DSMEM and HBM on H100; these are
 * sm_100a additions). Each returns the median event time of `reps` launches and the work of one launch;
 * the caller fits 1 / slope over two or more work amounts.
 *   dsmem_ceiling_tcgen05: one CTA per SM issues iters x 4 tcgen05.mma kind::f16 (M = 128, N = n in
 *     {64, 128, 256}, K = 16, bf16 operands in shared memory, fp32 accumulator in TMEM); flops = 2*M*N*K
 *     per instruction.
 *   dsmem_ceiling_l2_bw: a full grid reads a `bytes` buffer (it should fit the L2) `passes` times with
 *     16-byte L2 loads.
 *   dsmem_ceiling_smem_bw: one CTA per SM (1024 threads) reads a 96 KiB shared-memory tile `passes` times.
 */
dsmem_status dsmem_ceiling_tcgen05(int n, int iters, int reps, double* ms_median, double* flops_per_launch,
                                   int* ctas);
dsmem_status dsmem_ceiling_l2_bw(long long bytes, int passes, int reps, double* ms_median, double* bytes_per_launch);
dsmem_status dsmem_ceiling_smem_bw(int passes, int reps, double* ms_median, double* bytes_per_launch);

/*
 * Batch two-shot AllReduce that allocates no device memory. No counterpart in the reference (whose
 * harness allocates every buffer itself). dsmem_collective_launch allocates a device error word on its
 * first call per device; some callers cannot let a library do that: a framework whose caching allocator
 * has reserved the GPU's memory up front and accounts for every byte, or a program with a fixed memory map
 * in which nothing is allocated after start-up. This entry point keeps its scratch (error word + one status
 * word per cluster problem) in a fixed static device array of 4 * (64 + 65536) bytes, resident on every
 * GPU that loads the library until the process exits.
 *   Same result, bit for bit, as dsmem_collective_launch(DSMEM_OP_ALLREDUCE, DSMEM_ALG_TWO_SHOT_PUSH, ...)
 *   on the same arguments with the plain driver (dsmem_set_pipelined(0)): same shots, same summation order.
 *   num_clusters <= DSMEM_NOALLOC_MAX_PROBLEMS, else DSMEM_ERR_SCRATCH_LIMIT before anything is launched.
 *   status_out: host array of num_clusters words or NULL. If given, the call synchronises `stream`,
 *   copies each problem's error bits (DSMEM_ERRBIT_*) there and returns TIMEOUT/BOUNDS if any bit is set;
 *   if NULL the call returns right after the launch.
 *   num_clusters == 0 launches nothing; with status_out given, it synchronises `stream`, writes the previous
 *   call's device error bits to status_out[0] and returns TIMEOUT/BOUNDS/OK from them (how a caller that
 *   passed NULL learns of a device-side error).
 *   The first call on a device is its set-up, made with that device current: it looks up the array's
 *   device address and resolves all twelve kernels (3 dtypes x 4 cluster sizes), so the CUDA runtime loads
 *   their code then and not on a later call; make that first call before any stream capture. All calls
 *   share the array (cleared per call on `stream`); calls whose kernels overlap on the GPU race on it.
 */
#define DSMEM_NOALLOC_MAX_PROBLEMS 65536
dsmem_status dsmem_allreduce_two_shot_noalloc(dsmem_dtype dtype, int cluster_size, size_t bytes_per_cta,
                                              const void* in, void* out, int num_clusters, unsigned* status_out,
                                              dsmem_stream_t stream);

/*
 * Tensor-parallel AllReduce + RMSNorm across the GPUs of one node (one process per
 * GPU). y = RMSNorm(sum over ranks of x_rank (+ residual)) * w on every rank, bf16, fp32 sum and
 * statistics. Replaces the AllReduce + RMSNorm pipeline of
 * kernels/rmsnorm_lamport__fused_allreduce_rmsnorm__hpcops.cu:37-197 (which the reference declares but
 * never ran, roofline/.../hpcops_rmsnorm_lamport.yaml:35-50) with one fused kernel per rank over NVLink
 * peer memory, in one of two forms:
 *   two-shot  reduce-scatter by rows with peer loads, the cluster RMSNorm of the owned rows (DSMEM
 *             partial-sum push), all-gather by peer stores; 2 (tp-1)/tp of the tensor crosses NVLink each way;
 *   one-shot  (small tensors) every rank pushes its x into every peer's LL region (8-byte words of 4 data
 *             bytes and the call's epoch, polled by the receiver: no flags, no round trip) and reduces and
 *             normalises every row itself; (tp-1) * rows * hidden * 4 bytes leave each rank.
 * Both sum the ranks in rank order in fp32 and give the same bits when the residual is the same tensor on
 * every rank (a replicated residual stream, as in a TP decoder; the two-shot adds the residual of the row's
 * owning rank, the one-shot each rank's own). Set-up, per rank:
 *   dsmem_tp_alloc   allocate this rank's buffer (signals + x region + y region, capacity bytes each, and
 *                    an LL region of 2 x 8 slots of min(2 capacity, 4 MiB)) and return its CUDA IPC handle
 *                    (DSMEM_TP_HANDLE_BYTES) to share with the other ranks;
 *   dsmem_tp_open    map every rank's buffer (handles: tp handles in rank order);
 *   dsmem_tp_buffers the x and y regions: a producer may write x there and a consumer read y there, which
 *                    saves the copies that dsmem_tp_allreduce_rmsnorm makes for other pointers.
 * dsmem_tp_allreduce_rmsnorm: x (NULL: already in the x region) [rows x hidden]; residual (nullable) and
 * w local; y (NULL: leave in the y region). Every rank calls it with the same shape, in the same order;
 * cross-GPU waits are bounded (2 s) and report DSMEM_ERR_TIMEOUT through dsmem_tp_check. The one-shot form
 * runs when tp > 1, rows * hidden * 4 fits one LL slot and (tp - 1) * rows * hidden * 4 <= the context's
 * one-shot limit (dsmem_tp_set_oneshot_limit); it reads x and writes y in place (no copies).
 * Shapes: hidden a multiple of 8 * cluster_size, at most 2 KiB of a row per CTA; rows*hidden*2 <= capacity
 * (else DSMEM_ERR_SCRATCH_LIMIT). tp in {1, 2, 4, 8}.
 */
#define DSMEM_TP_HANDLE_BYTES 64
typedef struct dsmem_tp_ctx* dsmem_tp_t;
dsmem_status dsmem_tp_alloc(size_t capacity_bytes, dsmem_tp_t* ctx, void* ipc_handle);
dsmem_status dsmem_tp_open(dsmem_tp_t ctx, int rank, int tp, const void* handles);
dsmem_status dsmem_tp_buffers(dsmem_tp_t ctx, void** x, void** y, size_t* capacity_bytes);
dsmem_status dsmem_tp_allreduce_rmsnorm(dsmem_tp_t ctx, dsmem_dtype dtype, const void* x, const void* residual,
                                        const void* w, float eps, long long rows, int hidden, int cluster_size,
                                        void* y, dsmem_stream_t stream);
/* Read and clear the context's device error words (synchronous): TIMEOUT / BOUNDS / OK; detail as in
 * dsmem_last_error_detail (barrier 0x70 + r: entry wait for rank r, or the one-shot's wait for rank r's
 * data; 0x78 + r: exit wait). */
dsmem_status dsmem_tp_check(dsmem_tp_t ctx, unsigned* error_bits, unsigned* detail);
/* Limit of each cross-GPU flag wait of this context's calls (default 2 s; 1 ns .. 60 s). A call whose peer
 * never joins gives up after it (at entry, and again at exit), finishes without blocking, and dsmem_tp_check
 * reports DSMEM_ERR_TIMEOUT. After a timeout the ranks' call epochs disagree: close and reopen the context.
 * Replaces the reference's host watchdog (collectives/harness/main.cu:277-320) for the cross-GPU path. */
dsmem_status dsmem_tp_set_wait_limit_ns(dsmem_tp_t ctx, unsigned long long ns);
/* The one-shot form's limit on the LL bytes a rank sends per call, (tp - 1) * rows * hidden * 4 (default
 * 16 MiB; 0: always the two-shot; SIZE_MAX: the one-shot whenever the tensor fits an LL slot). */
dsmem_status dsmem_tp_set_oneshot_limit(dsmem_tp_t ctx, size_t bytes);
dsmem_status dsmem_tp_close(dsmem_tp_t ctx);
/* The same kernel for `tp` ranks emulated in one launch on one GPU (xs, ys: tp local buffers each; every
 * row computed once and written to all tp y buffers; no flags). For single-GPU parity tests. */
dsmem_status dsmem_tp_emulate(int tp, const void* const* xs, void* const* ys, dsmem_dtype dtype, const void* residual,
                              const void* w, float eps, long long rows, int hidden, int cluster_size,
                              dsmem_stream_t stream);
/* The one-shot kernel for `tp` ranks on one GPU: every rank's push launched first (into LL regions on this
 * GPU), then every rank's reduction into its own ys[r]; no launch waits for another. */
dsmem_status dsmem_tp_emulate_oneshot(int tp, const void* const* xs, void* const* ys, dsmem_dtype dtype,
                                      const void* residual, const void* w, float eps, long long rows, int hidden,
                                      int cluster_size, dsmem_stream_t stream);
/* Read and clear the emulation entry points' device error words (synchronous), as dsmem_tp_check. */
dsmem_status dsmem_tp_emulate_check(unsigned* error_bits, unsigned* detail);

/*
 * The NCCL composition (the baseline of the fused kernel, and the configs[4] pipeline as the reference
 * describes it): ncclAllReduce(bf16, sum) of x into `sum`, then dsmem_rmsnorm(_residual)_launch of sum.
 * comm is an ncclComm_t; NCCL is resolved at run time from the process (libnccl.so.2). The helpers make a
 * communicator for callers without one (uid: 128 bytes, an ncclUniqueId, shared by the caller).
 */
typedef void* dsmem_nccl_comm_t;
dsmem_status dsmem_nccl_unique_id(void* uid);
dsmem_status dsmem_nccl_comm_init(int world, int rank, const void* uid, dsmem_nccl_comm_t* comm);
dsmem_status dsmem_nccl_comm_destroy(dsmem_nccl_comm_t comm);
dsmem_status dsmem_tp_allreduce_rmsnorm_nccl(dsmem_nccl_comm_t comm, dsmem_dtype dtype, const void* x,
                                             const void* residual, const void* w, float eps, long long rows,
                                             int hidden, int cluster_size, void* sum, void* y, dsmem_stream_t stream);

/*
 * Llama-2-7B-shaped decoder layer, one decode step. Replaces the fused layer of
 * kernels/fused_decoder_layer__llama2_7b__clusterfusion.cu:291-922 (ClusterFusion's
 * llama_decoder_layer_sglang: fp16, batch 1, attention block only) with the whole layer for a batch of
 * 1..16 sequences, bf16, and the maths of roofline/harness/workloads/clusterfusion_llama2_7b_decoder.py:160-180:
 *   x = inp + res; xn = RMSNorm(x) w_rms; q, k, v = xn Wqkv^T (rows q | k | v, head-major); NEOX RoPE on q
 *   and k with the given cos/sin [head_dim] (fp32); k, v stored at token index seq_len of the caches;
 *   a = softmax(q K^T / sqrt(head_dim)) V over seq_len + 1 tokens; o = a Wo^T; h = x + o;
 *   hn = RMSNorm(h) w_post; out = (SiLU(hn Wg^T) * hn Wu^T) Wd^T with Wgu = [Wg; Wu] ([2 ffn][hidden]).
 * Shapes: head_dim 128, hidden = heads * 128, ffn a multiple of 64 and of 32 * cluster_size, cluster_size
 * 4 or 8 (the CTAs of a cluster split each projection's K dimension and each sequence-head's keys).
 * Caches [batch][cache_capacity][heads][head_dim] bf16, seq_len < cache_capacity. All tensors bf16
 * except cos/sin; weights in nn.Linear layout [out][in]. Outputs: out [batch][hidden] (layer output),
 * h_out [batch][hidden] (the residual stream after attention), o_out (nullable, the attention-block
 * output), k_new / v_new (nullable, [batch][heads][head_dim]). The caller owns a workspace of
 * dsmem_decoder_workspace_bytes(batch, hidden, ffn) bytes. Five stream-ordered launches; asynchronous.
 */
typedef struct {
    int batch, hidden, heads, head_dim, ffn;
    long long seq_len, cache_capacity;
    int cluster_size;
    float eps;
    const void *inp, *res, *w_rms, *wqkv, *wo, *w_post, *wgu, *wd;
    void *kcache, *vcache;
    const float *cos, *sin;
    void* workspace;
    size_t workspace_bytes;
    void *out, *h_out, *o_out, *k_new, *v_new;
} dsmem_decoder_params;
size_t dsmem_decoder_workspace_bytes(int batch, int hidden, int ffn);
dsmem_status dsmem_decoder_layer_launch(const dsmem_decoder_params* params, dsmem_stream_t stream);
/* Read and clear the decoder kernels' device error word of `device` (synchronous). */
dsmem_status dsmem_decoder_check(int device, unsigned* error_bits);

/* Library version string. */
const char* dsmem_version(void);

#ifdef __cplusplus
}
#endif
#endif /* DSMEM_B200_H */
