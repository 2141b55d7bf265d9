/*
 * gafime_b200.h -- C ABI of libgafime_cuda.so, the B200 (sm_100a) engine for
 * GAFIME's all-pairs scoring path.
 *
 * Every symbol the reference's loaders bind on this path keeps its exact name,
 * signature, status codes and ownership rules (reference: src/common/interfaces.h),
 * so gafime/backends/native_cuda_backend.py and the Rust libloading callers can
 * load this library in place of the reference's libgafime_cuda.so.  New entry
 * points (all-pairs scoring, sharding, top-k merge) are marked NEW.
 *
 * Conventions (interfaces.h:32-38, kernels.cu:886-889):
 *   - every function returns int: 0 success, negative GAFIME_ERROR_* on failure;
 *     no C++ exception crosses the ABI;
 *   - handles are opaque, owned by the library from *_alloc until *_free, and
 *     *_free(NULL) succeeds;
 *   - host pointers are borrowed for the duration of the call only;
 *   - calls are synchronous: results are in the caller's buffers on return.
 *   - a bucket remembers the CUDA device that was current at *_alloc and makes it
 *     current for every later call on that bucket (the reference always used the
 *     current device, kernels.cu:129-131).
 */
#ifndef GAFIME_B200_H
#define GAFIME_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes -- interfaces.h:32-38 */
#define GAFIME_SUCCESS 0
#define GAFIME_ERROR_INVALID_ARGS -1
#define GAFIME_ERROR_CUDA_NOT_AVAILABLE -2
#define GAFIME_ERROR_OUT_OF_MEMORY -3
#define GAFIME_ERROR_KERNEL_FAILED -4
#define GAFIME_ERROR_PIPELINE_FULL -5
#define GAFIME_ERROR_NO_RESULT -6

/* Unary operators -- interfaces.h:57-73 */
#define GAFIME_OP_IDENTITY 0
#define GAFIME_OP_LOG 1
#define GAFIME_OP_EXP 2
#define GAFIME_OP_SQRT 3
#define GAFIME_OP_TANH 4
#define GAFIME_OP_SIGMOID 5
#define GAFIME_OP_SQUARE 6
#define GAFIME_OP_NEGATE 7
#define GAFIME_OP_ABS 8
#define GAFIME_OP_INVERSE 9
#define GAFIME_OP_CUBE 10
#define GAFIME_OP_ROLLING_MEAN 11
#define GAFIME_OP_ROLLING_STD 12

/* Interaction types -- interfaces.h:83-88 */
#define GAFIME_INTERACT_MULT 0
#define GAFIME_INTERACT_ADD 1
#define GAFIME_INTERACT_SUB 2
#define GAFIME_INTERACT_DIV 3
#define GAFIME_INTERACT_MAX 4
#define GAFIME_INTERACT_MIN 5

/* 12-float stats layout -- interfaces.h:110-123 */
#define GAFIME_STATS_SIZE 12

/* NEW: metric ids, same numbering as gafime_core's MetricId (gafime_core.cpp:28-33) */
#define GAFIME_METRIC_PEARSON 0
#define GAFIME_METRIC_MUTUAL_INFO 2
/* NEW -- no counterpart in the reference (its bins are equal-width only).  Mutual information
 * with QUANTILE bins on the interaction: the cut points of a pair are the order statistics
 * sorted[floor(b n / mi_bins)], b = 1 .. mi_bins-1, of its n values, a value's bin is the
 * number of cut points <= it; y is binned equal-width as for GAFIME_METRIC_MUTUAL_INFO.
 * Exact (one device sort per pair), so much slower than the equal-width mode.  Accepted by
 * gafime_allpairs_topk / _topk_host / _topk_device / _scores wherever a metric is. */
#define GAFIME_METRIC_MUTUAL_INFO_QUANTILE 12

/* NEW: largest k the all-pairs top-k returns per operator */
#define GAFIME_ALLPAIRS_MAX_K 4096

typedef void* ContiguousBucket; /* interfaces.h:42 */

/* ---------------------------------------------------------------- device ---- */

/* interfaces.h:133 -- 1 when a CUDA device is usable, else 0. */
int gafime_cuda_available(void);

/* interfaces.h:144-150 -- name (>= 256 chars), total memory in MB, compute capability. */
int gafime_get_device_info(int device_id, char* name_out, int* memory_mb_out,
                           int* compute_cap_major_out, int* compute_cap_minor_out);

/* interfaces.h:167-175 -- launch geometry of the current device. */
int gafime_get_gpu_config(int* block_size_out, int* max_blocks_out, int* sm_count_out,
                          int* compute_major_out, int* compute_minor_out,
                          int* l2_cache_bytes_out, char* gpu_name_out);

/* interfaces.h:607 -- 1 and *precision_mode = 4 (tcgen05 f16/bf16/tf32) on sm_100. */
int gafime_tensor_core_available(int* precision_mode);

/* NEW: make device_id current for the calling thread (cudaSetDevice). */
int gafime_select_device(int device_id);

/* ------------------------------------------------------- contiguous bucket ---- */

/* interfaces.h:513-517 -- one device buffer for F feature columns + the target,
 * column-major, plus a uint8 fold mask.  Rows are padded to a multiple of 256 on
 * the device (zeros) so every tile of the all-pairs kernels is full. */
int gafime_contiguous_bucket_alloc(int n_samples, int n_features, ContiguousBucket* bucket_out);

/* interfaces.h:522-526 -- h_data = [F0 | F1 | ... | F_{F-1} | y], (F+1)*n floats,
 * column-major; h_mask = n bytes (may not be NULL, as in the reference). */
int gafime_contiguous_bucket_upload(ContiguousBucket bucket, const float* h_data,
                                    const uint8_t* h_mask);

/* interfaces.h:531-540 -- 12 stats of x = combine(op_a(F_a), op_b(F_b)), split by
 * mask == val_fold_id.  Rows with NaN x or y are skipped (cpu_backend.cpp:274).
 * Sums are accumulated in fp64 in a fixed order (deterministic), then cast to
 * float for this float* output. */
int gafime_contiguous_bucket_compute(ContiguousBucket bucket, int feature_a_idx,
                                     int feature_b_idx, int op_a, int op_b,
                                     int interact_type, int val_fold_id, float* h_stats_out);

/* interfaces.h:545 */
int gafime_contiguous_bucket_free(ContiguousBucket bucket);

/* interfaces.h:550-554 */
int gafime_contiguous_bucket_info(ContiguousBucket bucket, int* n_samples_out,
                                  int* n_features_out);

/* interfaces.h:392-401 (legacy interaction materialiser; the reference's CUDA
 * kernel is src/cuda/kernels.cu:1646-1676).  X row-major [n_samples][n_features] fp32,
 * output row-major [n_samples][n_combos]: for a one-feature combo the raw value, otherwise
 * the fp32 product of (X - means) over the combo's features in order; feature ids outside
 * [0, n_features) are skipped (an empty combo gives 1).  combo c spans
 * combo_indices[combo_offsets[c] .. combo_offsets[c+1]).  Synchronous; host buffers.
 * GAFIME_ERROR_INVALID_ARGS for NULL pointers, non-positive sizes or decreasing offsets. */
int gafime_feature_interaction_cuda(const float* X, const float* means, float* output,
                                    const int32_t* combo_indices, const int32_t* combo_offsets,
                                    int32_t n_samples, int32_t n_features, int32_t n_combos);

/* interfaces.h:420-425 (declared there without a GPU implementation): Pearson r of two
 * host vectors, arithmetic of gafime_pearson_cpu (cpu_backend.cpp:374-411), fp64 sums,
 * 0 when a variance is <= 0, result cast to float. */
int gafime_pearson_cuda(const float* x, const float* y, int32_t n, float* result_out);

/* ------------------------------------------- small bucket (GafimeBucket) ---- */
/* interfaces.h:176-382.  At most GAFIME_MAX_FEATURES columns; arity-2..5 chains
 * x = t_{a-2}(...t_1(t_0(op_0(f_0), op_1(f_1)), op_2(f_2))..., op_{a-1}(f_{a-1})) in fp32
 * (the per-pair-type form of cpu_backend.cpp:229-310), 12 stats split by the fold mask,
 * NaN rows skipped, fp64 sums cast to float.  Used by the reference's StaticBucket and
 * FusedKernelWrapper (gafime/backends/fused_kernel.py:318-848). */
typedef void* GafimeBucket;  /* interfaces.h:185 */
#define GAFIME_MAX_FEATURES 5
#define GAFIME_MAX_BATCH_SIZE 1024

/* interfaces.h:203-207 */
int gafime_bucket_alloc(int n_samples, int n_features, GafimeBucket* bucket_out);
/* interfaces.h:220-224; feature_idx in [0, n_features) */
int gafime_bucket_upload_feature(GafimeBucket bucket, int feature_idx, const float* h_data);
/* interfaces.h:233-236 */
int gafime_bucket_upload_target(GafimeBucket bucket, const float* h_target);
/* interfaces.h:245-248 */
int gafime_bucket_upload_mask(GafimeBucket bucket, const uint8_t* h_mask);
/* interfaces.h:266-274: feature_indices[arity], ops[arity], interaction_types[arity-1] */
int gafime_bucket_compute(GafimeBucket bucket, const int* feature_indices, const int* ops, int arity,
                          const int* interaction_types, int val_fold_id, float* h_stats);
/* interfaces.h:284 */
int gafime_bucket_free(GafimeBucket bucket);
/* interfaces.h:310-318: batch_size pairs, h_stats_batch[batch_size * 12] */
int gafime_bucket_compute_batch(GafimeBucket bucket, const int* batch_indices, const int* batch_ops,
                                const int* batch_interact, int batch_size, int val_fold_id,
                                float* h_stats_batch);
/* interfaces.h:347-361: two arity-2 interactions over the same rows; a row whose y or
 * either slot's x is NaN counts for neither slot (kernels.cu:1217-1218); rolling
 * operators evaluate to NaN (kernels.cu:298-306), window_size is accepted and unused. */
int gafime_interleaved_compute(GafimeBucket bucket, const int* feature_indices_A, const int* ops_A,
                               int arity_A, int interact_A, const int* feature_indices_B, const int* ops_B,
                               int arity_B, int interact_B, int window_size, int val_fold_id,
                               float* h_stats_A, float* h_stats_B);
/* interfaces.h:372-382: one-shot form with one interaction type for every chain step
 * (gafime_fused_interaction_cpu, cpu_backend.cpp:127-213). */
int gafime_fused_interaction(const float** h_inputs, const float* h_target, const uint8_t* h_mask,
                             const int* h_ops, int arity, int interaction_type, int val_fold_id,
                             int n_samples, float* h_stats);

/* ------------------------------------------------------- async pipeline ---- */
/* interfaces.h:433-504.  A 4-slot ring of arity-2 batches on a GafimeBucket: submit
 * returns at once (GAFIME_ERROR_PIPELINE_FULL with *slot_id_out = -1 when four batches
 * are in flight); poll (GAFIME_ERROR_NO_RESULT while the oldest batch runs) and wait
 * return the oldest batch's [batch_size * 12] stats; flush drains all in submission
 * order; pending returns 0-4 (0 for NULL). */
typedef void* GafimePipeline;  /* interfaces.h:41 */
#define PIPELINE_SLOTS 4
#define PIPELINE_MAX_BATCH 1024
int gafime_pipeline_init(GafimeBucket bucket, int val_fold_id, GafimePipeline* pipeline_out);
int gafime_pipeline_submit(GafimePipeline pipeline, const int* h_indices, const int* h_ops,
                           const int* h_interact, int batch_size, int* slot_id_out);
int gafime_pipeline_poll(GafimePipeline pipeline, float* h_stats_out, int* batch_size_out);
int gafime_pipeline_wait(GafimePipeline pipeline, float* h_stats_out, int* batch_size_out);
int gafime_pipeline_pending(GafimePipeline pipeline);
int gafime_pipeline_flush(GafimePipeline pipeline, float* h_all_stats_out, int* total_batch_size_out);
int gafime_pipeline_free(GafimePipeline pipeline);

/* ------------------------------------------------------- NEW: all pairs ---- */

/*
 * NEW.  Score every pair i<j of the bucket's features (or, with n_shards > 1,
 * this process's share of them) for n_ops interaction types and return the k
 * best pairs per operator.  Replaces the reference's per-pair loop
 * gafime/backends/native_cuda_backend.py:368-379 (one gafime_contiguous_bucket_compute
 * launch + sync per pair) with one call.
 *
 *   interact_types  n_ops ids among GAFIME_INTERACT_MULT/ADD/SUB/DIV; x = F_i op F_j
 *                   with i < j (subtract and divide are not commutative).
 *   metric          GAFIME_METRIC_PEARSON (rank by |r|) or GAFIME_METRIC_MUTUAL_INFO.
 *   center          0: raw kernel-API semantics (src/cpu/cpu_backend.cpp:229-295);
 *                   1: columns centred by their fp64 means first (Selector / Engine /
 *                      gafime_core semantics, gafime_core.cpp:570-577).
 *   div_eps         safe-divide clamp |b| < eps -> copysign(eps, b) (reference 1e-8).
 *   mi_bins         2..255 equal-width bins on the interaction and on y (gafime_core.cpp:200-333).
 *   k               1..GAFIME_ALLPAIRS_MAX_K.
 *   shard_id/n_shards  pair-tile sharding across processes (0/1 = everything).
 *   out_i, out_j, out_score   [n_ops * k]: per operator, pairs ordered by |score|
 *                   descending then (i, j) ascending; out_score is the signed score.
 *   out_count       [n_ops]: entries written per operator (< k when fewer pairs).
 *
 * The input must be finite (the engine's coerce_inputs guarantees it,
 * gafime/utils/arrays.py:26-30); non-finite values return GAFIME_ERROR_INVALID_ARGS.
 * Results are bit-identical from run to run (fixed-order fp64 reductions).
 */
int gafime_allpairs_topk(ContiguousBucket bucket, const int* interact_types, int n_ops,
                         int metric, int center, float div_eps, int mi_bins, int k,
                         int shard_id, int n_shards, int32_t* out_i, int32_t* out_j,
                         double* out_score, int* out_count);

/*
 * NEW.  gafime_contiguous_bucket_upload(bucket, h_data, h_mask) followed by
 * gafime_allpairs_topk(bucket, ...), with the host-to-device copy overlapped with the
 * scoring: the target goes first, then the features in 128-column blocks on a copy stream,
 * and the tiles each block completes are scored while the next block is in flight.  The
 * reference uploads the whole bucket before any launch (native_cuda_backend.py:339-352,
 * contiguous_layout.rs:64-156).  h_data is the upload's layout ([F0 | ... | F_{F-1} | y],
 * n floats each); pinned host memory is what lets the copies overlap.  Same results as the
 * two calls (the same kernels on the same data and row chunks); non-finite input returns
 * GAFIME_ERROR_INVALID_ARGS like the upload's check.  Pearson with center = 0 on the
 * tensor-core path streams; other metrics and modes run the two calls.  With n_shards > 1
 * only the 128-column blocks that this shard's tiles read are copied and checked (a
 * process of a multi-GPU job moves its share of the matrix); the bucket's other columns
 * keep what they held, so a later call of another kind on this bucket needs a full upload.
 */
int gafime_allpairs_topk_host(ContiguousBucket bucket, const float* h_data, const uint8_t* h_mask,
                              const int* interact_types, int n_ops, int metric, int center,
                              float div_eps, int mi_bins, int k, int shard_id, int n_shards,
                              int32_t* out_i, int32_t* out_j, double* out_score, int* out_count);

/*
 * NEW.  gafime_allpairs_topk for one shard with the result left on the device, for the
 * candidate exchange of a multi-GPU job (the all-gather runs on device buffers, with no
 * host copy in between).  Queues the scoring on the bucket's stream
 * (gafime_contiguous_bucket_stream) and returns without waiting for it.  d_cands (device,
 * 16-byte aligned) receives, per operator, next_pow2(k) candidate records of 16 bytes
 * (fp64 signed score, uint32 pair id i * F + j, 4 bytes padding) sorted by |score|
 * descending then pair id ascending; empty slots have pair id 0xFFFFFFFF.  Finish with
 * gafime_topk_merge_device on the same bucket, which reports any kernel failure.
 */
int gafime_allpairs_topk_device(ContiguousBucket bucket, const int* interact_types, int n_ops,
                                int metric, int center, float div_eps, int mi_bins, int k,
                                int shard_id, int n_shards, void* d_cands);

/*
 * NEW.  Device merge of n_shards shards' gafime_allpairs_topk_device lists, as they lie after
 * an all-gather: d_gathered holds n_shards blocks of n_ops lists of next_pow2(k) records.
 * Orders them on the bucket's stream (after the work queued there, so an all-gather run on
 * that stream is waited for), copies the k best per operator to the host in the layout of
 * gafime_allpairs_topk and waits for them.  Same ranking as gafime_topk_merge.
 */
int gafime_topk_merge_device(ContiguousBucket bucket, const void* d_gathered, int n_shards, int n_ops, int k,
                             int32_t* out_i, int32_t* out_j, double* out_score, int* out_count);

/*
 * NEW.  Signed score of every pair i<j for one operator, in row-major
 * upper-triangle order (p = i*F - i*(i+1)/2 + j - i - 1), P = F*(F-1)/2 entries.
 * Serves Backend.score_combos (gafime/backends/base.py:67-78) when the combo list
 * is all pairs of the bucket's features.
 */
int gafime_allpairs_scores(ContiguousBucket bucket, int interact_type, int metric, int center,
                           float div_eps, int mi_bins, double* out_scores);

/*
 * NEW.  Number of (pair, operator) Pearson scores that the last gafime_allpairs_topk,
 * gafime_allpairs_topk_host or gafime_allpairs_scores call on this bucket took from an
 * exact re-score.  The pair moments come from fp32 accumulations; an accuracy guard
 * estimates each pair's rounding of its interaction's variance (the pair's sum of squares
 * for columns far from zero, the columns' spreads for products tiny against them) and
 * re-scores the pairs where it is not small against that variance with fp64 sums of
 * fl32(a op b) per row, the reference CPU arithmetic (cpu_backend.cpp:87-103,274-293).
 * 0 for mutual information and on data with well-conditioned pairs.
 */
int gafime_allpairs_rescored(ContiguousBucket bucket, int64_t* out_count);

/*
 * NEW.  Score of every single feature (unary combo) against the target, F entries:
 * Pearson of the raw column (pearson_from_sums, gafime_core.cpp:179-198) or equal-width
 * mutual information of the raw column (gafime_core.cpp:559-569 with k == 1).  Serves
 * the engine's unary stage (gafime/engine.py:39-51), which picks the features whose
 * pairs are scored next.
 */
int gafime_unary_scores(ContiguousBucket bucket, int metric, int mi_bins, double* out_scores);

/*
 * NEW.  Host only.  The 64 x 64 pair tiles (block row bi, block column bj, bi <= bj;
 * pairs i in [64 bi, 64 bi + 64) x j in [64 bj, 64 bj + 64), i < j) that shard shard_id
 * of n_shards scores in gafime_allpairs_topk.  The pair space is dealt out in 128 x 128
 * blocks (the tensor-core tile).  A shard's cost is 4 x the 64-tiles it computes (a block
 * holds 4, or 3 on the diagonal) + 3 x the 128-column blocks its tiles read (its statistics
 * pass covers those); the plan with the lowest busiest-shard cost is kept, from a
 * least-loaded greedy split and group-pair splits, each refined by moving and swapping
 * blocks.  Every process derives the same split without communicating; a shard scores the
 * 64-tiles inside its blocks.  out_tiles receives
 * 2 * *out_count ints (bi, bj); returns GAFIME_ERROR_INVALID_ARGS with *out_count set
 * when max_tiles is too small.
 */
int gafime_shard_tiles(int n_features, int shard_id, int n_shards, int32_t* out_tiles,
                       int max_tiles, int* out_count);

/*
 * NEW.  Deterministic host merge of per-shard candidates (the step after the
 * allgather of every shard's top-k): keeps the k best of n_cand entries by
 * |score| descending then (i, j) ascending.  out_* hold min(k, n_cand) entries;
 * *out_count receives that number.
 */
int gafime_topk_merge(const int32_t* cand_i, const int32_t* cand_j, const double* cand_score,
                      int64_t n_cand, int k, int32_t* out_i, int32_t* out_j, double* out_score,
                      int* out_count);

/* ------------------------------------------------------ NEW: profiling ---- */

/* Kernel ids of the timing registry. */
#define GAFIME_KERNEL_COLUMN_STATS 1
#define GAFIME_KERNEL_PAIR_MOMENTS 2
#define GAFIME_KERNEL_EPILOGUE_TOPK 3
#define GAFIME_KERNEL_MERGE 4
#define GAFIME_KERNEL_MI_PASS1 5
#define GAFIME_KERNEL_MI_PASS2 6
#define GAFIME_KERNEL_MI_FINISH 7
#define GAFIME_KERNEL_LEGACY_PAIR 8
#define GAFIME_KERNEL_FINITE_CHECK 9
#define GAFIME_KERNEL_GRAM_TC 10
#define GAFIME_KERNEL_GRAM_PREP 11
#define GAFIME_KERNEL_GRAM_REDUCE 12
#define GAFIME_KERNEL_MI_CLASS_COPY 13
#define GAFIME_KERNEL_GUARD 14

/* NEW.  enable = 1: drop any previous records, then bracket every engine kernel
 * launch with CUDA events on its stream.  enable = 0: stop recording (the records
 * stay readable until the next enable = 1). */
int gafime_profile_enable(int enable);

/* NEW.  Total device milliseconds and number of launches recorded for one kernel
 * id (kernel_id < 0: all kernels).  Waits for the recorded events. */
int gafime_profile_read(int kernel_id, double* total_ms, int* launches);

/* NEW.  The CUDA stream (cudaStream_t) every call on this bucket runs on, so a
 * caller can order its own work or events against it. */
int gafime_contiguous_bucket_stream(ContiguousBucket bucket, void** stream_out);

/* NEW.  Spearman rank correlation of each combo against the target, as gafime_core's
 * "spearman" metric computes it (gafime_core.cpp:156-177 average-tie ranks,
 * 503-517 target ranks, 595-607 Pearson of the ranks).  Combo c is feature feat_a[c] alone
 * when feat_b[c] < 0 (the raw column, gafime_core.cpp:558-568), else the pair
 * x = (a - mean_a) op (b - mean_b) in fp64 (center = 1; gafime_core.cpp:571-577 for
 * multiply) or fl32(a op b) (center = 0; cpu_backend.cpp:87-103).  interact_type as
 * gafime_allpairs_topk; out_scores receives n_combos values.  One device-wide sort per
 * combo (the reference sorts per combo on the host: gafime_core.cpp:596). */
int gafime_spearman_scores(ContiguousBucket bucket, const int32_t* feat_a, const int32_t* feat_b,
                           int64_t n_combos, int interact_type, int center, float div_eps,
                           double* out_scores);

/* NEW.  gafime_contiguous_bucket_upload from the caller's row-major matrix: h_rows holds
 * n_samples rows of n_features floats (X[i, f] at h_rows[i * n_features + f], numpy's C
 * order), h_y n_samples floats, h_mask n_samples bytes.  The rows are copied in chunks and
 * transposed into the bucket's column layout on the device, so the caller does not build the
 * column-major host buffer (the reference's backend transposes on the host:
 * native_cuda_backend.py:339-342).  Checks the data like the upload. */
int gafime_contiguous_bucket_upload_rows(ContiguousBucket bucket, const float* h_rows, const float* h_y,
                                         const uint8_t* h_mask);

/* NEW.  Replace only the target of an uploaded bucket with n_samples floats from the host
 * (the features stay resident).  Permutation tests re-score the same matrix against
 * permuted targets; the reference re-uploads matrix and target per call
 * (gafime/backends/native_cuda_backend.py:344-352).  Checks the new target for non-finite
 * values like an upload does. */
int gafime_contiguous_bucket_upload_target(ContiguousBucket bucket, const float* h_y);

/* NEW.  Fill dst from a resident bucket on the same device, without a host copy of the
 * matrix: feature c of dst is feature cols[c] of src, and row r of dst (features, target
 * and fold mask) is row rows[r] of src (rows == NULL: every row, n_rows == src's rows).
 * dst must have been allocated with n_rows samples and n_cols features.  Column subsets and
 * bootstrap resamples of the engine (gafime/validation/stability.py:35-42 indexes X[idx],
 * y[idx] on the host) come from the matrix uploaded once.  GAFIME_ERROR_INVALID_ARGS for an
 * index out of range or a size mismatch. */
int gafime_contiguous_bucket_gather(ContiguousBucket dst, ContiguousBucket src, const int32_t* cols,
                                    int32_t n_cols, const int64_t* rows, int64_t n_rows);

/* NEW.  Sharded ingest of a bucket replicated on several GPUs (one process per GPU): each
 * rank copies only features [c0, c1) from the host with this call, and a collective over
 * NVLink (an all-gather on the bucket's stream, on the device range that
 * gafime_contiguous_bucket_device_columns reports) fills in the others, so the host link
 * carries the matrix once however many GPUs hold it.  h_cols holds features c0..c1-1 as
 * (c1 - c0) x n_samples floats (the same layout as rows c0..c1-1 of the upload's h_data),
 * h_y the n_samples target values and h_mask the fold mask, all ideally pinned.  The copies
 * are queued on the bucket's stream and the call returns without waiting for them; the
 * caller keeps the host buffers intact until that stream has passed them.  The data is
 * checked for non-finite values by the next scoring call, as after an upload. */
int gafime_contiguous_bucket_upload_columns(ContiguousBucket bucket, const float* h_cols, int64_t c0, int64_t c1,
                                            const float* h_y, const uint8_t* h_mask);

/* NEW.  Device address of feature c0 of a bucket and the distance between consecutive
 * features in floats (*ld >= n_samples; rows n_samples..ld-1 of every feature are zero and
 * stay zero).  Features c0..c1-1 are the contiguous range [*d_ptr, *d_ptr + (c1 - c0) * ld),
 * which a collective may fill in place; the caller then calls
 * gafime_contiguous_bucket_mark_updated before scoring. */
int gafime_contiguous_bucket_device_columns(ContiguousBucket bucket, int64_t c0, int64_t c1, float** d_ptr,
                                            int64_t* ld);

/* NEW.  Declares that features were written through gafime_contiguous_bucket_device_columns:
 * the next scoring call checks the whole matrix for non-finite values again. */
int gafime_contiguous_bucket_mark_updated(ContiguousBucket bucket);

/* ------------------------------------------- NEW: no device allocation ---- */

/* Largest problem gafime_allpairs_scores_noalloc accepts. */
#define GAFIME_NOALLOC_MAX_FEATURES 256
#define GAFIME_NOALLOC_MAX_ROWS 2097152

/*
 * NEW -- no counterpart in the reference.  Signed Pearson score of every pair i<j
 * (row-major upper-triangle order, as gafime_allpairs_scores, raw kernel-API
 * semantics) for a matrix that is already on the GPU, without allocating any GPU
 * memory: no cudaMalloc, no cudaFree, no allocating library call.
 *
 * For programs that own the GPU's memory themselves -- an arena or caching allocator
 * that has reserved most of the device, or a host application that hands out device
 * buffers it carved out of its own pool -- where a library that calls cudaMalloc can
 * fail for lack of room, fragment the owner's pool, or stall other streams with the
 * device-wide synchronisation cudaMalloc/cudaFree may imply.
 *
 *   d_x           device, column-major: column f at d_x + f*ld, 16-byte aligned;
 *                 rows n_samples..ld-1 of every column must be zero.
 *   ld            multiple of 256, n_samples <= ld <= GAFIME_NOALLOC_MAX_ROWS.
 *   d_y           device, n_samples floats.
 *   n_features    1..GAFIME_NOALLOC_MAX_FEATURES.
 *   interact_type GAFIME_INTERACT_MULT/ADD/SUB/DIV;  div_eps as gafime_allpairs_topk.
 *   d_scores_out  device, F*(F-1)/2 doubles, written on success.
 *   stream        cudaStream_t to run on (NULL: the default stream); the call waits
 *                 for it before returning.
 *
 * Sizes beyond the limits, a misaligned d_x or an ld that is not a multiple of 256
 * return GAFIME_ERROR_INVALID_ARGS before any GPU work; non-finite input returns
 * GAFIME_ERROR_INVALID_ARGS as gafime_allpairs_scores does.
 *
 * All intermediates live in one fixed 32 MiB __device__ array that every GPU loading
 * the library holds until the process exits.  Every call reuses that array, so calls
 * that overlap on the GPU (other streams or threads) race and must be serialised.
 * The first call on each device looks the array's address up with
 * cudaGetSymbolAddress; make it before any stream capture starts.
 */
int gafime_allpairs_scores_noalloc(const float* d_x, int64_t ld, const float* d_y, int n_samples,
                                   int n_features, int interact_type, float div_eps,
                                   double* d_scores_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GAFIME_B200_H */
