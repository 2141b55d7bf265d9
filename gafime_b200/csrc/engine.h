// engine.h -- internal declarations of libgafime_cuda.so (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "../../include/gafime_b200.h"

namespace gafime {

// Rows of every device column are padded to a multiple of this (zeros), so the
// tiled kernels never see a partial chunk.  Zero rows add nothing to any sum of
// products the all-pairs kernels form (x = a*g(b) with a = 0).
constexpr int64_t kRowPad = 256;

// Pair tiles of the CUDA-core moment kernel: kTile x kTile columns.
constexpr int kTile = 64;
constexpr int kTilePairs = kTile * kTile;

// One candidate of the top-k selection: signed score + pair id (i * F + j).
struct Cand {
    double score;
    uint32_t pid;
    uint32_t pad;
};
constexpr uint32_t kNoPair = 0xFFFFFFFFu;

// Device-side record of a pair tile: columns [bi*kTile, +kTile) x [bj*kTile, +kTile).
struct TileCoord {
    int bi, bj;
};

// Scratch buffers owned by a bucket and grown on demand (never shrunk until free).
struct DeviceBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
};

struct Bucket {
    int device = 0;
    int64_t n = 0;        // rows
    int64_t f = 0;        // feature columns
    int64_t ld = 0;       // padded rows per device column
    float* d_data = nullptr;   // (f + 1) * ld floats: features then target
    uint8_t* d_mask = nullptr; // n bytes
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;       // host-to-device copies of a streamed call
    std::vector<cudaEvent_t> arrived;         // one per column block (+ the target) of it
    double* h_pinned = nullptr;  // small pinned staging for stats
    int finite_state = -1;       // -1 unknown, 0 some value is NaN/inf, 1 all finite (per upload)
    int sm_count = 148;
    // scratch
    DeviceBuf stats_part, stats, ycen, xcen, moments, cands, cands2, scores, flags, tiles, mi,
        mi_hist, mi_mm, mi_xs, mi_split, gather, rank, gram, gram_cols, gram_planes, guard;
    // (pair, operator) scores the accuracy guard re-scored exactly in the last all-pairs call
    int64_t last_rescored = 0;
    bool guard_ran = false;      // the guard's counter (start of `guard`) belongs to this call
    int pending_gram = 0;        // a device top-k ran Gram kernels whose error flag is still unread
};

// Grow a scratch buffer to at least `bytes`; returns cudaSuccess or an error.
cudaError_t ensure(DeviceBuf& b, size_t bytes);

// Column statistics, all fp64 and deterministic (fixed reduction order).
//   colstats[c*4 + 0] = sum x, [1] = sum x^2, [2] = sum x*ycen, [3] = mean
//   ystats[0] = n, [1] = sum y, [2] = var_y = sum y^2 - (sum y)^2 / n, [3] = mean y
// With centred=true the statistics describe the centred copy written to xcen.
struct ColumnStats {
    const double* d_col = nullptr;  // [f * 4]
    const double* d_y = nullptr;    // [4]
    const float* d_x = nullptr;     // matrix the pair kernels read (raw or centred)
    const float* d_ycen = nullptr;  // fl32(y - mean y), zero padded
    double h_y[4];
};
// x_sums = false leaves colstats to the caller (the tensor-core path computes the column
// sums in its own pass over the columns, before anything reads them).
int compute_column_stats(Bucket& b, bool centred, ColumnStats& out, bool x_sums = true);

// Finite-input check over the features and y, run once per upload and cached.
int check_finite(Bucket& b, bool* all_finite);
// flag |= 1 when any of n_floats (a multiple of 4, 16-byte aligned) is NaN or infinite
cudaError_t launch_finite_check(const float* x, int64_t n_floats, int* flag, int blocks, cudaStream_t stream);

// Column-statistics kernels of bucket.cu, declared for other translation units.
__global__ void col_partial_kernel(const float* __restrict__ x, int64_t ld, int64_t n,
                                   const float* __restrict__ ycen, int64_t span,
                                   double* __restrict__ part);
__global__ void col_combine_kernel(const double* __restrict__ part, int cols, int splits,
                                   int64_t n, double* __restrict__ colstats);
__global__ void ystats_kernel(const double* __restrict__ ycol, int64_t n, double* __restrict__ ystats);
__global__ void ycen_kernel(const float* __restrict__ y, int64_t n, int64_t ld,
                            const double* __restrict__ ystats, float* __restrict__ ycen);
__global__ void finite_kernel(const float* __restrict__ x, int64_t cols, int64_t ld, int64_t n,
                              int* __restrict__ flag);

// CUDA-core three-moment pair kernel (moments.cu).  For every pair (i, j) of the
// listed tiles: S1 = sum a*g(b), S2 = sum (a*g(b))^2, S3 = sum a*g(b)*ycen with
// a = X[:, i], b = X[:, j], g = identity (recip = false) or 1/safe(b).
// Output layout: moments[((split * n_tiles + t) * 3 + m) * kTilePairs + li*kTile + lj].
cudaError_t launch_pair_moments(const float* d_x, int64_t ld, const float* d_ycen, int64_t f,
                                const TileCoord* d_tiles, int n_tiles, int splits,
                                int64_t rows_per_split, bool recip, float eps, double* d_moments,
                                cudaStream_t stream);

// Tensor-core pair moments (gram.cu): the same S1/S2/S3 as launch_pair_moments for the
// shard's 64-tiles, computed as tcgen05 Gram tiles over 128-blocks; writes one split
// (splits = 1) into d_moments.  *host_err != 0 reports a bounded wait that gave up.
// prep_mode: GRAM_PREP_OWN computes the per-column scales this group needs, GRAM_PREP_BOTH
// those of both groups (a divide group follows), GRAM_PREP_DONE reuses them.
enum { GRAM_PREP_OWN = 0, GRAM_PREP_BOTH = 1, GRAM_PREP_DONE = 2 };
bool gram_path_enabled(const Bucket& b);
// Per-column preparation of the Gram path, split so a streamed call can prepare column
// blocks as they arrive: the scaled target once (after the target statistics), then the
// statistics and operand scales of columns [c0, c1) (recip: the divide side's too).
cudaError_t gram_prep_target(Bucket& b, const ColumnStats& cs, cudaStream_t stream);
cudaError_t gram_prep_columns(Bucket& b, const ColumnStats& cs, bool recip, float eps, int64_t c0, int64_t c1,
                              cudaStream_t stream);
// chunk_rows > 0 fixes the row chunk of the tiles; 0 takes gram_chunk_rows, which depends
// on the matrix alone (every shard and every streamed tile set gets the same chunks).
// use_planes: 1 the B-planes kernel, 0 the fused kernel, -1 chosen from this tile set
// (gram_use_planes); a streamed call decides once for its whole tile set.
cudaError_t launch_gram_moments(Bucket& b, const ColumnStats& cs, const TileCoord* d_tiles64,
                                const std::vector<TileCoord>& tiles64, bool recip, float eps,
                                double* d_moments, cudaStream_t stream, int* host_err, int prep_mode,
                                int64_t chunk_rows = 0, int use_planes = -1);
// True when a tile set reuses its B blocks enough for the B-planes kernel (or when
// GAFIME_GRAM_KERNEL forces it).
bool gram_use_planes(const Bucket& b, const std::vector<TileCoord>& tiles64);
int64_t gram_chunk_rows(const Bucket& b);
// host_err null: launch_gram_moments neither clears nor reads the Gram kernels' error flag
// (no host sync); the caller clears it before its launches and reads it once at the end.
cudaError_t gram_error_reset(Bucket& b, cudaStream_t stream);
cudaError_t gram_error_read(Bucket& b, cudaStream_t stream, int* host_err);
// Per-column state of the Gram path (12 doubles per column; [6] sum g, [7] sum g^2 of the
// divide side g = 1/safe(x)), valid after gram_prep_columns of this call.
const double* gram_col_state(Bucket& b);

// Scoring epilogue + per-tile top-k (select.cu).
struct EpilogueArgs {
    // per operator (blockIdx.z): moments from the pair-moment kernels (mul or div group),
    // their row splits, the GAFIME_INTERACT_* id, and the candidate lists
    const double* moments[4];
    int splits[4];
    int op[4];
    Cand* cands[4];              // [n_tiles * sub_lists * k_pad] per op (nullptr: scores only)
    int n_ops;
    const TileCoord* tiles;
    int n_tiles;
    int64_t f;
    const double* colstats;      // [f*4]
    const double* ystats;        // [4]
    int k_pad;                   // power of two >= k, <= 4096
    int sub_lists;               // candidate lists per tile (power of two, 4096 / sub_lists >= k_pad)
    double* all_scores;          // nullable, [P] triangle order (n_ops = 1)
    // accuracy guard (guard.cu), nullable: a pair whose flag is set takes its exact score
    const uint8_t* guard_flags;  // [n_ops][n_tiles][kTilePairs]
    const double* exact;         // [n_ops][n_tiles][kTilePairs], written for flagged pairs only
};
cudaError_t launch_epilogue_topk(const EpilogueArgs& a, cudaStream_t stream);

// Accuracy guard of the Pearson epilogue (guard.cu): flags the pairs whose estimated
// rounding of n var_x is not small against it, and re-scores them exactly (fp64 sums of
// fl32(a op b) per row, the reference CPU arithmetic).
struct GuardArgs {
    const double* moments[4];
    int splits[4];
    int op[4];
    int n_ops;
    const TileCoord* tiles;
    int n_tiles;
    int64_t f;
    const double* colstats;      // [f*4]
    const double* ystats;        // [4]
    const double* gstats;        // Gram column state (12 doubles per column), required when gram
    int gram;                    // moments from the tensor-core Gram path (S1 from centred Grams)
    uint8_t* flags;              // out: [n_ops][n_tiles][kTilePairs]
    unsigned long long* count;   // out: flagged entries (cleared by launch_guard)
    uint2* list;                 // out: [capacity] (t * kTilePairs + e, operator index)
};
struct RescoreArgs {
    const float* x;              // matrix the pair kernels read (f columns of ld floats)
    const float* y;              // raw target (n floats, 16-byte aligned)
    int64_t ld, n;               // column stride, rows
    float eps;
    int op[4];
    const TileCoord* tiles;
    int n_tiles;
    const double* ystats;        // [4]
    const unsigned long long* count;
    const uint2* list;
    double* exact;               // out: [n_ops][n_tiles][kTilePairs]
};
cudaError_t launch_guard(const GuardArgs& g, const RescoreArgs& r, int sm_count, cudaStream_t stream);
// Candidate lists per tile for a top-k call: enough CTAs to fill the GPU.
int epilogue_sub_lists(int n_tiles, int k_pad, int sm_count);

// Merge n_lists sorted candidate lists of k_pad entries down to one, for n_ops operators at
// once (operator o's lists start op_stride entries after operator o-1's, in buf and tmp);
// ping-pong between buf and tmp.  *final_list holds operator 0's result; operator o's is
// op_stride entries further.
cudaError_t merge_candidates(Cand* buf, Cand* tmp, int n_lists, int k_pad, int n_ops, size_t op_stride,
                             Cand** final_list, cudaStream_t stream);
// n entries of "no pair" (the empty list a shard without tiles contributes)
cudaError_t fill_empty_lists(Cand* out, size_t n, cudaStream_t stream);
// Gathered shard lists [shard][op][k_pad] -> [op][shard][k_pad]
cudaError_t reorder_shard_lists(const Cand* in, Cand* out, int n_shards, int n_ops, int k_pad, cudaStream_t stream);

// Mutual-information scoring (mi.cu): centred product, equal-width bins.
// cs must hold raw-column statistics (means of the uncentred columns).
cudaError_t launch_mi_scores(Bucket& b, const ColumnStats& cs, bool centred, int op, float div_eps,
                             int mi_bins, const TileCoord* d_tiles, int n_tiles, int k_pad,
                             Cand* cands, double* all_scores, cudaStream_t stream);

// Mutual information with quantile bins on the interaction (mi.cu): exact order-statistic
// cut points per pair, equal-width y bins; candidate lists / all_scores as launch_mi_scores.
cudaError_t launch_mi_quantile(Bucket& b, const ColumnStats& cs, bool centred, int op, float div_eps, int mi_bins,
                               const std::vector<TileCoord>& tiles, const TileCoord* d_tiles, int k_pad,
                               Cand* cands, double* all_scores, cudaStream_t stream);

// Unary (single-feature) mutual information of every raw column against y
// (gafime_core.cpp:559-569 with k == 1: the raw column, no centring).
cudaError_t launch_mi_unary(Bucket& b, int mi_bins, double* d_out, cudaStream_t stream);

// Upper-triangle 64 x 64 pair tiles assigned to one shard (allpairs.cu): tiles in
// row-major order, each to the least-loaded shard by pair count, ties to the lowest id.
std::vector<TileCoord> shard_tiles(int64_t f, int shard_id, int n_shards);

// Ranking used everywhere: |score| descending, NaN after every number, empty
// slots last; ties by pair id ascending.  cand_key orders like that rank as an unsigned
// integer (|score| bits order like |score| for non-NaN doubles), so a comparison is two
// integer compares.
__host__ __device__ inline uint64_t cand_key(const Cand& c) {
    if (c.pid == kNoPair) return 0;
    uint64_t u;
    memcpy(&u, &c.score, sizeof(u));
    u &= 0x7FFFFFFFFFFFFFFFull;
    if (u > 0x7FF0000000000000ull) return 1;  // NaN
    return u + 2;
}
__host__ __device__ inline bool cand_before(const Cand& a, const Cand& b) {
    const uint64_t ka = cand_key(a), kb = cand_key(b);
    if (ka != kb) return ka > kb;
    return a.pid < b.pid;
}

// Map a CUDA error to the ABI status code.
int status_from(cudaError_t e);

// Brackets one kernel launch with CUDA events on its stream while profiling is
// enabled (profile.cu); kernel ids are the GAFIME_KERNEL_* values of the ABI.
class KernelTimer {
  public:
    KernelTimer(cudaStream_t stream, int kernel_id);
    ~KernelTimer();
    KernelTimer(const KernelTimer&) = delete;
    KernelTimer& operator=(const KernelTimer&) = delete;

  private:
    cudaStream_t stream_;
    int id_;
    bool active_ = false;
    cudaEvent_t start_{}, stop_{};
};

}  // namespace gafime
