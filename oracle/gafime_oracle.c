/*
 * gafime_oracle.c -- CPU restatement of GAFIME's pair-scoring arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle for the CUDA path: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
 * The product (gafime_b200/) never calls it and has no CPU fallback.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here against
 * golden vectors produced by the reference's own code (gafime_core.cpp and
 * cpu_backend.cpp compiled unmodified by oracle/Makefile, and the reference's
 * numpy metrics), committed under tests/golden/ with the script that made them.
 *
 * Three semantics are restated, each citing the reference lines it follows:
 *
 *  1. Raw-operator moments (kernel-API path, src/cpu/cpu_backend.cpp):
 *     x = combine(a, b) evaluated in fp32 (cpu_backend.cpp:87-103), rows with
 *     NaN x or y skipped (cpu_backend.cpp:274), sums of n, x, y, x^2, y^2, x*y
 *     accumulated in fp64 (cpu_backend.cpp:276-293).  Unlike the reference the
 *     six sums are returned in fp64 instead of being cast to float
 *     (cpu_backend.cpp:296-307), and the divide epsilon is a parameter instead
 *     of the literal 1e-8f (cpu_backend.cpp:94).
 *
 *  2. Pearson from the six sums (gafime/backends/native_cuda_backend.py:471-486).
 *
 *  3. Centred-product scoring (Selector / Engine / gafime_core path,
 *     gafime_core/src/gafime_core.cpp:425-623): column means in fp64 in serial
 *     row order (gafime_core.cpp:134-150), centred product in fp64
 *     (gafime_core.cpp:571-577), Pearson via pearson_from_sums
 *     (gafime_core.cpp:179-198) against the centred target
 *     (gafime_core.cpp:486-497), mutual information with equal-width min/max
 *     bins on both axes (gafime_core.cpp:200-226, 267-333).
 *
 *  4. Chains of the small-bucket ABI (gafime_bucket_compute / gafime_fused_interaction):
 *     per-feature unary operators of cpu_backend.cpp:30-77, left-to-right combination
 *     with per-step interaction types (combine_cpu, cpu_backend.cpp:85-103, literal
 *     divide epsilon 1e-8f), NaN rows skipped, 12 fp64 sums split by the fold mask
 *     (cpu_backend.cpp:229-295), returned in fp64.
 *
 *  5. The interaction materialiser (legacy ABI gafime_feature_interaction_cuda,
 *     src/cuda/kernels.cu:1646-1676): out[i, c] = X[i, f] for a one-feature combo,
 *     otherwise the fp32 product over the combo's features of (X[i, f] - means[f]) in
 *     combo order; feature ids outside [0, F) are skipped, so an empty combo (or one whose
 *     features are all invalid) yields 1.  cpu_backend.cpp:316-370 agrees on every combo
 *     whose features are valid (it writes 0 for the degenerate ones).
 *
 *  7. Mutual information with quantile bins on the interaction (a mode this library adds; the
 *     reference has equal-width bins only, so it is parity unpinned): order-statistic cut
 *     points, equal-width y bins, the reference's MI sum.
 *
 *  6. Mutual information of any operator (raw fp32 or centred fp64 interaction) and of raw
 *     columns, and Spearman rank correlation (rankdata with average ties and the Pearson of
 *     ranks, gafime_core.cpp:156-177,503-517,595-607), for unaries and pairs.
 *
 * Data layout: X is column-major fp32, column f at X + f * ld, n rows (the materialiser
 * takes the reference's row-major X, row i at X + i * F).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_MULT 0
#define OR_ADD 1
#define OR_SUB 2
#define OR_DIV 3

/* combine_cpu, cpu_backend.cpp:87-103, with the divide epsilon as a parameter. */
static inline float or_combine(float a, float b, int op, float eps) {
    switch (op) {
        case OR_ADD: return a + b;
        case OR_SUB: return a - b;
        case OR_DIV: return a / (fabsf(b) < eps ? copysignf(eps, b) : b);
        case OR_MULT:
        default: return a * b;
    }
}

/* Six fp64 sums of one pair: out = [n, sx, sy, sxx, syy, sxy].
 * Follows gafime_fused_interaction_perpair_cpu (cpu_backend.cpp:229-295) for
 * arity 2, identity unary ops and every row in the "train" split
 * (val_fold_id = 255 never matches the all-zero mask the reference uploads,
 * native_cuda_backend.py:344,371). */
void gafime_oracle_pair_moments(const float* xa, const float* xb, const float* y,
                                int64_t n, int op, float div_eps, double* out) {
    double cn = 0, sx = 0, sy = 0, sxx = 0, syy = 0, sxy = 0;
    for (int64_t r = 0; r < n; ++r) {
        float x = or_combine(xa[r], xb[r], op, div_eps);
        float yv = y[r];
        if (isnan(x) || isnan(yv)) continue;
        double xd = (double)x, yd = (double)yv;
        cn += 1.0;
        sx += xd;
        sy += yd;
        sxx += xd * xd;
        syy += yd * yd;
        sxy += xd * yd;
    }
    out[0] = cn; out[1] = sx; out[2] = sy; out[3] = sxx; out[4] = syy; out[5] = sxy;
}

/* _pearson_from_stats, native_cuda_backend.py:471-486. */
double gafime_oracle_pearson_from_stats(const double* s) {
    double n = s[0];
    if (n <= 1.0) return 0.0;
    double var_x = s[3] - s[1] * s[1] / n;
    double var_y = s[4] - s[2] * s[2] / n;
    double cov = s[5] - s[1] * s[2] / n;
    double denom_sq = var_x * var_y;
    if (denom_sq <= 0.0) return 0.0;
    return cov / sqrt(denom_sq);
}

/* Signed raw-operator Pearson for a list of pairs (i, j): x = X[:,i] op X[:,j].
 * Pairs are independent; the loop over pairs is parallel when built with OpenMP. */
void gafime_oracle_raw_pearson(const float* X, int64_t ld, const float* y, int64_t n,
                               const int32_t* pi, const int32_t* pj, int64_t n_pairs,
                               int op, float div_eps, double* out_r, double* out_stats) {
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t p = 0; p < n_pairs; ++p) {
        double s[6];
        gafime_oracle_pair_moments(X + (int64_t)pi[p] * ld, X + (int64_t)pj[p] * ld, y, n,
                                   op, div_eps, s);
        out_r[p] = gafime_oracle_pearson_from_stats(s);
        if (out_stats) memcpy(out_stats + 6 * p, s, sizeof(s));
    }
}

/* ---------------------------------------------------------------------------
 * Centred-product semantics of gafime_core.score_combos.
 * ------------------------------------------------------------------------- */

/* compute_means, gafime_core.cpp:134-150: serial row order, fp64. */
void gafime_oracle_column_means(const float* X, int64_t ld, int64_t n, int64_t f_count,
                                double* means) {
    for (int64_t f = 0; f < f_count; ++f) {
        double sum = 0.0;
        const float* col = X + f * ld;
        for (int64_t r = 0; r < n; ++r) sum += (double)col[r];
        means[f] = (n == 0) ? 0.0 : sum / (double)n;
    }
}

/* pearson_from_sums, gafime_core.cpp:179-198. */
static double or_pearson_from_sums(double sum_x, double sum_x2, double dot_xy, double var_y,
                                   int64_t n) {
    if (n == 0) return 0.0;
    double mean_x = sum_x / (double)n;
    double var_x = sum_x2 - (sum_x * mean_x);
    if (var_x <= 0.0 || var_y <= 0.0) return 0.0;
    double denom = sqrt(var_x * var_y);
    if (denom == 0.0) return 0.0;
    return dot_xy / denom;
}

/* build_bins, gafime_core.cpp:200-226 (fp64 values). Returns 0 when the
 * values are constant or bins < 2, as the reference does. */
static int or_build_bins(const double* v, int64_t n, int bins, int32_t* out) {
    if (bins < 2 || n == 0) return 0;
    double vmin = v[0], vmax = v[0];
    for (int64_t i = 1; i < n; ++i) {
        vmin = v[i] < vmin ? v[i] : vmin;
        vmax = v[i] > vmax ? v[i] : vmax;
    }
    if (vmin == vmax) return 0;
    double scale = (double)bins / (vmax - vmin);
    for (int64_t i = 0; i < n; ++i) {
        int b = (int)((v[i] - vmin) * scale);
        if (b < 0) b = 0; else if (b >= bins) b = bins - 1;
        out[i] = b;
    }
    return 1;
}

/* mutual_info_from_vector, gafime_core.cpp:267-333. */
static double or_mutual_info(const double* x, int64_t n, int bins, const int32_t* y_bins,
                             double* joint, double* p_x, double* p_y) {
    if (bins < 2 || n == 0) return 0.0;
    double xmin = x[0], xmax = x[0];
    for (int64_t i = 1; i < n; ++i) {
        xmin = x[i] < xmin ? x[i] : xmin;
        xmax = x[i] > xmax ? x[i] : xmax;
    }
    if (xmin == xmax) return 0.0;
    size_t b2 = (size_t)bins * (size_t)bins;
    memset(joint, 0, b2 * sizeof(double));
    memset(p_x, 0, (size_t)bins * sizeof(double));
    memset(p_y, 0, (size_t)bins * sizeof(double));
    double scale = (double)bins / (xmax - xmin);
    for (int64_t i = 0; i < n; ++i) {
        int xb = (int)((x[i] - xmin) * scale);
        if (xb < 0) xb = 0; else if (xb >= bins) xb = bins - 1;
        int yb = y_bins[i];
        joint[(size_t)xb * bins + yb] += 1.0;
        p_x[xb] += 1.0;
        p_y[yb] += 1.0;
    }
    double inv_total = 1.0 / (double)n;
    double inv_total_sq = inv_total * inv_total;
    double mi = 0.0;
    for (int bx = 0; bx < bins; ++bx) {
        for (int by = 0; by < bins; ++by) {
            double count = joint[(size_t)bx * bins + by];
            if (count <= 0.0) continue;
            double p = count * inv_total;
            double expected = (p_x[bx] * p_y[by]) * inv_total_sq;
            if (expected > 0.0) mi += p * log(p / expected);
        }
    }
    return mi;
}

static int or_cmp_double(const void* a, const void* b) {
    const double x = *(const double*)a, y = *(const double*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* Mutual information with QUANTILE bins on the interaction (no counterpart in the
 * reference, which bins equal-width only: gafime_core.cpp:200-226).  Definition used by
 * this library: sort the n values; the cut points are the order statistics
 * t_b = sorted[floor(b n / bins)] for b = 1 .. bins-1; the bin of x is the number of cut
 * points t_b <= x (ties share a bin, repeated cut points leave bins empty); a constant
 * interaction scores 0.  The y bins and the MI sum (natural log, bx-major, then by) are
 * those of mutual_info_from_vector (gafime_core.cpp:267-333). */
static double or_mutual_info_quantile(const double* x, int64_t n, int bins, const int32_t* y_bins,
                                      double* sorted, double* cuts, double* joint, double* p_x,
                                      double* p_y) {
    if (bins < 2 || n == 0) return 0.0;
    memcpy(sorted, x, (size_t)n * sizeof(double));
    qsort(sorted, (size_t)n, sizeof(double), or_cmp_double);
    if (sorted[0] == sorted[n - 1]) return 0.0;
    for (int b = 1; b < bins; ++b) cuts[b - 1] = sorted[(int64_t)b * n / bins];
    size_t b2 = (size_t)bins * (size_t)bins;
    memset(joint, 0, b2 * sizeof(double));
    memset(p_x, 0, (size_t)bins * sizeof(double));
    memset(p_y, 0, (size_t)bins * sizeof(double));
    for (int64_t i = 0; i < n; ++i) {
        /* number of cut points <= x[i] (upper bound in the sorted cuts) */
        int lo = 0, hi = bins - 1;
        while (lo < hi) {
            int mid = (lo + hi) / 2;
            if (cuts[mid] <= x[i]) lo = mid + 1; else hi = mid;
        }
        const int xb = lo, yb = y_bins[i];
        joint[(size_t)xb * bins + yb] += 1.0;
        p_x[xb] += 1.0;
        p_y[yb] += 1.0;
    }
    double inv_total = 1.0 / (double)n;
    double inv_total_sq = inv_total * inv_total;
    double mi = 0.0;
    for (int bx = 0; bx < bins; ++bx) {
        for (int by = 0; by < bins; ++by) {
            double count = joint[(size_t)bx * bins + by];
            if (count <= 0.0) continue;
            double p = count * inv_total;
            double expected = (p_x[bx] * p_y[by]) * inv_total_sq;
            if (expected > 0.0) mi += p * log(p / expected);
        }
    }
    return mi;
}

/* Quantile-bin mutual information of x = X[:,i] op X[:,j] (centred in fp64 when center is
 * set, else the fp32 kernel-API interaction) against equal-width y bins, per pair. */
int gafime_oracle_pair_mi_quantile(const float* X, int64_t ld, const float* y, int64_t n, int64_t f_count,
                                   const int32_t* pi, const int32_t* pj, int64_t n_pairs, int op, float eps,
                                   int center, int mi_bins, double* out_mi) {
    double* means = (double*)malloc((size_t)(f_count > 0 ? f_count : 1) * sizeof(double));
    double* yd = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
    int32_t* y_bins = (int32_t*)malloc((size_t)(n > 0 ? n : 1) * sizeof(int32_t));
    if (!means || !yd || !y_bins) {
        free(means); free(yd); free(y_bins);
        return -3;
    }
    if (center) gafime_oracle_column_means(X, ld, n, f_count, means);
    for (int64_t r = 0; r < n; ++r) yd[r] = (double)y[r];
    const int ready = or_build_bins(yd, n, mi_bins, y_bins);
    int status = 0;
#pragma omp parallel
    {
        double* inter = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
        double* sorted = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
        size_t nb = mi_bins >= 2 ? (size_t)mi_bins : 2;
        double* joint = (double*)malloc(nb * nb * sizeof(double));
        double* p_x = (double*)malloc(nb * sizeof(double));
        double* p_y = (double*)malloc(nb * sizeof(double));
        double* cuts = (double*)malloc(nb * sizeof(double));
        if (!inter || !sorted || !joint || !p_x || !p_y || !cuts) {
#pragma omp atomic write
            status = -3;
        } else {
#pragma omp for schedule(dynamic, 8)
            for (int64_t p = 0; p < n_pairs; ++p) {
                const float* ca = X + (int64_t)pi[p] * ld;
                const float* cb = X + (int64_t)pj[p] * ld;
                for (int64_t r = 0; r < n; ++r) {
                    if (center) {
                        double a = (double)ca[r] - means[pi[p]], b = (double)cb[r] - means[pj[p]];
                        double v;
                        switch (op) {
                            case OR_ADD: v = a + b; break;
                            case OR_SUB: v = a - b; break;
                            case OR_DIV: v = a / (fabs(b) < (double)eps ? copysign((double)eps, b) : b); break;
                            default: v = a * b;
                        }
                        inter[r] = v;
                    } else {
                        inter[r] = (double)or_combine(ca[r], cb[r], op, eps);
                    }
                }
                out_mi[p] = ready ? or_mutual_info_quantile(inter, n, mi_bins, y_bins, sorted, cuts, joint, p_x,
                                                            p_y)
                                  : 0.0;
            }
        }
        free(inter); free(sorted); free(joint); free(p_x); free(p_y); free(cuts);
    }
    free(means); free(yd); free(y_bins);
    return status;
}

/* Centred-product scores for pairs (i, j) as gafime_core.score_combos computes
 * them for 2-combos (gafime_core.cpp:531-618).  want_pearson / want_mi select
 * the metrics; out_pearson / out_mi receive one value per pair (either may be
 * NULL when not wanted).  X is column-major fp32 (exactly representable in
 * fp64, so it equals the reference's float64 input of the same values). */
int gafime_oracle_centred_scores(const float* X, int64_t ld, const float* y, int64_t n,
                                 int64_t f_count, const int32_t* pi, const int32_t* pj,
                                 int64_t n_pairs, int mi_bins, double* out_pearson,
                                 double* out_mi) {
    double* means = (double*)malloc((size_t)f_count * sizeof(double));
    double* yc = (double*)malloc((size_t)n * sizeof(double));
    double* yd = (double*)malloc((size_t)n * sizeof(double));
    int32_t* y_bins = (int32_t*)malloc((size_t)n * sizeof(int32_t));
    if (!means || !yc || !yd || !y_bins) {
        free(means); free(yc); free(yd); free(y_bins);
        return -3;
    }
    gafime_oracle_column_means(X, ld, n, f_count, means);
    /* gafime_core.cpp:486-497 */
    double sum_y = 0.0, sum_y2 = 0.0;
    for (int64_t r = 0; r < n; ++r) {
        yd[r] = (double)y[r];
        sum_y += yd[r];
        sum_y2 += yd[r] * yd[r];
    }
    double mean_y = (n == 0) ? 0.0 : sum_y / (double)n;
    for (int64_t r = 0; r < n; ++r) yc[r] = yd[r] - mean_y;
    double var_y = sum_y2 - sum_y * mean_y;
    int mi_ready = 0;
    if (out_mi) mi_ready = or_build_bins(yd, n, mi_bins, y_bins);

    int status = 0;
#pragma omp parallel
    {
        double* inter = (double*)malloc((size_t)n * sizeof(double));
        size_t nb = mi_bins >= 2 ? (size_t)mi_bins : 2;
        double* joint = (double*)malloc(nb * nb * sizeof(double));
        double* p_x = (double*)malloc(nb * sizeof(double));
        double* p_y = (double*)malloc(nb * sizeof(double));
        if (!inter || !joint || !p_x || !p_y) {
#pragma omp atomic write
            status = -3;
        } else {
#pragma omp for schedule(dynamic, 8)
            for (int64_t p = 0; p < n_pairs; ++p) {
                const float* ca = X + (int64_t)pi[p] * ld;
                const float* cb = X + (int64_t)pj[p] * ld;
                double ma = means[pi[p]], mb = means[pj[p]];
                double sum_x = 0.0, sum_x2 = 0.0, dot_xy = 0.0;
                for (int64_t r = 0; r < n; ++r) {
                    /* value = 1.0; value *= (a - ma); value *= (b - mb) */
                    double v = 1.0;
                    v *= ((double)ca[r] - ma);
                    v *= ((double)cb[r] - mb);
                    inter[r] = v;
                    sum_x += v;
                    sum_x2 += v * v;
                    dot_xy += v * yc[r];
                }
                if (out_pearson) out_pearson[p] = or_pearson_from_sums(sum_x, sum_x2, dot_xy, var_y, n);
                if (out_mi) {
                    out_mi[p] = (mi_ready && mi_bins >= 2)
                                    ? or_mutual_info(inter, n, mi_bins, y_bins, joint, p_x, p_y)
                                    : 0.0;
                }
            }
        }
        free(inter); free(joint); free(p_x); free(p_y);
    }
    free(means); free(yc); free(yd); free(y_bins);
    return status;
}

/* Mutual information of x = a op b for pairs (i, j), binned as gafime_core does
 * (y bins: build_bins, gafime_core.cpp:200-226; x bins and MI:
 * mutual_info_from_vector, gafime_core.cpp:267-333).
 *   center = 0: x = fl32(a op b), the kernel-API interaction (cpu_backend.cpp:87-103);
 *   center = 1: x = (a - mean_a) op (b - mean_b) in fp64 with fp64 column means in serial
 *               row order (gafime_core.cpp:134-150); for multiply this is the reference's
 *               centred product (gafime_core.cpp:571-577), the other operators extend it
 *               with the same divide rule as combine_cpu (copysign clamp at eps). */
int gafime_oracle_pair_mi(const float* X, int64_t ld, const float* y, int64_t n, int64_t f_count,
                          const int32_t* pi, const int32_t* pj, int64_t n_pairs, int op, float eps,
                          int center, int mi_bins, double* out_mi) {
    double* means = (double*)malloc((size_t)(f_count > 0 ? f_count : 1) * sizeof(double));
    double* yd = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
    int32_t* y_bins = (int32_t*)malloc((size_t)(n > 0 ? n : 1) * sizeof(int32_t));
    if (!means || !yd || !y_bins) {
        free(means); free(yd); free(y_bins);
        return -3;
    }
    if (center) gafime_oracle_column_means(X, ld, n, f_count, means);
    for (int64_t r = 0; r < n; ++r) yd[r] = (double)y[r];
    const int ready = or_build_bins(yd, n, mi_bins, y_bins);
    int status = 0;
#pragma omp parallel
    {
        double* inter = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
        size_t nb = mi_bins >= 2 ? (size_t)mi_bins : 2;
        double* joint = (double*)malloc(nb * nb * sizeof(double));
        double* p_x = (double*)malloc(nb * sizeof(double));
        double* p_y = (double*)malloc(nb * sizeof(double));
        if (!inter || !joint || !p_x || !p_y) {
#pragma omp atomic write
            status = -3;
        } else {
#pragma omp for schedule(dynamic, 8)
            for (int64_t p = 0; p < n_pairs; ++p) {
                const float* ca = X + (int64_t)pi[p] * ld;
                const float* cb = X + (int64_t)pj[p] * ld;
                for (int64_t r = 0; r < n; ++r) {
                    if (center) {
                        double a = (double)ca[r] - means[pi[p]], b = (double)cb[r] - means[pj[p]];
                        double v;
                        switch (op) {
                            case OR_ADD: v = a + b; break;
                            case OR_SUB: v = a - b; break;
                            case OR_DIV: v = a / (fabs(b) < (double)eps ? copysign((double)eps, b) : b); break;
                            default: v = a * b;
                        }
                        inter[r] = v;
                    } else {
                        inter[r] = (double)or_combine(ca[r], cb[r], op, eps);
                    }
                }
                out_mi[p] = ready ? or_mutual_info(inter, n, mi_bins, y_bins, joint, p_x, p_y) : 0.0;
            }
        }
        free(inter); free(joint); free(p_x); free(p_y);
    }
    free(means); free(yd); free(y_bins);
    return status;
}

/* Mutual information of each raw column against y: a one-feature combo of
 * gafime_core.score_combos scores the column's own values (gafime_core.cpp:558-568),
 * binned by mutual_info_from_vector (gafime_core.cpp:267-333). */
int gafime_oracle_unary_mi(const float* X, int64_t ld, const float* y, int64_t n, int64_t f_count,
                           int mi_bins, double* out_mi) {
    double* yd = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
    double* xd = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
    int32_t* y_bins = (int32_t*)malloc((size_t)(n > 0 ? n : 1) * sizeof(int32_t));
    size_t nb = mi_bins >= 2 ? (size_t)mi_bins : 2;
    double* joint = (double*)malloc(nb * nb * sizeof(double));
    double* p_x = (double*)malloc(nb * sizeof(double));
    double* p_y = (double*)malloc(nb * sizeof(double));
    int status = 0;
    if (!yd || !xd || !y_bins || !joint || !p_x || !p_y) {
        status = -3;
    } else {
        for (int64_t r = 0; r < n; ++r) yd[r] = (double)y[r];
        const int ready = or_build_bins(yd, n, mi_bins, y_bins);
        for (int64_t c = 0; c < f_count; ++c) {
            for (int64_t r = 0; r < n; ++r) xd[r] = (double)X[c * ld + r];
            out_mi[c] = ready ? or_mutual_info(xd, n, mi_bins, y_bins, joint, p_x, p_y) : 0.0;
        }
    }
    free(yd); free(xd); free(y_bins); free(joint); free(p_x); free(p_y);
    return status;
}

/* rankdata, gafime_core.cpp:156-177: stable ascending order, a run of equal values gets
 * the average 0-based rank 0.5 * (first + last).  Sorting (value, index) pairs gives the
 * stable order. */
typedef struct {
    double v;
    int64_t i;
} OrRankItem;

static int or_rank_cmp(const void* pa, const void* pb) {
    const OrRankItem* a = (const OrRankItem*)pa;
    const OrRankItem* b = (const OrRankItem*)pb;
    if (a->v < b->v) return -1;
    if (a->v > b->v) return 1;
    return (a->i > b->i) - (a->i < b->i);
}

static void or_rankdata(const double* v, int64_t n, OrRankItem* items, double* out) {
    for (int64_t i = 0; i < n; ++i) {
        items[i].v = v[i];
        items[i].i = i;
    }
    qsort(items, (size_t)n, sizeof(OrRankItem), or_rank_cmp);
    int64_t i = 0;
    while (i < n) {
        int64_t j = i + 1;
        while (j < n && items[j].v == items[i].v) ++j;
        double avg = 0.5 * (double)(i + j - 1);
        for (int64_t k = i; k < j; ++k) out[items[k].i] = avg;
        i = j;
    }
}

/* Spearman of each combo against y as gafime_core.score_combos computes it
 * (gafime_core.cpp:503-517 target ranks, 595-607 the metric).  Combo c is column a[c]
 * alone when b[c] < 0, else x = (a - mean_a) op (b - mean_b) in fp64 (center = 1) or
 * fl32(a op b) (center = 0), with the operators and divide rule of gafime_oracle_pair_mi. */
int gafime_oracle_spearman(const float* X, int64_t ld, const float* y, int64_t n, int64_t f_count,
                           const int32_t* ca_idx, const int32_t* cb_idx, int64_t n_combos, int op,
                           float eps, int center, double* out) {
    size_t nn = (size_t)(n > 0 ? n : 1);
    double* means = (double*)malloc((size_t)(f_count > 0 ? f_count : 1) * sizeof(double));
    double* yd = (double*)malloc(nn * sizeof(double));
    double* yr = (double*)malloc(nn * sizeof(double));
    double* ycr = (double*)malloc(nn * sizeof(double));
    OrRankItem* items = (OrRankItem*)malloc(nn * sizeof(OrRankItem));
    double* xv = (double*)malloc(nn * sizeof(double));
    double* xr = (double*)malloc(nn * sizeof(double));
    int status = 0;
    if (!means || !yd || !yr || !ycr || !items || !xv || !xr) {
        status = -3;
        goto done;
    }
    gafime_oracle_column_means(X, ld, n, f_count, means);
    for (int64_t r = 0; r < n; ++r) yd[r] = (double)y[r];
    or_rankdata(yd, n, items, yr);
    {
        double sum_r = 0.0, sum_r2 = 0.0;
        for (int64_t r = 0; r < n; ++r) {
            sum_r += yr[r];
            sum_r2 += yr[r] * yr[r];
        }
        double mean_r = n == 0 ? 0.0 : sum_r / (double)n;
        for (int64_t r = 0; r < n; ++r) ycr[r] = yr[r] - mean_r;
        double var_y_rank = sum_r2 - (sum_r * mean_r);
        for (int64_t c = 0; c < n_combos; ++c) {
            const float* pa = X + (int64_t)ca_idx[c] * ld;
            const float* pb = cb_idx[c] >= 0 ? X + (int64_t)cb_idx[c] * ld : NULL;
            for (int64_t r = 0; r < n; ++r) {
                if (!pb) {
                    xv[r] = (double)pa[r];
                } else if (center) {
                    double a = (double)pa[r] - means[ca_idx[c]], b = (double)pb[r] - means[cb_idx[c]];
                    double v;
                    switch (op) {
                        case OR_ADD: v = a + b; break;
                        case OR_SUB: v = a - b; break;
                        case OR_DIV: v = a / (fabs(b) < (double)eps ? copysign((double)eps, b) : b); break;
                        default: v = 1.0; v *= a; v *= b;
                    }
                    xv[r] = v;
                } else {
                    xv[r] = (double)or_combine(pa[r], pb[r], op, eps);
                }
            }
            or_rankdata(xv, n, items, xr);
            double s1 = 0.0, s2 = 0.0, s3 = 0.0;
            for (int64_t r = 0; r < n; ++r) {
                s1 += xr[r];
                s2 += xr[r] * xr[r];
                s3 += xr[r] * ycr[r];
            }
            out[c] = or_pearson_from_sums(s1, s2, s3, var_y_rank, n);
        }
    }
done:
    free(means); free(yd); free(yr); free(ycr); free(items); free(xv); free(xr);
    return status;
}

/* Interaction materialiser, src/cuda/kernels.cu:1646-1676 (row-major X and out). */
void gafime_oracle_feature_interaction(const float* X, const float* means, float* out,
                                       const int32_t* idx, const int32_t* off, int32_t n,
                                       int32_t f, int32_t n_combos) {
    for (int32_t i = 0; i < n; ++i) {
        for (int32_t c = 0; c < n_combos; ++c) {
            const int32_t start = off[c], end = off[c + 1], size = end - start;
            float prod = 1.0f;
            for (int32_t j = start; j < end; ++j) {
                const int32_t feat = idx[j];
                if (feat < 0 || feat >= f) continue;
                const float v = X[(int64_t)i * f + feat];
                if (size == 1) prod = v;
                else prod *= (v - means[feat]);
            }
            out[(int64_t)i * n_combos + c] = prod;
        }
    }
}

/* Unary operators, cpu_backend.cpp:30-77. */
static inline float or_unary(float x, int op) {
    switch (op) {
        case 1: return logf(fabsf(x) + 1e-8f);
        case 2: return expf(fminf(fmaxf(x, -20.0f), 20.0f));
        case 3: return sqrtf(fabsf(x));
        case 4: {
            float c = fminf(fmaxf(x, -10.0f), 10.0f);
            float e2 = expf(2.0f * c);
            return (e2 - 1.0f) / (e2 + 1.0f);
        }
        case 5: {
            float c = fminf(fmaxf(x, -20.0f), 20.0f);
            return 1.0f / (1.0f + expf(-c));
        }
        case 6: return x * x;
        case 7: return -x;
        case 8: return fabsf(x);
        case 9: return 1.0f / (fabsf(x) < 1e-8f ? copysignf(1e-8f, x) : x);
        case 10: return x * x * x;
        case 11:
        case 12: return NAN;
        default: return x;
    }
}

/* combine_cpu with MAX / MIN, cpu_backend.cpp:85-103. */
static inline float or_combine_chain(float a, float b, int t) {
    switch (t) {
        case 4: return fmaxf(a, b);
        case 5: return fminf(a, b);
        default: return or_combine(a, b, t, 1e-8f);
    }
}

/* Chain statistics, cpu_backend.cpp:229-295: out = {train n, sx, sy, sxx, syy, sxy, the same
 * for rows whose mask equals val_fold_id}. */
void gafime_oracle_chain_stats(const float* const* cols, const float* y, const uint8_t* mask, int64_t n,
                               const int* ops, int arity, const int* inter, int val_fold_id, double* out) {
    for (int m = 0; m < 12; ++m) out[m] = 0.0;
    for (int64_t r = 0; r < n; ++r) {
        float x = or_combine_chain(or_unary(cols[0][r], ops[0]), or_unary(cols[1][r], ops[1]), inter[0]);
        for (int k = 2; k < arity; ++k) x = or_combine_chain(x, or_unary(cols[k][r], ops[k]), inter[k - 1]);
        const float yv = y[r];
        if (isnan(x) || isnan(yv)) continue;
        const double xd = x, yd = yv;
        double* o = out + (mask[r] == val_fold_id ? 6 : 0);
        o[0] += 1.0;
        o[1] += xd;
        o[2] += yd;
        o[3] += xd * xd;
        o[4] += yd * yd;
        o[5] += xd * yd;
    }
}
