/* rfx_b200 — B200-native forest growth and proximity for RFX-Fuse (C ABI).
 *
 * Replaces the reference's GPU seam `gpu_growtree_batch(...)` (include/rf_growtree.hpp:45,
 * cuda/rf_growtree.cu:3006, called from RandomForest::fit_batch_gpu,
 * src/rf_random_forest.cpp:2000-2464) and the CPU per-tree loop it stands in for
 * (RandomForest::grow_tree_single, src/rf_random_forest.cpp:1278-1997).  The results are
 * those of the reference CPU path: bootstrap (src/rf_bootstrap.cpp:15-84), quantile binning
 * (src/rf_histogram.cpp:13-160), histogram growth (src/rf_growtree.cpp:616-1161), OOB drop
 * (src/rf_testreebag.cpp:13-125), permutation importance (src/rf_varimp.cpp:218-597),
 * proximity (src/rf_proximity.cpp:99-230) and finishprox (src/rf_finishprox.cpp:12-74).
 *
 * Conventions: plain pointers and sizes only.  Host pointers unless the name ends in
 * `_dev`.  Every function returns RFX_OK (0) or a negative RFX_ERR_* code and never
 * throws; rfx_last_error() gives the message of the calling thread's last failure.  A
 * context is bound to one CUDA device and is not re-entrant.
 */
#ifndef RFX_B200_H
#define RFX_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define RFX_ABI_VERSION 5

enum {
    RFX_OK = 0,
    RFX_ERR_ARG = -1,          /* invalid argument */
    RFX_ERR_CUDA = -2,         /* CUDA runtime failure (message has the CUDA error) */
    RFX_ERR_OOM = -3,          /* device allocation failed */
    RFX_ERR_UNSUPPORTED = -4,  /* option outside what the device path implements */
    RFX_ERR_STATE = -5,        /* call order violated (e.g. grow before load) */
    RFX_ERR_DEVICE = -6,       /* a kernel reported an internal consistency error */
    RFX_ERR_CANCELLED = -7     /* the progress callback asked to stop */
};

enum { RFX_TASK_CLASSIFICATION = 0, RFX_TASK_REGRESSION = 1, RFX_TASK_UNSUPERVISED = 2 };

/* Effective fit parameters (already resolved the way the estimator wrappers resolve them:
 * python/randomforest_py.cpp:1270-1320, 1404-1411, 3123-3124, 3232-3234, 4687-4692;
 * include/rf_config.hpp:15-32). */
typedef struct {
    int task;               /* RFX_TASK_* */
    int n;                  /* rows supplied (real rows for unsupervised) */
    int p;                  /* features */
    int mtry;               /* features drawn (with replacement) per searched node */
    int minndsize;          /* split needs >= minndsize rows (2x for regression) */
    int maxnode;            /* node cap per tree */
    int iseed;              /* grower seed base: tree t draws from MT19937(iseed + t) */
    int boot_seed;          /* bootstrap seed base: MT19937(boot_seed + t); 12345 in the reference */
    int nbins;              /* histogram bins, <= 256 */
    int maxcat;             /* the estimator's maxcat (category bound of importance walks) */
    int compute_importance; /* permutation importance (rf_varimp.cpp) */
    int compute_proximity;  /* OOB x in-bag leaf co-membership counts */
    int prox_rows;          /* proximity covers rows [0, prox_rows); 0 = all grown rows */
    int batch_trees;        /* trees grown concurrently on the device; 0 = automatic */
    int keep_tree_oob;      /* keep per-tree OOB predictions for rfx_oob_fold (regression) */
    int lowrank_rank;       /* > 0 with compute_proximity: low-rank mode (use_qlora=True,
                               include/rf_proximity_lowrank.hpp:27-439).  No dense counts are
                               kept; every tree's leaf groups are stored instead for
                               rfx_lowrank_build.  Rank <= 64. */
    int keep_forest;        /* keep the grown trees on the device (packed) for rfx_predict */
    int keep_leaves;        /* compute_leaf_assignments: keep every row's terminal node per
                               tree and the per-tree OOB flags on the device (rfx_leaf_*) */
    int keep_trees;         /* keep the tree arrays (reference layout) of every tree grown
                               since the load on the device, for rfx_get_trees */
} rfx_fit_params;

typedef struct {
    const float* X;              /* [n x p] row-major */
    const int* y_class;          /* [n] class labels (any integers), classification only */
    const float* y_reg;          /* [n] targets, regression only */
    const float* sample_weights; /* [n] bootstrap weights or NULL (uniform) */
    const int* cat;              /* [p] 1 = quantitative, k > 1 = k categories; NULL = all 1 */
    const float* classwt;        /* [nclass] OOB vote weights or NULL */
} rfx_inputs;

/* Per-tree arrays of one rfx_grow call, [ntree x maxnode] (treemap [ntree x 2*maxnode]),
 * laid out like the reference RandomForest members (src/rf_random_forest.cpp:358-452).
 * Any pointer may be NULL. */
typedef struct {
    int* nodestatus; int* bestvar; float* xbestsplit; int* treemap; int* nodeclass;
    int* nnode; float* nodepred; float* tnodewt;
    int* nin;        /* [ntree x N] bootstrap multiplicities */
    int* oob_leaf;   /* [ntree x N] terminal node of OOB rows, in-bag rows -1 */
    float* tree_rr;  /* [ntree x p] per-tree importance rr (0 where unused) */
    uint8_t* tree_used; /* [ntree x p] 1 where rr enters avimp */
} rfx_trees;

/* Forest accumulators after all rfx_grow calls since rfx_load (N = grown rows: n, or 2n
 * for unsupervised).  Any pointer may be NULL. */
typedef struct {
    int nclass;      /* out: classes (1 for regression, 2 for unsupervised) */
    int N;           /* out: grown rows */
    int* nout;       /* [N] times each row was out of bag */
    int* votes;      /* [N x nclass] integer OOB vote counts */
    float* q;        /* [N x nclass] raw OOB vote sums (classwt-weighted), reference q_ */
    float* oob_sum;  /* [N] regression: sum of OOB predictions in tree order */
    float* avimp;    /* [p] summed importance in tree order */
    float* sqsd;     /* [p] summed squared importance in tree order */
    int* labels;     /* [N] 0-based labels the trees were grown on (classification) */
} rfx_accum;

const char* rfx_last_error(void);
int rfx_abi_version(void);
int rfx_device_count(void);

/* Device memory of destroyed contexts is kept in a process-wide cache per device and reused
 * by the next contexts (each estimator fit makes a new context).  No counterpart in the
 * reference, whose CPU path allocates host memory per fit.  rfx_cached_bytes reports the
 * bytes cached for `device` (-1: all devices); rfx_empty_cache frees them (another library
 * in the process that needs the memory calls it first).  Contexts alive keep their own
 * buffers either way. */
long long rfx_cached_bytes(int device);
int rfx_empty_cache(int device);

/* Context bound to CUDA device `device`; NULL on failure (see rfx_last_error). */
void* rfx_create(int device);
void rfx_destroy(void* ctx);

/* Upload inputs, bin features on the device and reset all accumulators. */
int rfx_load(void* ctx, const rfx_fit_params* prm, const rfx_inputs* in);

/* Grow trees [tree_begin, tree_begin + ntree) on the loaded data and fold their OOB votes,
 * predictions, importance and proximity into the accumulators.  Successive calls must
 * cover increasing tree ids for the float folds to follow the reference's tree order.
 * `out` (may be NULL) receives the per-tree arrays of these trees. */
int rfx_grow(void* ctx, int tree_begin, int ntree, rfx_trees* out);

/* Start a new forest on the loaded dataset: zero the forest-level accumulators (OOB counts,
 * votes or OOB prediction sums, importance, proximity counts) and forget the stored trees,
 * keeping the binned data and the buffers.  The reference builds a new RandomForest per fit
 * (src/rf_random_forest.cpp:521, 691, 988); this is its counterpart for repeated fits on
 * device-resident data. */
int rfx_reset_forest(void* ctx);

/* Progress of rfx_grow / rfx_fit, the reference's progress_callback_(itree + 1, ntree)
 * (src/rf_random_forest.cpp:600-601; the wrapper drives tqdm from it,
 * python/randomforest_py.cpp:1560-1690).  Called on the caller's thread after every batch
 * of trees with the trees grown so far by this call and the call's total; a nonzero return
 * stops the call with RFX_ERR_CANCELLED after the batch.  NULL removes the callback. */
typedef int (*rfx_progress_fn)(void* user, int trees_done, int ntree);
int rfx_set_progress(void* ctx, rfx_progress_fn fn, void* user);

/* Tree arrays of the trees [tree_begin, tree_begin + count) grown since rfx_load (or
 * rfx_reset_forest), by position in growth order, from the device tree store that
 * keep_trees fills (the reference's RandomForest members, src/rf_random_forest.cpp:358-452:
 * the caller's host arrays).  Only nodestatus .. tnodewt are read from `out`; NULL
 * pointers are skipped.  RFX_ERR_STATE when the fit did not keep its trees. */
int rfx_get_trees(void* ctx, int tree_begin, int count, rfx_trees* out);

/* Copy the accumulators to the host. */
int rfx_results(void* ctx, rfx_accum* res);

/* rfx_load + rfx_grow(0, ntree) + rfx_results. */
int rfx_fit(void* ctx, const rfx_fit_params* prm, const rfx_inputs* in, int ntree,
            rfx_trees* trees, rfx_accum* res);

/* Proximity accumulation target: int32 upper triangle (i < j) of the OOB x in-bag
 * co-membership counts C_ij = P_ij + P_ji over rows [0, R), packed row by row
 * (index i*(2R-i-1)/2 + j-i-1), length R(R-1)/2.  The caller owns the device memory (so
 * that it can reduce it across GPUs with NCCL); NULL makes the context allocate its own.
 * Must be called after rfx_load. */
int rfx_set_prox_buffer(void* ctx, int* upper_dev, int64_t len);
/* Device pointer and length of the current proximity counts. */
int rfx_get_prox_buffer(void* ctx, int** upper_dev, int64_t* len);
/* Device pointers of the nout [N] and vote [N x nclass] accumulators (NCCL all-reduce). */
int rfx_get_vote_buffers(void* ctx, int** nout_dev, int** votes_dev);

/* finishprox of rows [row_begin, row_end) of the R x R matrix from upper-triangle counts
 * and nout (both device): out_dev[(i-row_begin)*R + j] = float32 of the reference's
 * double result (diag 1).  Stream-ordered on the context's stream. */
int rfx_prox_finish(void* ctx, const int* upper_dev, const int* nout_dev, int R,
                    int row_begin, int row_end, float* out_dev);

/* Finished values of the packed upper-triangle elements [elem_begin, elem_begin + elem_count)
 * of the R x R proximity (element e = (i, j), i < j, e = i (2R - i - 1) / 2 + j - i - 1):
 * upper_dev and out_dev hold that slice (index e - elem_begin), nout_dev all R counts.  The
 * finishprox arithmetic of rfx_prox_finish (src/rf_finishprox.cpp:12-74) needs only C_ij and
 * the two row scales, so each rank of a tree-sharded fit finishes the slice its NCCL
 * reduce-scatter left it.  Device pointers; returns after the slice is written. */
int rfx_prox_finish_packed(void* ctx, const int* upper_dev, int64_t elem_begin, int64_t elem_count,
                           const int* nout_dev, int R, float* out_dev);

/* Same as rfx_prox_finish on the context's own counts and nout, rows [row_begin, row_end)
 * of the R x R matrix written to host memory out_host[(i-row_begin)*R + j]; processed in
 * row blocks so the device scratch stays bounded (python/randomforest_py.cpp:2129-2155). */
int rfx_prox_dense(void* ctx, int row_begin, int row_end, float* out_host);

/* Allocation-free variant of rfx_prox_dense (no counterpart in the reference).
 * For callers that must not allocate device memory -- e.g. a serving process or a host
 * application whose memory pool owns the whole device budget, where a cudaMalloc would
 * fail or stall the device.  It needs no context: the caller passes the upper-triangle
 * counts and nout (device pointers, e.g. from rfx_get_prox_buffer / rfx_get_vote_buffers or
 * its own NCCL-reduced copies), the row range, the host destination and a CUDA stream
 * (NULL = legacy default stream); the current device is used.  Finished rows are staged in
 * one fixed device array of RFX_STATIC_SCRATCH_FLOATS floats (16 MiB) that every GPU which
 * loads the library keeps until the process exits; R must not exceed that size (one row
 * has to fit), otherwise RFX_ERR_ARG.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress), so make that first call before any stream capture;
 * with lazy module loading (CUDA's default) that first call is also when the 16 MiB are
 * reserved, so a caller whose pool takes the whole budget should make it (a warm-up call)
 * at start-up.  The address is kept for the life of the process: after cudaDeviceReset, or
 * any teardown of the device's primary context, the kept address is stale and the function
 * must not be called again in that process.
 * No cudaMalloc / cudaFree is called.  All calls share the array, which keeps the last
 * call's rows; it is fully rewritten before each use, so nothing needs clearing, but calls
 * that overlap on the GPU (other threads or streams) race on it.  Returns after the rows
 * are on the host. */
#define RFX_STATIC_SCRATCH_FLOATS (4 * 1024 * 1024)
int rfx_prox_dense_static(const int* upper_dev, const int* nout_dev, int R, int row_begin,
                          int row_end, float* out_host, void* stream);

/* Regression, keep_tree_oob: vec_dev[i] <- fold of the per-tree OOB predictions of the
 * trees grown so far, in tree order, starting from the incoming value (device, [N]). */
int rfx_oob_fold(void* ctx, float* vec_dev);

/* q_dev[i] = classwt[c] added votes_dev[i] times (float, sequential), the reference's
 * vote accumulation (src/rf_random_forest.cpp:1500-1520); classwt NULL = 1.0. */
int rfx_votes_to_q(void* ctx, const int* votes_dev, const float* classwt, int N, int nclass,
                   float* q_dev);

/* Stream-ordered device-to-host copy of `bytes` from src_dev (e.g. the proximity counts). */
int rfx_copy_to_host(void* ctx, void* dst_host, const void* src_dev, size_t bytes);

/* Measurement.  Counters since the last rfx_reset_stats: kernels launched by the library,
 * and, while profiling is on, the CUDA-event time of the histogram kernels of every level
 * together with the algorithmic bytes they read (sum over searched nodes of
 * rows * (mtry + target bytes)), and of the proximity kernel with the pairs it added. */
typedef struct {
    int64_t kernel_launches;
    int64_t hist_launches;
    double hist_ms;
    double hist_bytes;
    int64_t levels;
    int64_t trees;
    double prox_pair_updates;  /* OOB x in-bag pairs added to the proximity counts */
    double prox_ms;            /* CUDA-event time of the proximity kernel (profiling on) */
    double topk_ms;            /* CUDA-event time of the low-rank product kernel (profiling on) */
    int64_t topk_tiles;        /* 128 x 256 x 64 product tiles it multiplied */
    double sketch_ms;          /* CUDA-event time of the low-rank sketch passes (profiling on) */
    double sketch_bytes;       /* their algorithmic bytes: per tree 2 R W 4 + 6 R */
} rfx_stats;
int rfx_get_stream(void* ctx, void** stream);   /* the context's cudaStream_t */
int rfx_set_profiling(void* ctx, int on);
int rfx_get_stats(void* ctx, rfx_stats* out);
int rfx_reset_stats(void* ctx);

/* ---- Prediction of new rows -----------------------------------------------------------
 * Replaces RandomForest::predict_classification / predict_proba (new-data branch) and
 * predict_regression (src/rf_random_forest.cpp:3403-3590, 3863-3945).  A fit with
 * keep_forest leaves its trees on the device; rfx_load_forest puts any forest there (e.g. the
 * arrays of a saved model).  Walks follow the reference exactly: at most maxnode steps per
 * tree; cat == 1 features go left when x <= xbestsplit; any other feature takes the
 * categorical branch, jcat = (int)(x + 0.5) in [0, cat) going right (catgoleft is empty for
 * histogram-grown trees) and any other jcat voting class 0 (regression: the root's value).
 * Classification folds classwt-weighted float votes in tree order (first maximum wins;
 * probabilities are votes / their sum); regression averages the values in tree order. */
typedef struct {
    int task;                 /* RFX_TASK_CLASSIFICATION or RFX_TASK_REGRESSION */
    int ntree, maxnode, nclass, p;
    const int* nodestatus;    /* [ntree][maxnode] */
    const int* bestvar;
    const float* xbestsplit;
    const int* treemap;       /* [ntree][2 * maxnode] */
    const int* nodeclass;     /* classification */
    const float* nodepred;    /* regression */
    const int* cat;           /* [p] */
    const float* classwt;     /* [nclass] or NULL (votes of 1) */
} rfx_forest;
int rfx_load_forest(void* ctx, const rfx_forest* forest);

/* X_host [n][p] row-major float; outputs may be NULL: class_out [n] (0-based class),
 * proba_out [n][nclass], value_out [n] (regression). */
int rfx_predict(void* ctx, const float* X_host, int n, int p, int* class_out, float* proba_out,
                float* value_out);

/* ---- Leaf assignments, top-k similar rows, outliers -----------------------------------
 * A fit with keep_leaves stores, per tree, every grown row's terminal node as int16 (the
 * reference's leaf_assignments_ [tree][sample], src/rf_random_forest.cpp:1543-1610, found by
 * walking the row down the tree like find_terminal_node, :3724-3770) and which rows were OOB
 * (oob_trees_, :1577-1590).  Numeric features only (RFX_ERR_UNSUPPORTED at fit time when a
 * categorical feature is present).  The queries below follow
 * include/rf_random_forest.hpp:296-365. */
/* get_leaf_assignments (python/randomforest_py.cpp:2373-2393): out [ntree][N] int16, N = the
 * grown rows (2n for unsupervised); out may be NULL to read the shape only. */
int rfx_leaf_assignments(void* ctx, int16_t* out, int* ntree_out, int* nrows_out);
/* build_inverted_leaf_index (src/rf_random_forest.cpp:4644-4675): rows grouped by (tree, leaf),
 * ascending inside a group.  The queries build it on first use, like the reference's bindings. */
int rfx_leaf_index(void* ctx);
/* get_top_k_similar (src/rf_random_forest.cpp:4677-4787) for nq training rows: counts of the
 * trees where the query was OOB and the row shares its leaf, the nonzero ones ranked with the
 * reference's std::partial_sort (descending count); similarity = count / (query's OOB trees).
 * idx_out / sim_out [nq][k]; counts_out[q] = entries written (0: no OOB tree, no match, or an
 * invalid query -- the reference returns an empty list). */
int rfx_leaf_top_k_similar(void* ctx, const int* queries, int nq, int k, int exclude_self,
                           int* idx_out, float* sim_out, int* counts_out);
/* compute_proximity_from_leaves (src/rf_random_forest.cpp:4605-4642): matches over the trees
 * where row i was OOB / their number; 0 when unavailable or out of range. */
int rfx_leaf_proximity(void* ctx, int i, int j, float* out);
/* predict_leaf_assignments (src/rf_random_forest.cpp:4789-4850) on the device forest (fit with
 * keep_forest): X_host [n][p], out [n][ntree] int16.  A node whose feature is out of range, or a
 * categorical value outside [0, cat), keeps the walk where it is (the reference's loop then
 * runs out its maxnode steps on that node). */
int rfx_predict_leaves(void* ctx, const float* X_host, int n, int p, int16_t* out);
/* predict_top_k_similar (python/randomforest_py.cpp:2496-2560): for each new row the fraction
 * of all trees where a training row shares its leaf, top k by std::partial_sort over every
 * training row (the reference's tie order); idx_out / sim_out [n][k], k <= N. */
int rfx_predict_top_k_similar(void* ctx, const float* X_host, int n, int p, int k, int* idx_out,
                              float* sim_out);
/* select_outlier_anchors (src/rf_random_forest.cpp:4305-4386): method 0 "random" (std::mt19937
 * (iseed) shuffle of 0..N-1), 1 "diverse" (start at a uniform draw, then repeatedly the first
 * row of least leaf proximity to the anchors so far); n_anchors >= N gives all rows.
 * anchors_out [min(n_anchors, N)], count_out = entries. */
int rfx_leaf_select_anchors(void* ctx, int n_anchors, int method, uint32_t iseed, int* anchors_out,
                            int* count_out);
/* compute_outlier_scores (src/rf_random_forest.cpp:4110-4277).  mode 0 "full": raw = (N - 1) /
 * sum over the other rows of (shared trees / ntree)^2 over all trees; mode 1 "greedy": raw =
 * n_anchors / the same sum over `anchors` (skipping the row itself).  Scores = (raw - median) /
 * MAD, per class when labels (0-based, [N]) are given, else over all rows.  raw_out may be NULL.
 * Greedy is the reference's arithmetic exactly; full sums the squares exactly in integers and
 * rounds once (the reference adds float terms in hash-map order). */
int rfx_leaf_outlier_scores(void* ctx, int mode, const int* anchors, int n_used, int n_anchors,
                            const int* labels, float* scores_out, float* raw_out);
/* predict_outlier_scores (src/rf_random_forest.cpp:5210-5330; python/randomforest_py.cpp:
 * 2649-2684) for new rows X_host [n][p]: proximity to every training row over all trees; raw =
 * m / sum of squares over the positive proximities (mode 0 "full": all, in row order; mode 1
 * "greedy": the n_anchors largest); normalised with the (median, MAD) of the last
 * rfx_leaf_outlier_scores (classes [n] = predicted 0-based classes for per-class statistics,
 * or NULL for the global ones).  RFX_ERR_STATE before any training outlier scores. */
int rfx_predict_outlier_scores(void* ctx, const float* X_host, int n, int p, int mode,
                               int n_anchors, const int* classes, float* scores_out);
/* compute_outliers' ranking (src/rf_random_forest.cpp:4279-4303): std::sort of (index, score)
 * by score descending, first k.  Host only. */
int rfx_rank_scores_desc(const float* scores, int n, int k, int* idx_out, float* val_out);

/* ---- Proximity-weighted imputation ---------------------------------------------------
 * One round of rfx_impute_proximity's fill (python/rfx_impute.py:730-775, aggregation
 * 'mean', top_k None) from this context's dense proximity counts (a fit over n rows with
 * compute_proximity; n == its proximity rows).  xc_host [p][n] column-major current values,
 * miss_host [p][n] (1 = missing in the original data), is_cat_host [p]; cells_host
 * [ncells][2] (row, column) of the cells to fill, sorted by row; out_host [ncells] the new
 * value, or NaN where no other observed row has positive proximity (the reference keeps
 * the old value).  Continuous: proximity-weighted mean with the weights normalised first;
 * categorical: the value with the largest proximity sum (ascending values, first maximum);
 * every sum is numpy's pairwise float32 summation, so the values are the reference's, bit
 * for bit. */
int rfx_impute_round(void* ctx, const float* xc_host, const uint8_t* miss_host,
                     const uint8_t* is_cat_host, int n, int p, const int* cells_host, int ncells,
                     float* out_host);

/* Aggregations of rfx_impute_round_ex (rfx_impute_proximity's `aggregation`). */
#define RFX_IMPUTE_MEAN 0   /* 'mean' / 'weighted_mean' */
#define RFX_IMPUTE_MEDIAN 1 /* 'median': np.median; categorical: the most frequent value */

/* rfx_impute_round with the reference's top_k and aggregation (python/rfx_impute.py:744-762).
 * top_k -1 = None (all qualifying rows, row order); top_k >= 0: when more rows qualify, the
 * top_k by proximity (0: all of them) in ascending (proximity, row) order.  The reference
 * orders them with np.argsort's default sort, whose order among equal proximities depends
 * on numpy's sort implementation; here it is the stable one (ties by ascending row).
 * aggregation RFX_IMPUTE_MEAN or RFX_IMPUTE_MEDIAN.  rfx_impute_round(...) equals
 * rfx_impute_round_ex(..., -1, RFX_IMPUTE_MEAN, out_host). */
int rfx_impute_round_ex(void* ctx, const float* xc_host, const uint8_t* miss_host,
                        const uint8_t* is_cat_host, int n, int p, const int* cells_host,
                        int ncells, int top_k, int aggregation, float* out_host);

/* ---- Low-rank proximity (use_qlora=True, quant_mode="int8") --------------------------
 * Replaces LowRankProximityMatrix (include/rf_proximity_lowrank.hpp:27-439,
 * cuda/rf_proximity_lowrank.cu:414-1340) and get_lowrank_factors
 * (src/rf_random_forest.cpp:4562-4603, python/randomforest_py.cpp:2183-2223).  S is the
 * finishprox'd proximity of rows [0, R) (S_ij = C_ij (1/nout_i + 1/nout_j) / 4, S_ii = 1,
 * C the OOB x in-bag co-membership counts of the trees grown so far).  The factors A
 * ([R][rank]) give S ~ A A^T: a randomized range finder on S applied through per-leaf sums
 * (C is never formed), Cholesky-QR, a Jacobi eigensolve of the projected matrix and the
 * top-`rank` non-negative eigenpairs, then per-row symmetric int8 quantisation
 * (A_i = scale_i * q_i). */

/* Sum `count` floats of buf_dev over all processes in place (e.g. an NCCL all-reduce);
 * return 0 on success.  Called on the caller's thread with the context's stream idle. */
typedef int (*rfx_reduce_fn)(void* user, float* buf_dev, int64_t count);

/* Build the factors from the stored trees.  oversample extra sketch columns (rank +
 * oversample <= 96), power_iters extra passes, seed of the random test matrix.  nout_dev
 * (device, [R]) overrides the context's OOB counts (the all-reduced counts of a sharded
 * fit); reduce (may be NULL) sums every sketch pass over the processes that hold the other
 * trees.  Costs (power_iters + 2) passes over the stored trees. */
int rfx_lowrank_build(void* ctx, int rank, int oversample, int power_iters, uint64_t seed,
                      const int* nout_dev, rfx_reduce_fn reduce, void* reduce_user);

/* Use caller-supplied factors (no reference counterpart; e.g. factors saved from an earlier
 * fit, or built by another process): q_host [rows][rank] int8 in [-127, 127], scale_host
 * [rows] finite, >= 0.  No fit is needed; rfx_lowrank_topk / _product / _factors then
 * work on these rows. */
int rfx_lowrank_set_factors(void* ctx, const int8_t* q_host, const float* scale_host, int rows,
                            int rank);

/* The factors: A_host [R][rank] dequantised float (may be NULL), q_host [R][rank] int8
 * (may be NULL), scale_host [R] (may be NULL); *rank_out = rank, *rows_out = R. */
int rfx_lowrank_factors(void* ctx, float* A_host, int8_t* q_host, float* scale_host,
                        int* rank_out, int* rows_out);

/* Top-k neighbours of rows [row_begin, row_end) under the quantised product
 * P_ij = (dot(q_i, q_j) * scale_i) * scale_j, j != i, ordered by value descending then
 * index ascending; k <= 64.  idx_host / val_host are [rows][k]; slots beyond R - 1
 * neighbours hold -1 / -inf.  The product runs on the tensor cores (tcgen05, bf16 operands
 * holding the int8 values exactly, fp32 accumulation) with the selection fused into the
 * accumulator read-out, so P is never written. */
int rfx_lowrank_topk(void* ctx, int k, int row_begin, int row_end, int* idx_host,
                     float* val_host);

/* The same top-k for part `part` of `nparts` equal shares of the product's internal row
 * order (rows by descending scale_i |q_i|; a contiguous share of that order is a
 * contiguous share of the kernel's work, unlike a range of row ids): rows_host [rows] gets
 * the original row ids, idx_host / val_host [rows][k] their results.  *nrows_out = rows;
 * with rows_host NULL only *nrows_out is set.  The shares of all parts cover every row once
 * (how a sharded fit splits the top-k over its GPUs). */
int rfx_lowrank_topk_part(void* ctx, int k, int part, int nparts, int* rows_host, int* idx_host,
                          float* val_host, int* nrows_out);

/* Rows [row_begin, row_end) of P (same kernel, every value written; diagonal included):
 * the reconstructed approximate proximity, out_host [rows][R]. */
int rfx_lowrank_product(void* ctx, int row_begin, int row_end, float* out_host);

/* Y_dev = S X_dev for the trees stored in low-rank mode (this context's trees only), X and
 * Y device [R][ncols] row-major, ncols <= 128; nout_dev as in rfx_lowrank_build. */
int rfx_prox_apply(void* ctx, const float* X_dev, int ncols, const int* nout_dev, float* Y_dev);

/* Wait for the context's stream. */
int rfx_sync(void* ctx);

#ifdef __cplusplus
}
#endif
#endif
