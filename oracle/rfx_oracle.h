/* TEST INFRASTRUCTURE ONLY — the CPU oracle for the forest-growth-and-proximity path.
 *
 * A plain, node-serial restatement of the reference RFX-Fuse CPU algorithm (every function
 * in rfx_oracle.cpp cites the reference file:line it follows).  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it, as the checker.  The
 * product library (librfx_b200.so) never links or calls it.
 *
 * Parity of this restatement is pinned against golden vectors produced by the reference
 * itself (oracle/_ref, built by oracle/Makefile; fixtures in tests/golden/).
 */
#ifndef RFX_ORACLE_H
#define RFX_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int task;          /* 0 classification, 1 regression, 2 unsupervised */
    int n;             /* rows supplied by the caller (real rows for unsupervised) */
    int p;
    int ntree;
    int mtry;
    int minndsize;
    int maxnode;       /* effective cap (already resolved by the caller) */
    int iseed;         /* grower seed base: tree t uses iseed + t */
    int boot_seed;     /* bootstrap seed base (12345 in the reference) */
    int nbins;
    int compute_importance;
    int compute_proximity;
    int n_threads;     /* OpenMP threads for proximity / importance (0 = default) */
} orc_params;

typedef struct {
    int nclass, N;                       /* N = rows grown on (2n for unsupervised) */
    int* nodestatus; int* bestvar; float* xbestsplit; int* treemap; int* nodeclass;
    int* nnode; float* nodepred; float* tnodewt;          /* [ntree x maxnode] (treemap x2) */
    int* nin_all;                        /* [ntree x N] or NULL */
    int* nodextr_all;                    /* [ntree x N] terminal node of every row, or NULL */
    int* nout;                           /* [N] */
    int* votes;                          /* [N x nclass] integer OOB vote counts, or NULL */
    float* q_raw;                        /* [N x nclass] float OOB vote sums, or NULL */
    float* oob_sum;                      /* [N] regression float sum of OOB predictions */
    float* tree_rr;                      /* [ntree x p] per-tree importance rr, or NULL */
    float* avimp; float* sqsd;           /* [p] */
    int* prox_pairs;                     /* [N x N] row-major raw counts P[i][j], or NULL */
    double* prox_final;                  /* [N x N] after finishprox, or NULL */
    float* oob_error;                    /* scalar (classification error or regression MSE) */
    float* oob_pred;                     /* [N] regression OOB mean prediction, or NULL */
} orc_out;

int orc_bootstrap(int n, int tree_id, int seed_base, const float* sample_weights, int* nin);
int orc_binning(const float* X, int n, int p, const int* cat, int nbins, float* edges,
                int* nb, int* kind, uint8_t* xb_rowmajor);
int orc_permutation(int n, uint32_t seed, int* perm);
int orc_synthetic(const float* X, int n, int p, int iseed, float* X_expanded);
int orc_maxnode(int n, int minndsize, int user_maxnode);
int orc_fit(const orc_params* prm, const float* X, const int* ycls, const float* yreg,
            const float* sample_weights, const int* cat, const float* classwt, orc_out* out);
int orc_finishprox(int N, const int* nout, const int* prox_pairs, double* out);
/* Prediction of new rows by tree traversal (X row-major [n][p]).  Classification: classwt-
 * weighted float votes -> cls_out [n] (0-based class) and proba_out [n][nclass]; regression:
 * reg_out [n].  catgoleft is empty for histogram-grown trees (all zero). */
int orc_predict(int task, int ntree, int maxnode, int nclass, int p, const int* cat,
                const float* classwt, const int* nodestatus, const int* bestvar,
                const float* xbestsplit, const int* treemap, const int* nodeclass,
                const float* nodepred, const float* X, int n, int* cls_out, float* proba_out,
                float* reg_out);

#ifdef __cplusplus
}
#endif
#endif
