// Prediction of new rows by tree traversal (RandomForest::predict_classification /
// predict_proba new-data branch, src/rf_random_forest.cpp:3403-3490 and 3863-3945;
// predict_regression, src/rf_random_forest.cpp:3494-3590).
//
// The forest is kept on the device as one 16-byte node per (tree, node) so a walk step is a
// single load: {feature, threshold-or-value, left, right}.  Terminal nodes (status -1) carry
// feature -1 and their class (classification) or value (regression); every other node --
// whatever its status -- is a split on bestvar, exactly as the reference walk treats it.
//
// Step 1 (k_predict_walk): thread per (row, tree), consecutive threads = consecutive rows of
// one tree (shared upper nodes, feature columns read contiguously from the transposed X);
// it records the tree's vote (class, or 0xFF for none) or value (NaN for none).
// Step 2 (k_predict_reduce): thread per row folds the trees in tree order -- float votes
// (classwt weights) and float value sums in the reference's sequential order -- then takes
// the first maximum, the vote fractions, or the mean.
#include <cuda_runtime.h>
#include <cstdint>

#include "rfx_predict.h"

namespace rfx {

namespace {

// static_cast<int>(float) as the reference's x86-64 build evaluates it (cvttss2si): NaN and
// values outside int range give INT_MIN.
__device__ __forceinline__ int x86_float_to_int(float y) {
    if (!(y >= -2147483648.0f && y < 2147483648.0f)) return (int)0x80000000;
    return (int)y;
}

}  // namespace

// Pack the trees of a grown batch: node (t, m) -> forest[(tree0 + t) * M + m].
__global__ void k_pack_forest(Batch B, int task, PNode* __restrict__ forest,
                              float* __restrict__ root_value) {
    const int t = blockIdx.y;
    const int M = B.M;
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const size_t k = (size_t)t * M + m;
        PNode nd;
        if (B.status[k] == -1) {
            nd.feat = -1;
            nd.val = task == 1 ? B.nodepred[k] : __int_as_float(B.nodeclass[k]);
            nd.left = nd.right = 0;
        } else {
            nd.feat = B.bestvar[k];
            nd.val = B.xbest[k];
            nd.left = B.treemap[2 * k];
            nd.right = B.treemap[2 * k + 1];
        }
        forest[k] = nd;
        if (m == 0) root_value[t] = B.nodepred[k];
    }
}

// One vote / value per (row, tree).  xc: [p][n] column-major rows of this chunk.
__global__ void k_predict_walk(const PNode* __restrict__ forest, const float* __restrict__ root_value,
                               int M, int T, const float* __restrict__ xc, int n, int p,
                               const int* __restrict__ cat, int task, int nclass,
                               uint8_t* __restrict__ vote, float* __restrict__ value) {
    const int t = blockIdx.y;
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const PNode* nodes = forest + (size_t)t * M;
    int kt = 0;
    int outcome = -2;      // classification: class voted; -2 = no vote
    float v = __int_as_float(0x7fc00000);  // regression: value added (NaN = none)
    for (int k = 0; k < M; ++k) {
        if (kt >= M) {     // classification only (the regression walk has no such test)
            if (task != 1) outcome = 0;
            break;
        }
        const PNode nd = nodes[kt];
        if (nd.feat == -1) {
            if (task == 1) {
                v = nd.val;
            } else {
                const int c = __float_as_int(nd.val);
                outcome = (c >= 0 && c < nclass) ? c : 0;
            }
            break;
        }
        const int m = nd.feat;
        if (m >= 0 && m < p) {
            const float x = xc[(size_t)m * n + s];
            if (cat[m] == 1) {
                kt = x <= nd.val ? nd.left : nd.right;
            } else {
                const int jcat = x86_float_to_int(x + 0.5f);
                if (jcat >= 0 && jcat < cat[m]) {
                    kt = nd.right;  // catgoleft is empty for histogram-grown trees
                } else {
                    if (task == 1) v = root_value[t];
                    else outcome = 0;
                    break;
                }
            }
        } else {
            if (task == 1) v = root_value[t];
            else outcome = 0;
            break;
        }
    }
    if (task == 1) value[(size_t)t * n + s] = v;
    else vote[(size_t)t * n + s] = outcome >= 0 ? (uint8_t)outcome : (uint8_t)0xFF;
}

// Fold the trees of every row in tree order.  cls [n], proba [n][nclass], pred [n].
__global__ void k_predict_reduce(const uint8_t* __restrict__ vote, const float* __restrict__ value,
                                 int n, int T, int task, int nclass, const float* __restrict__ classwt,
                                 int* __restrict__ cls, float* __restrict__ proba,
                                 float* __restrict__ pred) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    if (task == 1) {
        float sum = 0.0f;
        int count = 0;
        for (int t = 0; t < T; ++t) {
            const float v = value[(size_t)t * n + s];
            if (v == v) {
                sum += v;
                ++count;
            }
        }
        pred[s] = count > 0 ? sum / (float)count : 0.0f;
        return;
    }
    float votes[kPredMaxClass];
    for (int c = 0; c < nclass; ++c) votes[c] = 0.0f;
    for (int t = 0; t < T; ++t) {
        const int c = vote[(size_t)t * n + s];
        if (c != 0xFF) votes[c] += classwt ? classwt[c] : 1.0f;
    }
    int best = 0;
    float mx = votes[0];
    for (int c = 1; c < nclass; ++c)
        if (votes[c] > mx) {
            mx = votes[c];
            best = c;
        }
    if (cls) cls[s] = best;
    if (proba) {
        float tot = 0.0f;
        for (int c = 0; c < nclass; ++c) tot += votes[c];
        if (tot <= 0.0f) tot = 1.0f;
        for (int c = 0; c < nclass; ++c) proba[(size_t)s * nclass + c] = votes[c] / tot;
    }
}

}  // namespace rfx
