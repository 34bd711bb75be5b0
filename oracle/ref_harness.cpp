// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// Drives the reference RFX-Fuse CPU implementation, compiled unmodified from its own
// sources (recipe: oracle/Makefile, objects under oracle/_ref/), and exposes its outputs
// through a plain C ABI so that tests/golden/make_golden.py can dump golden vectors.
//
// It calls the reference's own entry points in the reference's own order:
//   rf::cpu_bootstrap                (src/rf_bootstrap.cpp:15)
//   rf::compute_bin_edges_quantile   (src/rf_histogram.cpp:36)
//   rf::bin_data_cpu                 (src/rf_histogram.cpp:134)
//   rf::RandomForest::fit            (src/rf_random_forest.cpp:502)  -> CPU per-tree loop
// Per-tree state that the reference keeps only in private workspaces (bootstrap counts,
// terminal node of every sample, the raw proximity sums before finishprox) is read from a
// progress callback that the reference invokes after every tree
// (src/rf_random_forest.cpp:597-601); the class members are made visible to this
// translation unit only, so no reference source is changed.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <functional>
#include <iostream>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#define private public
#define protected public
#include "rf_random_forest.hpp"
#undef private
#undef protected
#include "rf_bootstrap.hpp"
#include "rf_config.hpp"
#include "rf_histogram.hpp"

namespace rf { extern RFConfig g_config; }

extern "C" {

// nin_out[n] = bootstrap multiplicity of every row for tree `tree_id`; returns ninbag.
int ref_bootstrap(int n, int tree_id, const float* sample_weights, int* nin_out) {
    std::vector<float> weight(n, 1.0f), win(n);
    std::vector<int> nout(n, 0), jinbag(n), joobag(n);
    int ninbag = 0, noobag = 0;
    rf::cpu_bootstrap(weight.data(), n, win.data(), nin_out, nout.data(), jinbag.data(),
                      joobag.data(), ninbag, noobag, tree_id, sample_weights);
    return ninbag;
}

// edges_out[f*(nbins+1)+b], nb_out[f] = bins of feature f, kind_out[f] = 0 continuous,
// 1 binary, 2 categorical; xb_out row-major uint8 [n x p].
int ref_binning(const float* X, int n, int p, const int* cat, int nbins, float* edges_out,
                int* nb_out, int* kind_out, uint8_t* xb_out) {
    std::vector<rf::FeatureBinInfo> info(p);
    rf::compute_bin_edges_quantile(X, n, p, cat, nbins, info.data());
    rf::bin_data_cpu(X, n, p, info.data(), xb_out);
    for (int f = 0; f < p; ++f) {
        nb_out[f] = info[f].n_bins;
        kind_out[f] = info[f].is_categorical ? 2 : (info[f].is_binary ? 1 : 0);
        for (int b = 0; b <= nbins; ++b) edges_out[(size_t)f * (nbins + 1) + b] = info[f].bin_edges[b];
    }
    return 0;
}

struct RefFitOut {
    int nclass, maxnode, nsample_total, mtry;
    int* nodestatus; int* bestvar; float* xbestsplit; int* treemap; int* nodeclass;
    int* nnode; float* nodepred; float* tnodewt;
    int* nin_all;       // [ntree x N]
    int* nodextr_all;   // [ntree x N] terminal node of every row (when proximity is on)
    int* nout;          // [N]
    float* q_raw;       // [N x nclass] raw OOB votes before normalisation
    float* oob_pred;    // [N] regression: OOB mean prediction (after finalize)
    float* avimp;       // [p]
    float* sqsd;        // [p]
    double* prox_raw;   // [N x N] column-major raw sums before finishprox (N<=5000 only)
    double* prox_final; // [N x N] after finishprox
    float* oob_error;   // scalar
    float* X_expanded;  // unsupervised: [2n x p] synthetic expansion
};

// task: 0 classification (ycls), 1 regression (yreg), 2 unsupervised.
// Sizes of the tree arrays are ntree*maxnode (treemap 2x); the caller sizes them from
// ref_effective_maxnode().
int ref_effective_maxnode(int task, int n, int minndsize, int maxnode) {
    if (task == 2) return rf::calculate_maxnode(2 * n, minndsize);
    return rf::calculate_maxnode(n, minndsize, maxnode);
}

int ref_fit(int task, const float* X, const int* ycls, const float* yreg, const float* sw,
            const int* cat, const float* classwt, int n, int p, int ntree, int mtry,
            int minndsize, int maxnode, int iseed, int nbins, int compute_importance,
            int compute_proximity, RefFitOut* out) {
    rf::RandomForestConfig cfg;
    cfg.nsample = n;
    cfg.ntree = ntree;
    cfg.mdim = p;
    cfg.mtry = mtry;
    cfg.minndsize = minndsize;
    cfg.maxnode = rf::calculate_maxnode(n, minndsize, maxnode);
    cfg.iseed = iseed;
    cfg.n_bins = nbins;
    cfg.use_histogram = true;
    cfg.compute_importance = compute_importance != 0;
    cfg.compute_proximity = compute_proximity != 0;
    cfg.compute_local_importance = false;
    cfg.use_gpu = false;
    cfg.use_casewise = false;
    cfg.task_type = task == 0 ? rf::TaskType::CLASSIFICATION
                  : task == 1 ? rf::TaskType::REGRESSION : rf::TaskType::UNSUPERVISED;
    if (task == 0) {
        std::set<int> u(ycls, ycls + n);
        cfg.nclass = (int)u.size();
        if (classwt) cfg.classwt.assign(classwt, classwt + cfg.nclass);
    } else if (task == 1) {
        cfg.nclass = 1;
    } else {
        cfg.nclass = 2;
    }
    rf::RandomForest forest(cfg);
    std::vector<int> catv(p, 1);
    if (cat) catv.assign(cat, cat + p);
    forest.set_categorical_features(catv.data(), p);
    rf::RandomForest* fp = &forest;
    forest.set_progress_callback([fp, out](int done, int total) {
        const int N = fp->config_.nsample;
        const int t = done - 1;
        if (out->nin_all)
            std::copy(fp->nin_workspace_.begin(), fp->nin_workspace_.begin() + N,
                      out->nin_all + (size_t)t * N);
        if (out->nodextr_all)
            std::copy(fp->nodextr_workspace_.begin(), fp->nodextr_workspace_.begin() + N,
                      out->nodextr_all + (size_t)t * N);
        if (done == total) {
            if (out->prox_raw && !fp->proximity_matrix_.empty())
                std::copy(fp->proximity_matrix_.begin(), fp->proximity_matrix_.end(), out->prox_raw);
            if (out->q_raw && !fp->q_.empty())
                std::copy(fp->q_.begin(), fp->q_.end(), out->q_raw);
        }
    });
    const void* y = task == 0 ? (const void*)ycls : (const void*)yreg;
    forest.fit(X, y, sw);

    const auto& c = forest.config_;
    out->nclass = c.nclass;
    out->maxnode = c.maxnode;
    out->nsample_total = c.nsample;
    out->mtry = c.mtry;
    const size_t tm = (size_t)ntree * c.maxnode;
    std::copy(forest.nodestatus_.begin(), forest.nodestatus_.begin() + tm, out->nodestatus);
    std::copy(forest.bestvar_.begin(), forest.bestvar_.begin() + tm, out->bestvar);
    std::copy(forest.xbestsplit_.begin(), forest.xbestsplit_.begin() + tm, out->xbestsplit);
    std::copy(forest.treemap_.begin(), forest.treemap_.begin() + 2 * tm, out->treemap);
    std::copy(forest.nodeclass_.begin(), forest.nodeclass_.begin() + tm, out->nodeclass);
    std::copy(forest.nnode_.begin(), forest.nnode_.begin() + ntree, out->nnode);
    std::copy(forest.tnodewt_.begin(), forest.tnodewt_.begin() + tm, out->tnodewt);
    if (task == 1 && out->nodepred)
        std::copy(forest.node_predictions_regression_.begin(),
                  forest.node_predictions_regression_.begin() + tm, out->nodepred);
    std::copy(forest.nout_.begin(), forest.nout_.begin() + c.nsample, out->nout);
    if (task == 1 && out->oob_pred)
        std::copy(forest.oob_predictions_.begin(), forest.oob_predictions_.begin() + c.nsample,
                  out->oob_pred);
    if (out->avimp && !forest.avimp_.empty())
        std::copy(forest.avimp_.begin(), forest.avimp_.begin() + p, out->avimp);
    if (out->sqsd && !forest.sqsd_.empty())
        std::copy(forest.sqsd_.begin(), forest.sqsd_.begin() + p, out->sqsd);
    if (out->prox_final && !forest.proximity_matrix_.empty())
        std::copy(forest.proximity_matrix_.begin(), forest.proximity_matrix_.end(), out->prox_final);
    if (out->oob_error) *out->oob_error = forest.oob_error_;
    if (task == 2 && out->X_expanded && !forest.X_unsupervised_expanded_.empty())
        std::copy(forest.X_unsupervised_expanded_.begin(), forest.X_unsupervised_expanded_.end(),
                  out->X_expanded);
    return 0;
}

}  // extern "C"
