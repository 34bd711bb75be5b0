// Host-side context of rfx_b200: error plumbing, growing device buffers and the per-device
// context shared by the host translation units (rfx_host.cu, rfx_lowrank_host.cu).
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/rfx_b200.h"
#include "rfx_device.cuh"

namespace rfxh {
extern thread_local std::string g_last_error;

struct RfxError : std::runtime_error {
    int code;
    RfxError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define RFX_CUDA(call)                                                                     \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess)                                                             \
            throw RfxError(e_ == cudaErrorMemoryAllocation ? RFX_ERR_OOM : RFX_ERR_CUDA,   \
                           std::string(#call) + ": " + cudaGetErrorString(e_));            \
    } while (0)

#define RFX_LAUNCH(name)                                                                   \
    do {                                                                                   \
        cudaError_t e_ = cudaGetLastError();                                               \
        if (e_ != cudaSuccess)                                                             \
            throw RfxError(RFX_ERR_CUDA, std::string("launch ") + name + ": " +            \
                                             cudaGetErrorString(e_));                      \
    } while (0)

inline void require(bool ok, int code, const std::string& msg) {
    if (!ok) throw RfxError(code, msg);
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return RFX_OK;
    } catch (const RfxError& e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return RFX_ERR_ARG;
    }
}

// Device buffer that only grows.
// Device blocks released by destroyed contexts, per device, for the next contexts of the
// process (a fit through the estimator API makes a new context each time; cudaMalloc and
// the synchronising cudaFree of its buffers would otherwise recur on every fit).  A block is
// cached only after its context's stream has drained.  An allocation takes the smallest
// cached block of at least its size and at most twice it; when cudaMalloc runs out of
// memory, the device's cached blocks are freed and the allocation retried.
struct BlockCache {
    std::mutex mu;
    std::map<int, std::multimap<size_t, void*>> free;  // device -> (size, block)
};
inline BlockCache& block_cache() {
    static BlockCache* c = new BlockCache;  // never destroyed: exit-time order does not matter
    return *c;
}
inline void* cache_take(int dev, size_t bytes, size_t* got) {
    BlockCache& bc = block_cache();
    std::lock_guard<std::mutex> lock(bc.mu);
    auto& m = bc.free[dev];
    auto it = m.lower_bound(bytes);
    if (it == m.end() || it->first > 2 * bytes) return nullptr;
    void* p = it->second;
    *got = it->first;
    m.erase(it);
    return p;
}
inline void cache_put(int dev, void* p, size_t bytes) {
    BlockCache& bc = block_cache();
    std::lock_guard<std::mutex> lock(bc.mu);
    bc.free[dev].emplace(bytes, p);
}
inline void cache_flush(int dev) {
    BlockCache& bc = block_cache();
    std::lock_guard<std::mutex> lock(bc.mu);
    for (auto& kv : bc.free[dev]) cudaFree(kv.second);
    bc.free[dev].clear();
}
// Bytes cached for `dev` (-1: every device).
inline long long cache_bytes(int dev) {
    BlockCache& bc = block_cache();
    std::lock_guard<std::mutex> lock(bc.mu);
    long long n = 0;
    for (auto& d : bc.free)
        if (dev < 0 || d.first == dev)
            for (auto& kv : d.second) n += (long long)kv.first;
    return n;
}
// Free the blocks cached for `dev` (-1: every device), each with its device current.
inline void cache_empty(int dev) {
    BlockCache& bc = block_cache();
    std::lock_guard<std::mutex> lock(bc.mu);
    bool any = false;
    for (auto& d : bc.free) any = any || ((dev < 0 || d.first == dev) && !d.second.empty());
    if (!any) return;
    int prev = 0;
    RFX_CUDA(cudaGetDevice(&prev));
    for (auto& d : bc.free) {
        if (dev >= 0 && d.first != dev) continue;
        RFX_CUDA(cudaSetDevice(d.first));
        for (auto& kv : d.second) RFX_CUDA(cudaFree(kv.second));
        d.second.clear();
    }
    RFX_CUDA(cudaSetDevice(prev));
}

struct DBuf {
    void* p = nullptr;
    size_t cap = 0;
    void* get(size_t bytes) {
        if (bytes == 0) bytes = 16;
        if (bytes > cap) {
            if (p) cudaFree(p);  // synchronising: the context's queued work may still use it
            p = nullptr;
            cap = 0;
            int dev = 0;
            RFX_CUDA(cudaGetDevice(&dev));
            size_t got = 0;
            if (void* q = cache_take(dev, bytes, &got)) {
                p = q;
                cap = got;
                return p;
            }
            cudaError_t e = cudaMalloc(&p, bytes);
            if (e == cudaErrorMemoryAllocation) {
                cudaGetLastError();
                cache_flush(dev);
                e = cudaMalloc(&p, bytes);
            }
            if (e != cudaSuccess)
                throw RfxError(e == cudaErrorMemoryAllocation ? RFX_ERR_OOM : RFX_ERR_CUDA,
                               std::string("cudaMalloc: ") + cudaGetErrorString(e));
            cap = bytes;
        }
        return p;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    // Hand the block to the process's cache (the owner's stream has drained).
    void retire(int dev) {
        if (p) cache_put(dev, p, cap);
        p = nullptr;
        cap = 0;
    }
};

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Ctx {
    int device = 0;
    int sm_count = 148;
    cudaStream_t st = nullptr;
    int* h_counters = nullptr;  // pinned
    cudaEvent_t ev_stage[2] = {nullptr, nullptr};  // copies through the pinned staging buffers

    // loaded dataset
    bool loaded = false;
    rfx_fit_params prm{};
    int N = 0, p = 0, nclass = 0, task = 0, M = 0, R = 0;
    std::vector<int> labels0;   // 0-based labels (classification / unsupervised)
    std::vector<float> classwt;
    rfx::Data D{};
    DBuf xc, rows, edges, nb, kind, cat, lab, yreg, yv, perm, ks, cumw, totw, keys_a, keys_b;
    cudaEvent_t perm_event = nullptr;  // owned by the process-wide permutation cache

    // accumulators
    DBuf nout, votes, oob_sum, avimp, sqsd, prox_own, qtmp, cw_dev, tree_oob_all, fin_inv;
    int* prox = nullptr;
    int64_t prox_len = 0;
    int trees_done = 0;
    int tree_oob_cap = 0, tree_oob_n = 0;

    // device tree store (keep_trees): reference-layout arrays of the trees grown since the
    // load, [ts_cap][maxnode] (treemap [ts_cap][2 maxnode], nnode [ts_cap])
    DBuf ts_status, ts_bestvar, ts_xbest, ts_treemap, ts_nodeclass, ts_nnode, ts_nodepred,
        ts_tnodewt;
    int ts_cap = 0, ts_n = 0;

    // progress callback (rfx_set_progress), called between batches
    rfx_progress_fn progress = nullptr;
    void* progress_user = nullptr;

    // measurement
    bool profiling = false;
    bool level_log = std::getenv("RFX_LEVEL_LOG") != nullptr;  // per-level trace on stderr
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::vector<cudaEvent_t> ev_hist;  // per-level histogram timing within a level group
    long long launches = 0, hist_launches = 0, levels = 0, trees = 0;
    double hist_ms = 0.0;
    double prox_ms = 0.0;
    double prox_pull_pairs = 0.0;  // pairs added by the pull kernel (the push kernel counts its own)
    // proximity counting: 0 automatic, 1 push, 2 pull (RFX_PROX_MODE=push|pull)
    int prox_mode = std::getenv("RFX_PROX_MODE") == nullptr
                        ? 0
                        : (std::string(std::getenv("RFX_PROX_MODE")) == "push"
                               ? 1
                               : (std::string(std::getenv("RFX_PROX_MODE")) == "pull" ? 2 : 0));
    double topk_ms = 0.0;
    double sketch_ms = 0.0, sketch_bytes = 0.0;
    long long topk_tiles = 0;

    // low-rank proximity (rfx_lowrank_host.cu): per-tree leaf groups, then the factors
    int lr_rank = 0;            // requested rank, 0 = off
    int lr_n = 0, lr_cap = 0;   // trees stored / capacity
    int lr_G = 0;               // group-offset stride per tree (maxnode + 2)
    int lr_k = 0, lr_Rpad = 0;  // factor rank and rows padded to the product tile
    int lr_R = 0;               // factor rows
    bool lr_ready = false;
    std::vector<int> lr_pos;    // stored position of every original row (product order)
    DBuf lr_code, lr_order, lr_goff, lr_ngroups, lr_tmp;
    DBuf lr_X, lr_Z, lr_CZ, lr_Y, lr_ls, lr_part, lr_small, lr_A, lr_q, lr_qb, lr_s, lr_qbp, lr_sp, lr_perm, lr_blocks, lr_np, lr_norm, lr_ids, lr_keys, lr_order_s, lr_cub,
        lr_err, lr_out_i, lr_out_v;

    // stored forest for prediction (rfx_predict.cu)
    int f_T = 0, f_cap = 0, f_M = 0, f_p = 0, f_nclass = 0, f_task = 0;
    bool f_classwt = false;
    DBuf f_nodes, f_root, f_cat, f_cw, p_X, p_xc, p_vote, p_val, p_cls, p_proba, p_pred;
    // leaf assignments (rfx_leaves.cu): int16 leaf [l_cap][N], OOB bit words [l_cap][l_words],
    // the inverted index (rows grouped by (tree, leaf); group g = t * l_W + (uint16)leaf)
    int l_T = 0, l_cap = 0, l_words = 0, l_W = 0;
    bool l_index = false;
    std::vector<int> l_anchors;  // the last selected outlier anchors (reused like the reference)
    std::map<int, std::pair<float, float>> l_norm;  // outlier (median, MAD) per class (-1: all)
    DBuf l_leaf, l_oob, l_rows, l_gs, l_ge, l_keys, l_cub, l_cnt, l_cidx, l_cval, l_nnz, l_q,
        l_out, l_f;
    // imputation round (rfx_impute_host.cu)
    DBuf i_x, i_miss, i_cat, i_S, i_scratch, i_cells, i_out, i_prof;

    // batch buffers
    int Tcap = 0;
    rfx::Batch B{};
    DBuf b_nin, b_seg0, b_seg1, b_ninbag, b_oob, b_noob, b_mt, b_mtpos, b_status, b_bestvar,
        b_xbest, b_treemap, b_nodeclass, b_nodepred, b_tnodewt, b_ndstart, b_ndcnt, b_ndbuf,
        b_ndflag, b_ndcrit0, b_ndmaj, b_ndsum, b_ndkey, b_feat, b_lvl, b_srch, b_srchcnt,
        b_srchoff, b_srchsml, b_bigrec, b_smlrec, b_sml2rec, b_counters, b_oobleaf, b_used, b_right, b_rightimp, b_d2, b_d0, b_impnode, b_rr, b_rsum, b_srchbig, b_partbig, b_pcode, b_pocnt, b_ppairs;

    ~Ctx() {
        DBuf* all[] = {&xc, &rows, &edges, &nb, &kind, &cat, &lab, &yreg, &yv, &perm, &ks, &cumw,
                       &totw, &keys_a, &keys_b, &nout, &votes, &oob_sum, &avimp, &sqsd,
                       &prox_own, &qtmp, &cw_dev, &tree_oob_all, &fin_inv, &b_nin, &b_seg0, &b_seg1,
                       &b_ninbag, &b_oob, &b_noob, &b_mt, &b_mtpos, &b_status, &b_bestvar,
                       &b_xbest, &b_treemap, &b_nodeclass, &b_nodepred, &b_tnodewt, &b_ndstart,
                       &b_ndcnt, &b_ndbuf, &b_ndflag, &b_ndcrit0, &b_ndmaj, &b_ndsum, &b_ndkey,
                       &b_feat, &b_lvl, &b_srch, &b_srchcnt, &b_srchoff, &b_srchsml, &b_bigrec, &b_smlrec, &b_sml2rec, &b_counters,
                       &b_oobleaf, &b_used, &b_right, &b_rightimp, &b_d2, &b_d0, &b_impnode, &b_rr, &b_rsum, &b_srchbig, &b_partbig, &b_pcode, &b_pocnt, &b_ppairs,
                       &lr_code, &lr_order, &lr_goff, &lr_ngroups, &lr_tmp, &lr_X, &lr_Z,
                       &lr_CZ, &lr_Y, &lr_ls, &lr_part, &lr_small, &lr_A, &lr_q, &lr_qb, &lr_s, &lr_qbp, &lr_sp, &lr_perm, &lr_blocks, &lr_np, &lr_norm, &lr_ids, &lr_keys, &lr_order_s, &lr_cub, &f_nodes, &f_root, &f_cat, &f_cw, &p_X,
                       &p_xc, &p_vote, &p_val, &p_cls, &p_proba, &p_pred, &i_x, &i_miss, &i_cat,
                       &i_S, &i_scratch, &i_cells, &i_out, &i_prof, &l_leaf, &l_oob, &l_rows, &l_gs, &l_ge,
                       &l_keys, &l_cub, &l_cnt, &l_cidx, &l_cval, &l_nnz, &l_q, &l_out, &l_f,
                       &lr_err, &lr_out_i, &lr_out_v, &ts_status, &ts_bestvar, &ts_xbest, &ts_treemap,
                       &ts_nodeclass, &ts_nnode, &ts_nodepred, &ts_tnodewt};
        cudaSetDevice(device);
        const bool drained = !st || cudaStreamSynchronize(st) == cudaSuccess;
        for (DBuf* b : all) {
            if (drained) b->retire(device);
            else b->release();
        }
        if (h_counters) cudaFreeHost(h_counters);
        for (int b = 0; b < 2; ++b) {
            if (ev_stage[b]) cudaEventDestroy(ev_stage[b]);
        }
        for (cudaEvent_t e : ev_hist) cudaEventDestroy(e);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (st) cudaStreamDestroy(st);
    }
};

inline Ctx* as_ctx(void* c) {
    require(c != nullptr, RFX_ERR_ARG, "null context");
    Ctx* x = static_cast<Ctx*>(c);
    RFX_CUDA(cudaSetDevice(x->device));
    return x;
}

inline int grid_for(long long n, int threads, int cap) {
    return (int)std::max(1LL, std::min((long long)cap, (n + threads - 1) / threads));
}


// Low-rank proximity store (rfx_lowrank_host.cu): make room for `extra` more trees, and
// store the leaf groups of the T trees of a grown batch.
void lr_reserve(Ctx& c, int extra);
void lr_store_batch(Ctx& c, const rfx::Batch& B, int T);

// Prediction forest (rfx_predict_host.cu): room for `extra` more trees; pack a grown batch.
void forest_reserve(Ctx& c, int extra);
void forest_store_batch(Ctx& c, const rfx::Batch& B, int T);
void forest_reset(Ctx& c);

// Leaf assignments (rfx_leaves.cu): forget the stored trees; store a grown batch's leaves.
void leaves_reset(Ctx& c);
void leaves_store_batch(Ctx& c, const rfx::Batch& B, int T);

}  // namespace rfxh
