// Host orchestration and the C ABI of rfx_b200 (declared in include/rfx_b200.h).
//
// One context = one CUDA device + one stream.  rfx_load puts the dataset in HBM (raw
// values column-major, packed bin rows, bin edges, targets, the importance permutation);
// rfx_grow grows batches of trees level by level (rfx_grow.cu) and folds each batch's OOB
// votes, predictions, importance and proximity into device accumulators in tree order.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/rfx_b200.h"
#include "rfx_device.cuh"
#include "rfx_kernels.h"

#include "rfx_ctx.h"

thread_local std::string rfxh::g_last_error;

namespace {

using namespace rfxh;

// Importance permutation cache, one per (device, N), never freed (process lifetime).  It
// is computed on a side stream; only the importance kernels wait for its event.
struct PermEntry {
    int* perm = nullptr;
    cudaEvent_t done = nullptr;
};

const PermEntry& permutation_for(int device, int N) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, PermEntry> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({device, N});
    if (it != cache.end()) return it->second;
    PermEntry e;
    int* ks = nullptr;
    cudaStream_t side = nullptr;
    RFX_CUDA(cudaMalloc(&e.perm, (size_t)N * 4));
    RFX_CUDA(cudaMalloc(&ks, (size_t)std::max(N, 1) * 4));
    RFX_CUDA(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
    RFX_CUDA(cudaEventCreateWithFlags(&e.done, cudaEventDisableTiming));
    rfx::k_permutation<<<1, 256, 0, side>>>(N, 42u, ks, e.perm);
    RFX_LAUNCH("k_permutation");
    RFX_CUDA(cudaEventRecord(e.done, side));
    RFX_CUDA(cudaFreeAsync(ks, side));
    RFX_CUDA(cudaStreamDestroy(side));  // returns at once; queued work still completes
    return cache.emplace(std::make_pair(device, N), e).first->second;
}

// Synthetic rows of RandomForest::fit_unsupervised (src/rf_random_forest.cpp:1068-1086):
// column k is shuffled by std::shuffle with std::mt19937(iseed + k * 1000003).  Built on
// the host with the same C++ standard library algorithm so the rows are bit-identical.
void synthetic_rows(const float* X, int n, int p, int iseed, std::vector<float>& out) {
    out.resize((size_t)2 * n * p);
    std::memcpy(out.data(), X, sizeof(float) * (size_t)n * p);
    std::vector<float> col(n);
    for (int k = 0; k < p; ++k) {
        std::mt19937 g((uint32_t)(iseed + k * 1000003));
        for (int i = 0; i < n; ++i) col[i] = X[(size_t)i * p + k];
        std::shuffle(col.begin(), col.end(), g);
        for (int i = 0; i < n; ++i) out[(size_t)(n + i) * p + k] = col[i];
    }
}

void alloc_batch(Ctx& c, int Tcap) {
    const size_t N = c.N, M = c.M, T = Tcap, p = c.p;
    rfx::Batch& B = c.B;
    B.nin = (int*)c.b_nin.get(T * N * 4);
    B.seg[0] = (int*)c.b_seg0.get(T * N * 4);
    B.seg[1] = (int*)c.b_seg1.get(T * N * 4);
    B.ninbag = (int*)c.b_ninbag.get(T * 4);
    B.oob = (int*)c.b_oob.get(T * N * 4);
    B.noob = (int*)c.b_noob.get(T * 4);
    B.mt = (uint32_t*)c.b_mt.get(T * 624 * 4);
    B.mt_pos = (int*)c.b_mtpos.get(T * 4);
    B.status = (int*)c.b_status.get(T * M * 4);
    B.bestvar = (int*)c.b_bestvar.get(T * M * 4);
    B.xbest = (float*)c.b_xbest.get(T * M * 4);
    B.treemap = (int*)c.b_treemap.get(T * M * 8);
    B.nodeclass = (int*)c.b_nodeclass.get(T * M * 4);
    B.nodepred = (float*)c.b_nodepred.get(T * M * 4);
    B.tnodewt = (float*)c.b_tnodewt.get(T * M * 4);
    B.nd_start = (int*)c.b_ndstart.get(T * M * 4);
    B.nd_cnt = (int*)c.b_ndcnt.get(T * M * 4);
    B.nd_buf = (uint8_t*)c.b_ndbuf.get(T * M);
    B.nd_flag = (uint8_t*)c.b_ndflag.get(T * M);
    B.nd_crit0 = (float*)c.b_ndcrit0.get(T * M * 4);
    B.nd_maj = (int*)c.b_ndmaj.get(T * M * 4);
    B.nd_sum = (float*)c.b_ndsum.get(T * M * 4);
    B.nd_key = (unsigned long long*)c.b_ndkey.get(T * M * 8);
    B.feat = (uint16_t*)c.b_feat.get(T * M * c.prm.mtry * 2);
    int* lvl = (int*)c.b_lvl.get(T * 5 * 4 + 16);
    B.lvl_lo = lvl;
    B.lvl_hi = lvl + T;
    B.nxt_lo = lvl + 2 * T;
    B.nxt_hi = lvl + 3 * T;
    B.nnode = lvl + 4 * T;
    B.lvl_off = (int*)c.b_srchoff.get((T + 1) * 16);
    B.srch_off = B.lvl_off + (T + 1);
    B.srch_big_off = B.srch_off + (T + 1);
    B.srch_sml_off = B.srch_big_off + (T + 1);
    B.srch_big = (int*)c.b_srchbig.get(T * M * 4);
    B.srch_sml = (int*)c.b_srchsml.get(T * M * 4);
    B.big_rec = (int4*)c.b_bigrec.get(T * M * 16);
    B.sml_rec = (int4*)c.b_smlrec.get(T * M * 16);
    B.sml2_rec = (int4*)c.b_sml2rec.get(T * M * 16);
    B.part_big = (long long*)c.b_partbig.get(T * (N / rfx::kBigSegment + 2) * 8);
    B.srch = (int*)c.b_srch.get(T * M * 4);
    B.srch_cnt = (int*)c.b_srchcnt.get(T * 12);
    B.srch_big_cnt = B.srch_cnt + T;
    B.srch_sml_cnt = B.srch_cnt + 2 * T;
    B.counters = (int*)c.b_counters.get(128);
    B.hist_bytes = reinterpret_cast<unsigned long long*>(B.counters + 8);
    B.prox_pairs = reinterpret_cast<unsigned long long*>(B.counters + 10);
    B.diag = c.level_log ? reinterpret_cast<unsigned long long*>(B.counters + 12) : nullptr;
    B.oob_leaf = (int*)c.b_oobleaf.get(T * N * 4);
    B.used = (uint8_t*)c.b_used.get(T * p);
    B.right = (int*)c.b_right.get(T * 4);
    B.rightimp = (int*)c.b_rightimp.get(T * p * 4);
    B.rr = (float*)c.b_rr.get(T * p * 4);
    B.rsum = (float*)c.b_rsum.get(T * (p + 1) * 4);
    if (c.task == RFX_TASK_REGRESSION && c.prm.compute_importance) {
        B.d2 = (float*)c.b_d2.get(T * N * p * 4);
        B.d0 = (float*)c.b_d0.get(T * N * 4);
        B.imp_node = (int4*)c.b_impnode.get(T * M * 16);
    } else {
        B.d2 = nullptr;
        B.d0 = nullptr;
        B.imp_node = nullptr;
    }
    B.tree_oob = nullptr;
    B.M = c.M;
    B.mtry = c.prm.mtry;
    B.minsplit = c.task == RFX_TASK_REGRESSION ? 2 * c.prm.minndsize : c.prm.minndsize;
    B.lane_split = c.task == RFX_TASK_REGRESSION && c.prm.mtry <= 32 ? 1 : 0;
    B.iseed = c.prm.iseed;
    B.boot_seed = c.prm.boot_seed;
    c.Tcap = Tcap;
}

void load(Ctx& c, const rfx_fit_params* prm, const rfx_inputs* in) {
    require(prm && in && in->X, RFX_ERR_ARG, "null params / inputs / X");
    const rfx_fit_params P = *prm;
    require(P.task >= 0 && P.task <= 2, RFX_ERR_ARG, "task must be 0, 1 or 2");
    require(P.n >= 1 && P.p >= 1, RFX_ERR_ARG, "n and p must be positive");
    require(P.p <= 1000, RFX_ERR_UNSUPPORTED, "more than 1000 features is not supported");
    require(P.mtry >= 1 && P.mtry < (1 << 24), RFX_ERR_ARG, "mtry must be >= 1");
    require(P.maxnode >= 1, RFX_ERR_ARG, "maxnode must be >= 1");
    require(P.nbins >= 2 && P.nbins <= 256, RFX_ERR_ARG, "nbins must be in [2, 256]");
    require(P.minndsize >= 0, RFX_ERR_ARG, "minndsize must be >= 0");
    require(P.task != RFX_TASK_CLASSIFICATION || in->y_class, RFX_ERR_ARG, "y_class required");
    require(P.task != RFX_TASK_REGRESSION || in->y_reg, RFX_ERR_ARG, "y_reg required");
    c.loaded = false;
    c.prm = P;
    c.task = P.task;
    c.p = P.p;
    c.M = P.maxnode;
    const int n = P.n, p = P.p;
    std::vector<float> xs;
    const float* X = in->X;
    c.labels0.clear();
    if (P.task == RFX_TASK_UNSUPERVISED) {
        synthetic_rows(in->X, n, p, P.iseed, xs);
        X = xs.data();
        c.N = 2 * n;
        c.nclass = 2;
        c.labels0.assign(c.N, 0);
        std::fill(c.labels0.begin(), c.labels0.begin() + n, 1);
    } else if (P.task == RFX_TASK_CLASSIFICATION) {
        // setup_classification_task (src/rf_random_forest.cpp:3287-3309): labels -> rank
        // among the sorted distinct labels.
        c.N = n;
        std::vector<int> u(in->y_class, in->y_class + n);
        std::sort(u.begin(), u.end());
        u.erase(std::unique(u.begin(), u.end()), u.end());
        c.nclass = (int)u.size();
        c.labels0.resize(n);
        for (int i = 0; i < n; ++i)
            c.labels0[i] = (int)(std::lower_bound(u.begin(), u.end(), in->y_class[i]) - u.begin());
    } else {
        c.N = n;
        c.nclass = 1;
    }
    require(c.nclass <= rfx::kMaxClass, RFX_ERR_UNSUPPORTED,
            "more than 32 classes is not supported by the device histograms");
    const size_t N = c.N;
    std::vector<int> catv(p, 1);
    if (in->cat) catv.assign(in->cat, in->cat + p);
    bool has_cat = false;
    for (int f = 0; f < p; ++f) {
        require(catv[f] >= 1, RFX_ERR_ARG, "cat[f] must be >= 1");
        has_cat |= catv[f] != 1;
    }
    c.R = P.prox_rows > 0 ? std::min<int>(P.prox_rows, (int)N) : (int)N;
    require(!(P.compute_proximity && has_cat), RFX_ERR_UNSUPPORTED,
            "proximity with categorical features is not supported yet");
    require(!(P.keep_leaves && has_cat), RFX_ERR_UNSUPPORTED,
            "leaf assignments with categorical features are not supported yet");
    require(P.lowrank_rank >= 0 && P.lowrank_rank <= 64, RFX_ERR_UNSUPPORTED,
            "low-rank proximity rank must be in [0, 64]");
    require(P.lowrank_rank == 0 || P.maxnode + 1 < 65535, RFX_ERR_UNSUPPORTED,
            "low-rank proximity needs maxnode < 65534");
    c.classwt.clear();
    if (P.task == RFX_TASK_CLASSIFICATION && in->classwt)
        c.classwt.assign(in->classwt, in->classwt + c.nclass);

    cudaStream_t st = c.st;
    rfx::Data& D = c.D;
    D.N = (int)N;
    D.p = p;
    D.nclass = c.nclass;
    D.task = c.task;
    D.ro = (int)round_up(p, 8);  // the regression target is read as an 8-byte float2
    D.rs = (int)round_up(D.ro + 8, 16);
    D.maxcat = P.maxcat > 0 ? P.maxcat : 10;
    D.has_cat = has_cat ? 1 : 0;
    float* xc = (float*)c.xc.get(N * p * 4);
    uint8_t* rows = (uint8_t*)c.rows.get(N * D.rs);
    float* edges = (float*)c.edges.get((size_t)p * 257 * 4);
    int* nb = (int*)c.nb.get(p * 4);
    int* kind = (int*)c.kind.get(p * 4);
    int* catd = (int*)c.cat.get(p * 4);
    int* lab = (int*)c.lab.get(N * 4);
    uint32_t* ka = (uint32_t*)c.keys_a.get(N * p * 4);
    uint32_t* kb = (uint32_t*)c.keys_b.get(N * p * 4);
    RFX_CUDA(cudaMemcpyAsync(ka, X, N * p * 4, cudaMemcpyHostToDevice, st));
    RFX_CUDA(cudaMemcpyAsync(catd, catv.data(), p * 4, cudaMemcpyHostToDevice, st));
    RFX_CUDA(cudaMemsetAsync(rows, 0, N * D.rs, st));
    float* yregp = nullptr;
    float* yvp = nullptr;
    if (c.task == RFX_TASK_REGRESSION) {
        yregp = (float*)c.yreg.get(N * 4);
        yvp = (float*)c.yv.get(N * 4);
        RFX_CUDA(cudaMemcpyAsync(yregp, in->y_reg, N * 4, cudaMemcpyHostToDevice, st));
        rfx::k_regr_targets<<<grid_for(N, 256, 4096), 256, 0, st>>>(yregp, (int)N, lab, yvp);
        RFX_LAUNCH("k_regr_targets");
    } else {
        RFX_CUDA(cudaMemcpyAsync(lab, c.labels0.data(), N * 4, cudaMemcpyHostToDevice, st));
    }
    {
        dim3 grid((unsigned)((N + 31) / 32), (unsigned)((p + 31) / 32));
        rfx::k_transpose<<<grid, dim3(32, 8), 0, st>>>(reinterpret_cast<const float*>(ka), (int)N, p, xc);
        RFX_LAUNCH("k_transpose");
    }
    rfx::k_sort_columns<<<p, 1024, 0, st>>>(xc, (int)N, catd, ka, kb);
    RFX_LAUNCH("k_sort_columns");
    rfx::k_edges<<<p, 1024, 0, st>>>(kb, (int)N, catd, P.nbins, reinterpret_cast<float*>(ka), edges, nb, kind);
    RFX_LAUNCH("k_edges");
    D.xc = xc;
    D.rows = rows;
    D.edges = edges;
    D.nb = nb;
    D.kind = kind;
    D.cat = catd;
    D.lab = lab;
    D.yreg = yregp;
    D.yv = yvp;
    rfx::k_pack_rows<<<grid_for(N * p, 256, 8192), 256, 0, st>>>(D);
    RFX_LAUNCH("k_pack_rows");
    // bootstrap weights (ignored by the unsupervised fit: src/rf_random_forest.cpp:1043)
    D.cumw = nullptr;
    D.totw = 0.0f;
    if (in->sample_weights && c.task != RFX_TASK_UNSUPERVISED) {
        float* w = (float*)c.keys_b.get(N * p * 4);  // scratch
        float* cum = (float*)c.cumw.get(N * 4);
        float* tot = (float*)c.totw.get(16);
        RFX_CUDA(cudaMemcpyAsync(w, in->sample_weights, N * 4, cudaMemcpyHostToDevice, st));
        rfx::k_cumw<<<1, 1, 0, st>>>(w, (int)N, cum, tot);
        RFX_LAUNCH("k_cumw");
        float h = 0.0f;
        RFX_CUDA(cudaMemcpyAsync(&h, tot, 4, cudaMemcpyDeviceToHost, st));
        RFX_CUDA(cudaStreamSynchronize(st));
        D.cumw = cum;
        D.totw = h;
    }
    {
        // the importance permutation (only importance reads it)
        D.perm = nullptr;
        c.perm_event = nullptr;
        if (P.compute_importance) {
            const PermEntry& pe = permutation_for(c.device, (int)N);
            D.perm = pe.perm;
            c.perm_event = pe.done;
        }
    }
    // accumulators
    int* no = (int*)c.nout.get(N * 4);
    RFX_CUDA(cudaMemsetAsync(no, 0, N * 4, st));
    if (c.nclass > 1) {
        int* v = (int*)c.votes.get(N * c.nclass * 4);
        RFX_CUDA(cudaMemsetAsync(v, 0, N * c.nclass * 4, st));
    } else {
        float* o = (float*)c.oob_sum.get(N * 4);
        RFX_CUDA(cudaMemsetAsync(o, 0, N * 4, st));
    }
    float* av = (float*)c.avimp.get(p * 4);
    float* sq = (float*)c.sqsd.get(p * 4);
    RFX_CUDA(cudaMemsetAsync(av, 0, p * 4, st));
    RFX_CUDA(cudaMemsetAsync(sq, 0, p * 4, st));
    c.prox = nullptr;
    c.prox_len = 0;
    forest_reset(c);
    leaves_reset(c);
    c.lr_rank = P.compute_proximity && P.lowrank_rank > 0 ? P.lowrank_rank : 0;
    c.lr_n = 0;
    c.lr_G = c.M + 2;
    c.lr_ready = false;
    if (P.compute_proximity && c.lr_rank == 0) {
        c.prox_len = (int64_t)c.R * (c.R - 1) / 2;
        c.prox = (int*)c.prox_own.get((size_t)c.prox_len * 4);
        RFX_CUDA(cudaMemsetAsync(c.prox, 0, (size_t)c.prox_len * 4, st));
    }
    c.trees_done = 0;
    c.tree_oob_n = 0;
    c.tree_oob_cap = 0;
    c.ts_n = 0;
    // batch capacity
    size_t per_tree = N * 4 * 6 + (size_t)c.M * (4 * 12 + 2 * P.mtry + 16) + (size_t)p * 16;
    if (c.task == RFX_TASK_REGRESSION && P.compute_importance) per_tree += N * (size_t)(p + 1) * 4;
    size_t free_b = 0, total_b = 0;
    RFX_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const size_t budget = std::min<size_t>(free_b / 2, (size_t)32 << 30);
    int Tcap = P.batch_trees > 0 ? P.batch_trees : 512;
    Tcap = (int)std::max<size_t>(1, std::min<size_t>((size_t)Tcap, budget / per_tree));
    Tcap = std::min(Tcap, 4096);
    alloc_batch(c, Tcap);
    RFX_CUDA(cudaMemsetAsync(c.B.counters, 0, 128, st));
    RFX_CUDA(cudaStreamSynchronize(st));
    c.loaded = true;
}

// Launch shapes of the histogram kernels (rfx_hist.cu).
struct HistCfg {
    rfx::HistArgs a;
    int threads, smem, grid;
    int small_warp_bytes, small_smem, small_grid;  // k_hist_small (classification)
    int lane_slots, lane_grid, lane_bytes;         // k_hist_lane (regression, <= kLaneSmall rows)
    int mid_grid = 0, mid_bytes = 0;               // k_hist_lane_mid (up to kLaneNode rows)
    int tiny_grid = 0, tiny_bytes = 0;             // k_hist_lane_tiny (up to kLaneTiny rows)
    rfx::PipeArgs pa;                              // k_hist_pipe (regression)
    int pipe_threads = 0, pipe_smem = 0, pipe_grid = 0;
};

HistCfg hist_cfg(Ctx& c) {
    HistCfg h;
    const bool regr = c.nclass == 1;
    const int mtry = c.prm.mtry;
    // k_hist_warp: per-warp histogram (regression: bin sums + counts; classification: class
    // counts, class-major) + counts, bin list, candidate flags, class totals
    const int wb = regr ? 2048 + 1024 + 512 + 1024 : 1024 * c.nclass + 1024 + 512 + 128;
    h.a.warp_bytes = (int)round_up(wb, 16);
    const int fit = std::max(1, (200 * 1024) / h.a.warp_bytes);
    h.a.warps = std::max(1, std::min({16, mtry, fit}));
    h.a.groups = (mtry + h.a.warps - 1) / h.a.warps;
    h.threads = 32 * h.a.warps;
    h.smem = h.a.warps * h.a.warp_bytes;
    int per_sm = 0;
    if (regr) {
        RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_warp_regr, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      std::max(h.smem, 48 * 1024)));
        RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_warp_regr, h.threads, h.smem));
    } else {
        RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_warp_class, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      std::max(h.smem, 48 * 1024)));
        RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_warp_class, h.threads, h.smem));
    }
    h.grid = c.sm_count * std::max(1, per_sm);
    // k_hist_pipe (regression): a producer warp + up to 16 consumer warps, a ring of four
    // 64-row chunks; RFX_HIST_PIPE=0 keeps k_hist_warp
    const char* pe = std::getenv("RFX_HIST_PIPE");
    if (regr && !(pe && pe[0] == '0')) {
        int pw = 16;
        if (const char* e = std::getenv("RFX_PIPE_WARPS")) pw = std::max(1, std::min(16, std::atoi(e)));
        h.pa.warps = std::min(pw, mtry);
        h.pa.groups = (mtry + h.pa.warps - 1) / h.pa.warps;
        h.pa.ch = 64;
        h.pa.rstride = c.D.rs + 16;
        h.pipe_threads = 32 * (h.pa.warps + 1);
        h.pipe_smem = rfx::kPipeHead + rfx::kPipeBufs * h.pa.ch * h.pa.rstride + h.pa.warps * (256 * 16 + 512);
        if (h.pipe_smem <= 220 * 1024) {
            RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_pipe, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          h.pipe_smem));
            RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_pipe,
                                                                   h.pipe_threads, h.pipe_smem));
            h.pipe_grid = c.sm_count * std::max(1, per_sm);
        }
    }
    // k_hist_small (classification): bin list, set words, class prefixes + totals
    h.small_warp_bytes = (int)round_up(256 + 64 + (257 * c.nclass) * 4, 16);
    h.small_smem = 8 * h.small_warp_bytes;
    h.small_grid = 0;
    h.lane_slots = 0;
    h.lane_grid = 0;
    h.lane_bytes = 0;
    if (!regr) {
        RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      std::max(h.small_smem, 48 * 1024)));
        RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_small, 256, h.small_smem));
        h.small_grid = c.sm_count * std::max(1, per_sm);
    } else if (mtry <= 32) {
        h.lane_slots = std::min(rfx::kLaneSlots, 32 / mtry);
        h.lane_bytes = rfx::lane_bytes(rfx::kLaneSmall, h.lane_slots);
        RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_lane, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      h.lane_bytes));
        RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_lane, 32, h.lane_bytes));
        h.lane_grid = c.sm_count * std::max(1, per_sm);
        h.mid_bytes = rfx::lane_bytes(rfx::kLaneNode, h.lane_slots);
        RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_lane_mid, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      h.mid_bytes));
        RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_lane_mid, 32, h.mid_bytes));
        h.mid_grid = c.sm_count * std::max(1, per_sm);
        h.tiny_bytes = rfx::lane_bytes(rfx::kLaneTiny, h.lane_slots);
        RFX_CUDA(cudaFuncSetAttribute(rfx::k_hist_lane_tiny, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      h.tiny_bytes));
        RFX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rfx::k_hist_lane_tiny, 32, h.tiny_bytes));
        h.tiny_grid = c.sm_count * std::max(1, per_sm);
    }
    return h;
}

// Host memcpy split over a few threads (large staged chunks).
void parallel_copy(char* dst, const char* src, size_t bytes) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t parts = std::min<size_t>(std::min<unsigned>(8u, hw), std::max<size_t>(1, bytes >> 22));
    if (parts <= 1) {
        std::memcpy(dst, src, bytes);
        return;
    }
    std::vector<std::thread> th;
    const size_t step = (bytes + parts - 1) / parts;
    for (size_t k = 0; k < parts; ++k) {
        const size_t off = k * step;
        if (off >= bytes) break;
        const size_t n = std::min(step, bytes - off);
        th.emplace_back([=] { std::memcpy(dst + off, src + off, n); });
    }
    for (auto& t : th) t.join();
}

// Pinned staging buffers shared by every context of the process (portable, so any device's
// stream may copy through them), allocated on first use and kept until exit; one copy at a
// time holds them.
struct Staging {
    std::mutex mu;
    void* buf[2] = {nullptr, nullptr};
};
Staging& staging() {
    static Staging* s = new Staging;  // never destroyed: exit-time order does not matter
    return *s;
}

// Device -> host copy on the context's stream, complete on return.  A page-locked
// destination takes one DMA; a pageable one (numpy arrays) goes through two pinned staging
// buffers, the DMA of chunk i + 1 running while host threads copy chunk i out.
void copy_d2h(Ctx& c, void* dst, const void* src, size_t bytes) {
    if (bytes == 0) return;
    cudaPointerAttributes at{};
    const cudaError_t qe = cudaPointerGetAttributes(&at, dst);
    if (qe != cudaSuccess) cudaGetLastError();  // only the query's own status is dropped
    const bool pinned = qe == cudaSuccess && at.type == cudaMemoryTypeHost;
    constexpr size_t kChunk = (size_t)32 << 20;
    if (pinned || bytes < ((size_t)4 << 20)) {
        RFX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
        return;
    }
    Staging& sg = staging();
    std::lock_guard<std::mutex> lock(sg.mu);
    if (!sg.buf[0] || !sg.buf[1]) {
        // both buffers or neither: allocate into locals and publish the pair
        void* nb[2] = {nullptr, nullptr};
        for (int b = 0; b < 2; ++b) {
            const cudaError_t ae = cudaHostAlloc(&nb[b], kChunk, cudaHostAllocPortable);
            if (ae != cudaSuccess) {
                if (nb[0]) cudaFreeHost(nb[0]);
                throw RfxError(RFX_ERR_OOM, std::string("cudaHostAlloc: ") + cudaGetErrorString(ae));
            }
        }
        sg.buf[0] = nb[0];
        sg.buf[1] = nb[1];
    }
    // on any exit, this context's copies into the shared buffers have finished before the
    // lock is released
    struct Drain {
        cudaStream_t st;
        ~Drain() { cudaStreamSynchronize(st); }
    } drain{c.st};
    if (!c.ev_stage[0])
        for (int b = 0; b < 2; ++b) RFX_CUDA(cudaEventCreateWithFlags(&c.ev_stage[b], cudaEventDisableTiming));
    const size_t nch = (bytes + kChunk - 1) / kChunk;
    auto issue = [&](size_t i) {
        const size_t off = i * kChunk, n = std::min(kChunk, bytes - off);
        RFX_CUDA(cudaMemcpyAsync(sg.buf[i & 1], (const char*)src + off, n, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaEventRecord(c.ev_stage[i & 1], c.st));
    };
    issue(0);
    for (size_t i = 0; i < nch; ++i) {
        if (i + 1 < nch) issue(i + 1);  // the other buffer: its host copy finished last round
        RFX_CUDA(cudaEventSynchronize(c.ev_stage[i & 1]));
        const size_t off = i * kChunk;
        parallel_copy((char*)dst + off, (const char*)sg.buf[i & 1], std::min(kChunk, bytes - off));
    }
}

constexpr int kLevelGroup = 8;  // tree levels enqueued per host synchronisation

void grow_batch(Ctx& c, int tree0, int T, rfx_trees* out, int out_off) {
    cudaStream_t st = c.st;
    rfx::Batch B = c.B;
    B.T = T;
    B.tree0 = tree0;
    const size_t N = c.N, M = c.M, p = c.p;
    const bool keep = c.prm.keep_tree_oob && c.task == RFX_TASK_REGRESSION;
    if (keep) {
        if (c.tree_oob_n + T > c.tree_oob_cap) {
            // grow the per-tree OOB prediction store, keeping what is there
            const int ncap = std::max(c.tree_oob_n + T, 2 * c.tree_oob_cap);
            DBuf nb;
            float* np = (float*)nb.get((size_t)ncap * N * 4);
            if (c.tree_oob_n > 0)
                RFX_CUDA(cudaMemcpyAsync(np, c.tree_oob_all.p, (size_t)c.tree_oob_n * N * 4,
                                         cudaMemcpyDeviceToDevice, st));
            RFX_CUDA(cudaStreamSynchronize(st));
            c.tree_oob_all.release();
            c.tree_oob_all = nb;
            nb.p = nullptr;
            c.tree_oob_cap = ncap;
        }
        B.tree_oob = (float*)c.tree_oob_all.p + (size_t)c.tree_oob_n * N;
    }
    RFX_CUDA(cudaMemsetAsync(B.nin, 0, T * N * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.status, 0, T * M * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.bestvar, 0, T * M * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.xbest, 0, T * M * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.treemap, 0, T * M * 8, st));
    RFX_CUDA(cudaMemsetAsync(B.nodeclass, 0, T * M * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.nodepred, 0, T * M * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.tnodewt, 0, T * M * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.oob_leaf, 0xff, T * N * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.counters, 0, 32, st));  // level counters; hist_bytes persists
    RFX_CUDA(cudaMemsetAsync(B.right, 0, T * 4, st));
    RFX_CUDA(cudaMemsetAsync(B.rightimp, 0, T * p * 4, st));
    const rfx::Data D = c.D;
    rfx::k_bootstrap<<<T, 256, 0, st>>>(D, B);
    RFX_LAUNCH("k_bootstrap");
    rfx::k_compact<<<T, 1024, 0, st>>>(D, B);
    RFX_LAUNCH("k_compact");
    c.launches += 2;
    c.trees += T;
    const HistCfg hc = hist_cfg(c);
    const int gw = c.sm_count * 8;
    // Levels are enqueued kLevelGroup at a time with one host synchronisation per group: a
    // level after the last one has no nodes, so its kernels find no work (the ping-pong
    // segment buffers are not touched) and k_level_begin records the number of levels that
    // had nodes (counters[7]).  RFX_LEVEL_LOG synchronises every level for its trace.
    const int group = c.level_log ? 1 : kLevelGroup;
    if (c.profiling && c.ev_hist.empty()) {
        c.ev_hist.resize(2 * kLevelGroup);
        for (auto& e : c.ev_hist) RFX_CUDA(cudaEventCreate(&e));
    }
    int level = 0;
    for (;;) {
        require(level < 1000000, RFX_ERR_DEVICE, "tree growth did not terminate");
        const int lv0 = level;
        for (int k = 0; k < group; ++k, ++level) {
            const int cl = level & 1;
            rfx::k_level_begin<<<1, 1024, 0, st>>>(B, level);
            rfx::k_node_eval<<<gw, 256, 0, st>>>(D, B, cl);
            rfx::k_draw<<<T, 256, 0, st>>>(D, B);
            rfx::k_srch_scan<<<1, 1024, 0, st>>>(B);
            rfx::k_task_records<<<T, 256, 0, st>>>(B);
            if (c.profiling) RFX_CUDA(cudaEventRecord(c.ev_hist[2 * k], st));
            if (c.nclass == 1) {
                if (hc.pipe_grid > 0)
                rfx::k_hist_pipe<<<hc.pipe_grid, hc.pipe_threads, hc.pipe_smem, st>>>(D, B, cl, hc.pa);
            else
                rfx::k_hist_warp_regr<<<hc.grid, hc.threads, hc.smem, st>>>(D, B, cl, hc.a);
                if (hc.lane_grid > 0) {
                    rfx::k_hist_lane_tiny<<<hc.tiny_grid, 32, hc.tiny_bytes, st>>>(D, B, cl, hc.lane_slots);
                    rfx::k_hist_lane<<<hc.lane_grid, 32, hc.lane_bytes, st>>>(D, B, cl, hc.lane_slots);
                    rfx::k_hist_lane_mid<<<hc.mid_grid, 32, hc.mid_bytes, st>>>(D, B, cl, hc.lane_slots);
                }
            } else {
                rfx::k_hist_warp_class<<<hc.grid, hc.threads, hc.smem, st>>>(D, B, cl, hc.a);
                rfx::k_hist_small<<<hc.small_grid, 256, hc.small_smem, st>>>(D, B, cl, hc.small_warp_bytes);
            }
            if (c.profiling) RFX_CUDA(cudaEventRecord(c.ev_hist[2 * k + 1], st));
            rfx::k_commit<<<T, 1024, 0, st>>>(D, B);
            rfx::k_partition<<<gw, 256, 0, st>>>(D, B, cl);
            rfx::k_partition_big<<<c.sm_count * 2, 256, 0, st>>>(D, B, cl);
            RFX_LAUNCH("level kernels");
            c.launches += 8 + (c.nclass != 1 ? 2 : (hc.lane_grid > 0 ? 4 : 1));
        }
        RFX_CUDA(cudaMemcpyAsync(c.h_counters, B.counters, c.level_log ? 80 : 32, cudaMemcpyDeviceToHost, st));
        RFX_CUDA(cudaStreamSynchronize(st));
        require(c.h_counters[3] == 0, RFX_ERR_DEVICE,
                "a histogram pipeline wait timed out (the kernel stopped and reported it)");
        const int real = std::min(level, c.h_counters[7]);  // levels so far that had nodes
        if (c.profiling) {
            for (int k = 0; k < real - lv0; ++k) {
                float ms = 0.0f;
                RFX_CUDA(cudaEventElapsedTime(&ms, c.ev_hist[2 * k], c.ev_hist[2 * k + 1]));
                c.hist_ms += ms;
                c.hist_launches += 1;
                if (c.level_log)
                    std::fprintf(stderr, "[rfx] tree0=%d level=%d nodes=%d searched=%d big=%d small=%d next=%d hist_ms=%.3f exact=%llu rounds=%llu steps=%llu d3=%llu\n",
                                 tree0, lv0 + k, c.h_counters[0], c.h_counters[1], c.h_counters[4], c.h_counters[6], c.h_counters[2], ms,
                                 *reinterpret_cast<unsigned long long*>(c.h_counters + 12),
                                 *reinterpret_cast<unsigned long long*>(c.h_counters + 14),
                                 *reinterpret_cast<unsigned long long*>(c.h_counters + 16),
                                 *reinterpret_cast<unsigned long long*>(c.h_counters + 18));
            }
        }
        if (c.h_counters[2] == 0) {
            c.levels += real;
            break;
        }
    }
    const dim3 rg((unsigned)((N + 255) / 256), (unsigned)T);
    rfx::k_oob_drop<<<rg, 256, 0, st>>>(D, B);
    rfx::k_votes<<<(unsigned)((N + 255) / 256), 256, 0, st>>>(
        D, B, (int*)c.nout.p, c.nclass > 1 ? (int*)c.votes.p : nullptr,
        c.nclass == 1 ? (float*)c.oob_sum.p : nullptr, B.tree_oob, (int)N);
    RFX_LAUNCH("oob kernels");
    c.launches += 2;
    if (c.prm.compute_importance) {
        RFX_CUDA(cudaStreamWaitEvent(st, c.perm_event, 0));
        rfx::k_imp_used<<<T, 256, 0, st>>>(D, B);
        if (c.nclass > 1) {
            rfx::k_imp_class<<<rg, 256, 0, st>>>(D, B);
            rfx::k_imp_class_rr<<<T, 256, 0, st>>>(D, B);
        } else {
            rfx::k_imp_pack<<<dim3((unsigned)((M + 255) / 256), (unsigned)T), 256, 0, st>>>(B);
            rfx::k_imp_regr<<<rg, 256, 0, st>>>(D, B);
            const size_t warps = (size_t)T * (p + 1);
            rfx::k_imp_regr_sum<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(D, B);
            rfx::k_imp_regr_rr<<<T, 256, 0, st>>>(D, B);
        }
        rfx::k_imp_fold<<<1, 256, 0, st>>>(D, B, (float*)c.avimp.p, (float*)c.sqsd.p);
        RFX_LAUNCH("importance kernels");
        c.launches += c.nclass > 1 ? 4 : 6;
    }
    if (c.prm.compute_proximity && c.prox) {
        if (c.profiling) RFX_CUDA(cudaEventRecord(c.ev0, st));
        // push (k_prox: one atomic per pair) or pull (k_prox_pull: every tile of the
        // triangle compares the batch's leaf codes), whichever the batch's exact pair count
        // makes cheaper: push ~ pairs / 2e10 s, pull ~ tiles * 128^2 * T/2 * 3 / 3e13 s
        bool pull = c.prox_mode == 2;
        if (c.prox_mode != 1) {
            const int R = c.R, Tp = T + (T & 1);
            uint16_t* code = (uint16_t*)c.b_pcode.get((size_t)Tp * R * 2);
            int* ocnt = (int*)c.b_pocnt.get((size_t)T * M * 4);
            unsigned long long* pairs_d = (unsigned long long*)c.b_ppairs.get(16);
            if (T & 1) RFX_CUDA(cudaMemsetAsync(code + (size_t)T * R, 0xFF, (size_t)R * 2, st));
            RFX_CUDA(cudaMemsetAsync(pairs_d, 0, 8, st));
            rfx::k_prox_codes<<<T, 1024, 0, st>>>(B, (int)N, R, code, ocnt, pairs_d);
            RFX_LAUNCH("k_prox_codes");
            c.launches += 1;
            unsigned long long pairs = 0;
            RFX_CUDA(cudaMemcpyAsync(&pairs, pairs_d, 8, cudaMemcpyDeviceToHost, st));
            RFX_CUDA(cudaStreamSynchronize(st));
            const long long nb = (R + 127) / 128;
            const long long tiles = nb * (nb + 1) / 2;
            if (c.prox_mode == 0) {
                const double push_s = (double)pairs / 2e10;
                const double pull_s = (double)tiles * 16384.0 * (Tp / 2) * 3.0 / 3e13;
                pull = pull_s < push_s;
            }
            if (pull) {
                rfx::k_prox_pull<<<(unsigned)tiles, 256, 0, st>>>(code, Tp, R, (int)nb, c.prox);
                RFX_LAUNCH("k_prox_pull");
                c.launches += 1;
                c.prox_pull_pairs += (double)pairs;
            }
        }
        if (!pull) {
            rfx::k_prox<<<rg, 256, 0, st>>>(D, B, c.R, c.prox);
            RFX_LAUNCH("k_prox");
            c.launches += 1;
        }
        if (c.profiling) {
            RFX_CUDA(cudaEventRecord(c.ev1, st));
            RFX_CUDA(cudaEventSynchronize(c.ev1));
            float ms = 0.0f;
            RFX_CUDA(cudaEventElapsedTime(&ms, c.ev0, c.ev1));
            c.prox_ms += ms;
        }
    }
    if (c.lr_rank > 0) lr_store_batch(c, B, T);
    if (c.prm.keep_forest) forest_store_batch(c, B, T);
    if (c.prm.keep_trees) {
        // device-to-device into the tree store (the host copies only when asked)
        const size_t o = (size_t)c.ts_n;
        auto st_cp = [&](DBuf& dst, const void* src, size_t per) {
            RFX_CUDA(cudaMemcpyAsync((char*)dst.p + o * per, src, (size_t)T * per,
                                     cudaMemcpyDeviceToDevice, st));
        };
        st_cp(c.ts_status, B.status, M * 4);
        st_cp(c.ts_bestvar, B.bestvar, M * 4);
        st_cp(c.ts_xbest, B.xbest, M * 4);
        st_cp(c.ts_treemap, B.treemap, 2 * M * 4);
        st_cp(c.ts_nodeclass, B.nodeclass, M * 4);
        st_cp(c.ts_nnode, B.nnode, 4);
        st_cp(c.ts_nodepred, B.nodepred, M * 4);
        st_cp(c.ts_tnodewt, B.tnodewt, M * 4);
        c.ts_n += T;
    }
    if (c.prm.keep_leaves) leaves_store_batch(c, B, T);
    if (keep) c.tree_oob_n += T;
    if (out) {
        auto cp = [&](void* dst, const void* src, size_t elems, size_t esz) {
            if (dst) copy_d2h(c, (char*)dst + (size_t)out_off * elems * esz, src, (size_t)T * elems * esz);
        };
        cp(out->nodestatus, B.status, M, 4);
        cp(out->bestvar, B.bestvar, M, 4);
        cp(out->xbestsplit, B.xbest, M, 4);
        cp(out->treemap, B.treemap, 2 * M, 4);
        cp(out->nodeclass, B.nodeclass, M, 4);
        cp(out->nnode, B.nnode, 1, 4);
        cp(out->nodepred, B.nodepred, M, 4);
        cp(out->tnodewt, B.tnodewt, M, 4);
        cp(out->nin, B.nin, N, 4);
        cp(out->oob_leaf, B.oob_leaf, N, 4);
        if (c.prm.compute_importance) {
            cp(out->tree_rr, B.rr, p, 4);
            if (out->tree_used) {
                if (c.nclass > 1) cp(out->tree_used, B.used, p, 1);
                else std::memset(out->tree_used + (size_t)out_off * p, 1, (size_t)T * p);
            }
        }
    }
    RFX_CUDA(cudaStreamSynchronize(st));
}

}  // namespace

void rfx_record_error(const std::string& msg) { g_last_error = msg; }

extern "C" {

const char* rfx_last_error(void) { return g_last_error.c_str(); }
int rfx_abi_version(void) { return RFX_ABI_VERSION; }

int rfx_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

long long rfx_cached_bytes(int device) { return cache_bytes(device); }

int rfx_empty_cache(int device) {
    return guarded([&] { cache_empty(device); });
}

void* rfx_create(int device) {
    Ctx* c = nullptr;
    const int rc = guarded([&] {
        int n = 0;
        RFX_CUDA(cudaGetDeviceCount(&n));
        require(device >= 0 && device < n, RFX_ERR_ARG, "device index out of range");
        c = new Ctx();
        c->device = device;
        RFX_CUDA(cudaSetDevice(device));
        RFX_CUDA(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device));
        RFX_CUDA(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking));
        RFX_CUDA(cudaMallocHost(&c->h_counters, 128));
    });
    if (rc != RFX_OK) {
        delete c;
        return nullptr;
    }
    return c;
}

void rfx_destroy(void* ctx) { delete static_cast<Ctx*>(ctx); }

int rfx_load(void* ctx, const rfx_fit_params* prm, const rfx_inputs* in) {
    return guarded([&] { load(*as_ctx(ctx), prm, in); });
}

void trees_reserve(Ctx& c, int need);

int rfx_grow(void* ctx, int tree_begin, int ntree, rfx_trees* out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded, RFX_ERR_STATE, "rfx_grow before rfx_load");
        require(tree_begin >= 0 && ntree >= 0, RFX_ERR_ARG, "bad tree range");
        lr_reserve(c, ntree);
        if (c.prm.keep_forest) forest_reserve(c, ntree);
        if (c.prm.keep_trees) trees_reserve(c, c.ts_n + ntree);
        for (int b0 = 0; b0 < ntree; b0 += c.Tcap) {
            const int T = std::min(c.Tcap, ntree - b0);
            grow_batch(c, tree_begin + b0, T, out, b0);
            c.trees_done += T;
            if (c.progress && c.progress(c.progress_user, b0 + T, ntree) != 0)
                throw RfxError(RFX_ERR_CANCELLED, "stopped by the progress callback");
        }
    });
}

int rfx_set_progress(void* ctx, rfx_progress_fn fn, void* user) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        c.progress = fn;
        c.progress_user = user;
    });
}

int rfx_reset_forest(void* ctx) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded, RFX_ERR_STATE, "rfx_reset_forest before rfx_load");
        const size_t N = c.N, p = c.p;
        cudaStream_t st = c.st;
        RFX_CUDA(cudaMemsetAsync(c.nout.p, 0, N * 4, st));
        if (c.nclass > 1) RFX_CUDA(cudaMemsetAsync(c.votes.p, 0, N * c.nclass * 4, st));
        else RFX_CUDA(cudaMemsetAsync(c.oob_sum.p, 0, N * 4, st));
        RFX_CUDA(cudaMemsetAsync(c.avimp.p, 0, p * 4, st));
        RFX_CUDA(cudaMemsetAsync(c.sqsd.p, 0, p * 4, st));
        if (c.prox) RFX_CUDA(cudaMemsetAsync(c.prox, 0, (size_t)c.prox_len * 4, st));
        forest_reset(c);
        leaves_reset(c);
        c.lr_n = 0;
        c.lr_ready = false;
        c.trees_done = 0;
        c.tree_oob_n = 0;
        c.ts_n = 0;
        RFX_CUDA(cudaStreamSynchronize(st));
    });
}

// Room for `need` trees in the device tree store, keeping the stored ones.
void trees_reserve(Ctx& c, int need) {
    if (need <= c.ts_cap) return;
    const int cap = std::max(need, 2 * c.ts_cap);
    const size_t M = c.M;
    DBuf* bufs[8] = {&c.ts_status, &c.ts_bestvar, &c.ts_xbest, &c.ts_treemap, &c.ts_nodeclass,
                     &c.ts_nnode, &c.ts_nodepred, &c.ts_tnodewt};
    const size_t per[8] = {M * 4, M * 4, M * 4, 2 * M * 4, M * 4, 4, M * 4, M * 4};
    for (int k = 0; k < 8; ++k) {
        DBuf nb;
        nb.get((size_t)cap * per[k]);
        if (c.ts_n > 0)
            RFX_CUDA(cudaMemcpyAsync(nb.p, bufs[k]->p, (size_t)c.ts_n * per[k],
                                     cudaMemcpyDeviceToDevice, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
        bufs[k]->release();
        *bufs[k] = nb;
        nb.p = nullptr;
    }
    c.ts_cap = cap;
}

int rfx_get_trees(void* ctx, int tree_begin, int count, rfx_trees* out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.prm.keep_trees, RFX_ERR_STATE, "the fit did not keep its trees (keep_trees)");
        require(out != nullptr && tree_begin >= 0 && count >= 0 && tree_begin + count <= c.ts_n,
                RFX_ERR_ARG, "bad tree range");
        const size_t M = c.M;
        auto cp = [&](void* dst, const DBuf& src, size_t per) {
            if (dst && count > 0)
                copy_d2h(c, dst, (const char*)src.p + (size_t)tree_begin * per, (size_t)count * per);
        };
        cp(out->nodestatus, c.ts_status, M * 4);
        cp(out->bestvar, c.ts_bestvar, M * 4);
        cp(out->xbestsplit, c.ts_xbest, M * 4);
        cp(out->treemap, c.ts_treemap, 2 * M * 4);
        cp(out->nodeclass, c.ts_nodeclass, M * 4);
        cp(out->nnode, c.ts_nnode, 4);
        cp(out->nodepred, c.ts_nodepred, M * 4);
        cp(out->tnodewt, c.ts_tnodewt, M * 4);
    });
}

int rfx_results(void* ctx, rfx_accum* r) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded, RFX_ERR_STATE, "rfx_results before rfx_load");
        require(r != nullptr, RFX_ERR_ARG, "null results");
        const size_t N = c.N;
        r->nclass = c.nclass;
        r->N = (int)N;
        cudaStream_t st = c.st;
        if (r->nout) RFX_CUDA(cudaMemcpyAsync(r->nout, c.nout.p, N * 4, cudaMemcpyDeviceToHost, st));
        if (c.nclass > 1) {
            if (r->votes)
                RFX_CUDA(cudaMemcpyAsync(r->votes, c.votes.p, N * c.nclass * 4, cudaMemcpyDeviceToHost, st));
            if (r->q) {
                float* q = (float*)c.qtmp.get(N * c.nclass * 4);
                float* w = nullptr;
                if (!c.classwt.empty()) {
                    w = (float*)c.cw_dev.get(c.nclass * 4);
                    RFX_CUDA(cudaMemcpyAsync(w, c.classwt.data(), c.nclass * 4, cudaMemcpyHostToDevice, st));
                }
                rfx::k_votes_to_q<<<grid_for(N * c.nclass, 256, 8192), 256, 0, st>>>(
                    (const int*)c.votes.p, w, (int)N, c.nclass, q);
                RFX_LAUNCH("k_votes_to_q");
                RFX_CUDA(cudaMemcpyAsync(r->q, q, N * c.nclass * 4, cudaMemcpyDeviceToHost, st));
            }
            if (r->labels) std::memcpy(r->labels, c.labels0.data(), N * 4);
        } else if (r->oob_sum) {
            RFX_CUDA(cudaMemcpyAsync(r->oob_sum, c.oob_sum.p, N * 4, cudaMemcpyDeviceToHost, st));
        }
        if (r->avimp) RFX_CUDA(cudaMemcpyAsync(r->avimp, c.avimp.p, c.p * 4, cudaMemcpyDeviceToHost, st));
        if (r->sqsd) RFX_CUDA(cudaMemcpyAsync(r->sqsd, c.sqsd.p, c.p * 4, cudaMemcpyDeviceToHost, st));
        RFX_CUDA(cudaStreamSynchronize(st));
    });
}

int rfx_fit(void* ctx, const rfx_fit_params* prm, const rfx_inputs* in, int ntree,
            rfx_trees* trees, rfx_accum* res) {
    int rc = rfx_load(ctx, prm, in);
    if (rc != RFX_OK) return rc;
    rc = rfx_grow(ctx, 0, ntree, trees);
    if (rc != RFX_OK) return rc;
    return res ? rfx_results(ctx, res) : RFX_OK;
}

int rfx_set_prox_buffer(void* ctx, int* upper_dev, int64_t len) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.prm.compute_proximity, RFX_ERR_STATE, "proximity is not enabled");
        require(len == (int64_t)c.R * (c.R - 1) / 2, RFX_ERR_ARG, "proximity buffer length mismatch");
        if (upper_dev == nullptr) {
            c.prox = (int*)c.prox_own.get((size_t)len * 4);
        } else {
            c.prox = upper_dev;
            c.prox_own.release();  // the caller's buffer replaces the context's own
        }
        RFX_CUDA(cudaMemsetAsync(c.prox, 0, (size_t)len * 4, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_get_prox_buffer(void* ctx, int** upper_dev, int64_t* len) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(upper_dev && len, RFX_ERR_ARG, "null output");
        *upper_dev = c.prox;
        *len = c.prox_len;
    });
}

int rfx_get_vote_buffers(void* ctx, int** nout_dev, int** votes_dev) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded, RFX_ERR_STATE, "not loaded");
        if (nout_dev) *nout_dev = (int*)c.nout.p;
        if (votes_dev) *votes_dev = c.nclass > 1 ? (int*)c.votes.p : nullptr;
    });
}

int rfx_prox_finish(void* ctx, const int* upper_dev, const int* nout_dev, int R, int row_begin,
                    int row_end, float* out_dev) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(upper_dev && nout_dev && out_dev, RFX_ERR_ARG, "null pointer");
        require(R >= 1 && row_begin >= 0 && row_begin <= row_end && row_end <= R, RFX_ERR_ARG,
                "bad row range");
        if (row_begin == 0 && row_end == R)
            RFX_CUDA(rfx::launch_prox_finish_full(upper_dev, nout_dev, R,
                                                  (double*)c.fin_inv.get((size_t)R * 8), out_dev, c.st));
        else
            RFX_CUDA(rfx::launch_prox_finish(upper_dev, nout_dev, R, row_begin, row_end, out_dev, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_prox_finish_packed(void* ctx, const int* upper_dev, int64_t elem_begin, int64_t elem_count,
                           const int* nout_dev, int R, float* out_dev) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(upper_dev && nout_dev && out_dev, RFX_ERR_ARG, "null pointer");
        const int64_t L = (int64_t)R * (R - 1) / 2;
        require(R >= 2 && elem_begin >= 0 && elem_count >= 0 && elem_begin + elem_count <= L,
                RFX_ERR_ARG, "bad element range");
        double* inv = (double*)c.fin_inv.get((size_t)R * 8);
        RFX_CUDA(rfx::launch_prox_finish_packed(upper_dev, elem_begin, elem_count, nout_dev, R, inv,
                                                out_dev, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_prox_dense(void* ctx, int row_begin, int row_end, float* out_host) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.prox, RFX_ERR_STATE, "proximity was not computed");
        require(out_host, RFX_ERR_ARG, "null output");
        const int R = c.R;
        require(row_begin >= 0 && row_begin <= row_end && row_end <= R, RFX_ERR_ARG, "bad row range");
        const int rows_per = (int)std::max<long long>(1, ((long long)256 << 20) / ((long long)R * 4));
        float* tmp = (float*)c.qtmp.get((size_t)std::min(rows_per, std::max(1, row_end - row_begin)) * R * 4);
        for (int r0 = row_begin; r0 < row_end; r0 += rows_per) {
            const int r1 = std::min(row_end, r0 + rows_per);
            const long long total = (long long)(r1 - r0) * R;
            if (r0 == 0 && r1 == R)  // the whole matrix in one pass: tile pairs
                RFX_CUDA(rfx::launch_prox_finish_full(c.prox, (const int*)c.nout.p, R,
                                                      (double*)c.fin_inv.get((size_t)R * 8), tmp, c.st));
            else
                RFX_CUDA(rfx::launch_prox_finish(c.prox, (const int*)c.nout.p, R, r0, r1, tmp, c.st));
            RFX_CUDA(cudaMemcpyAsync(out_host + (size_t)(r0 - row_begin) * R, tmp, (size_t)total * 4,
                                     cudaMemcpyDeviceToHost, c.st));
            RFX_CUDA(cudaStreamSynchronize(c.st));
        }
    });
}

int rfx_oob_fold(void* ctx, float* vec_dev) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.prm.keep_tree_oob && c.task == RFX_TASK_REGRESSION, RFX_ERR_STATE,
                "keep_tree_oob regression fit required");
        if (c.tree_oob_n > 0) {
            rfx::k_oob_fold<<<(c.N + 255) / 256, 256, 0, c.st>>>((const float*)c.tree_oob_all.p,
                                                               c.tree_oob_n, c.N, vec_dev);
            RFX_LAUNCH("k_oob_fold");
        }
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_votes_to_q(void* ctx, const int* votes_dev, const float* classwt, int N, int nclass,
                   float* q_dev) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(votes_dev && q_dev && N >= 0 && nclass >= 1, RFX_ERR_ARG, "bad arguments");
        float* w = nullptr;
        if (classwt) {
            w = (float*)c.cw_dev.get(nclass * 4);
            RFX_CUDA(cudaMemcpyAsync(w, classwt, nclass * 4, cudaMemcpyHostToDevice, c.st));
        }
        rfx::k_votes_to_q<<<grid_for((long long)N * nclass, 256, 8192), 256, 0, c.st>>>(
            votes_dev, w, N, nclass, q_dev);
        RFX_LAUNCH("k_votes_to_q");
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_copy_to_host(void* ctx, void* dst_host, const void* src_dev, size_t bytes) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(dst_host && src_dev, RFX_ERR_ARG, "null pointer");
        RFX_CUDA(cudaMemcpyAsync(dst_host, src_dev, bytes, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_get_stream(void* ctx, void** stream) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(stream != nullptr, RFX_ERR_ARG, "null output");
        *stream = (void*)c.st;
    });
}

int rfx_set_profiling(void* ctx, int on) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        if (on && !c.ev0) {
            RFX_CUDA(cudaEventCreate(&c.ev0));
            RFX_CUDA(cudaEventCreate(&c.ev1));
        }
        c.profiling = on != 0;
    });
}

int rfx_get_stats(void* ctx, rfx_stats* s) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(s != nullptr, RFX_ERR_ARG, "null output");
        unsigned long long hb[2] = {0, 0};
        if (c.B.hist_bytes) {
            RFX_CUDA(cudaMemcpyAsync(hb, c.B.hist_bytes, 16, cudaMemcpyDeviceToHost, c.st));
            RFX_CUDA(cudaStreamSynchronize(c.st));
        }
        s->kernel_launches = c.launches;
        s->hist_launches = c.hist_launches;
        s->hist_ms = c.hist_ms;
        s->hist_bytes = (double)hb[0];
        s->prox_pair_updates = (double)hb[1] + c.prox_pull_pairs;
        s->prox_ms = c.prox_ms;
        s->topk_ms = c.topk_ms;
        s->topk_tiles = c.topk_tiles;
        s->sketch_ms = c.sketch_ms;
        s->sketch_bytes = c.sketch_bytes;
        s->levels = c.levels;
        s->trees = c.trees;
    });
}

int rfx_reset_stats(void* ctx) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        c.launches = c.hist_launches = c.levels = c.trees = 0;
        c.hist_ms = 0.0;
        c.prox_ms = 0.0;
        c.prox_pull_pairs = 0.0;
        c.topk_ms = 0.0;
        c.topk_tiles = 0;
        c.sketch_ms = c.sketch_bytes = 0.0;
        if (c.B.hist_bytes) RFX_CUDA(cudaMemsetAsync(c.B.hist_bytes, 0, 16, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_sync(void* ctx) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

}  // extern "C"
