// Host side of prediction (kernels in rfx_predict.cu, ABI in include/rfx_b200.h): the
// device forest kept from a fit (keep_forest) or loaded from host arrays, and rfx_predict.
#include <cstring>
#include <vector>

#include "rfx_ctx.h"
#include "rfx_kernels.h"
#include "rfx_predict.h"

namespace rfxh {

void forest_reset(Ctx& c) {
    c.f_T = 0;
    c.f_M = c.M;
    c.f_p = c.p;
    c.f_nclass = c.nclass;
    c.f_task = c.task;
    c.f_classwt = false;
    if (!c.prm.keep_forest) return;
    int* cat = (int*)c.f_cat.get((size_t)c.p * 4);
    RFX_CUDA(cudaMemcpyAsync(cat, c.D.cat, (size_t)c.p * 4, cudaMemcpyDeviceToDevice, c.st));
    if (c.task == RFX_TASK_CLASSIFICATION && !c.classwt.empty()) {
        float* w = (float*)c.f_cw.get(c.classwt.size() * 4);
        RFX_CUDA(cudaMemcpyAsync(w, c.classwt.data(), c.classwt.size() * 4, cudaMemcpyHostToDevice, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));  // classwt is a host vector
        c.f_classwt = true;
    }
}

void forest_reserve(Ctx& c, int extra) {
    const int need = c.f_T + extra;
    if (need <= c.f_cap) return;
    const size_t M = c.f_M;
    DBuf nodes, root;
    nodes.get((size_t)need * M * sizeof(rfx::PNode));
    root.get((size_t)need * 4);
    if (c.f_T > 0) {
        RFX_CUDA(cudaMemcpyAsync(nodes.p, c.f_nodes.p, (size_t)c.f_T * M * sizeof(rfx::PNode),
                                 cudaMemcpyDeviceToDevice, c.st));
        RFX_CUDA(cudaMemcpyAsync(root.p, c.f_root.p, (size_t)c.f_T * 4, cudaMemcpyDeviceToDevice, c.st));
    }
    RFX_CUDA(cudaStreamSynchronize(c.st));
    c.f_nodes.release();
    c.f_root.release();
    c.f_nodes = nodes;
    c.f_root = root;
    nodes.p = root.p = nullptr;
    c.f_cap = need;
}

void forest_store_batch(Ctx& c, const rfx::Batch& B, int T) {
    forest_reserve(c, T);
    const size_t M = c.f_M;
    const dim3 grid((unsigned)std::min<size_t>((M + 255) / 256, 64), (unsigned)T);
    rfx::k_pack_forest<<<grid, 256, 0, c.st>>>(B, c.task, (rfx::PNode*)c.f_nodes.p + (size_t)c.f_T * M,
                                                (float*)c.f_root.p + c.f_T);
    RFX_LAUNCH("k_pack_forest");
    c.launches += 1;
    c.f_T += T;
}

}  // namespace rfxh

using namespace rfxh;

extern "C" {

int rfx_load_forest(void* ctx, const rfx_forest* f) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(f && f->nodestatus && f->bestvar && f->xbestsplit && f->treemap && f->cat,
                RFX_ERR_ARG, "incomplete forest");
        require(f->task == RFX_TASK_CLASSIFICATION || f->task == RFX_TASK_REGRESSION,
                RFX_ERR_UNSUPPORTED, "prediction is for classification and regression forests");
        require(f->task != RFX_TASK_CLASSIFICATION || f->nodeclass, RFX_ERR_ARG, "nodeclass required");
        require(f->task != RFX_TASK_REGRESSION || f->nodepred, RFX_ERR_ARG, "nodepred required");
        require(f->ntree >= 1 && f->maxnode >= 1 && f->p >= 1, RFX_ERR_ARG, "bad forest shape");
        require(f->task == RFX_TASK_REGRESSION || (f->nclass >= 1 && f->nclass <= rfx::kPredMaxClass),
                RFX_ERR_UNSUPPORTED, "nclass must be in [1, 32]");
        const size_t T = f->ntree, M = f->maxnode;
        std::vector<rfx::PNode> nodes(T * M);
        std::vector<float> root(T);
        for (size_t k = 0; k < T * M; ++k) {
            rfx::PNode& nd = nodes[k];
            if (f->nodestatus[k] == -1) {
                nd.feat = -1;
                if (f->task == RFX_TASK_REGRESSION) {
                    nd.val = f->nodepred[k];
                } else {
                    std::memcpy(&nd.val, &f->nodeclass[k], 4);
                }
                nd.left = nd.right = 0;
            } else {
                nd.feat = f->bestvar[k];
                nd.val = f->xbestsplit[k];
                nd.left = f->treemap[2 * k];
                nd.right = f->treemap[2 * k + 1];
            }
        }
        for (size_t t = 0; t < T; ++t) root[t] = f->nodepred ? f->nodepred[t * M] : 0.0f;
        c.f_T = 0;
        c.f_cap = 0;
        c.f_nodes.release();
        c.f_root.release();
        c.f_M = (int)M;
        forest_reserve(c, (int)T);
        RFX_CUDA(cudaMemcpyAsync(c.f_nodes.p, nodes.data(), nodes.size() * sizeof(rfx::PNode),
                                 cudaMemcpyHostToDevice, c.st));
        RFX_CUDA(cudaMemcpyAsync(c.f_root.p, root.data(), T * 4, cudaMemcpyHostToDevice, c.st));
        int* cat = (int*)c.f_cat.get((size_t)f->p * 4);
        RFX_CUDA(cudaMemcpyAsync(cat, f->cat, (size_t)f->p * 4, cudaMemcpyHostToDevice, c.st));
        c.f_classwt = false;
        if (f->task == RFX_TASK_CLASSIFICATION && f->classwt) {
            float* w = (float*)c.f_cw.get((size_t)f->nclass * 4);
            RFX_CUDA(cudaMemcpyAsync(w, f->classwt, (size_t)f->nclass * 4, cudaMemcpyHostToDevice, c.st));
            c.f_classwt = true;
        }
        RFX_CUDA(cudaStreamSynchronize(c.st));  // host staging vectors go out of scope
        c.f_T = (int)T;
        c.f_p = f->p;
        c.f_nclass = f->task == RFX_TASK_REGRESSION ? 1 : f->nclass;
        c.f_task = f->task;
    });
}

int rfx_predict(void* ctx, const float* X_host, int n, int p, int* class_out, float* proba_out,
                float* value_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.f_T > 0, RFX_ERR_STATE, "no forest on the device (fit with keep_forest or rfx_load_forest)");
        require(c.f_task == RFX_TASK_CLASSIFICATION || c.f_task == RFX_TASK_REGRESSION,
                RFX_ERR_UNSUPPORTED, "prediction is for classification and regression forests");
        require(X_host && n >= 0 && p == c.f_p, RFX_ERR_ARG, "X must be [n][p] with the forest's p");
        require(c.f_task != RFX_TASK_CLASSIFICATION || c.f_nclass <= rfx::kPredMaxClass,
                RFX_ERR_UNSUPPORTED, "more than 32 classes");
        if (n == 0) return;
        cudaStream_t st = c.st;
        const int T = c.f_T, nc = c.f_nclass;
        const bool regr = c.f_task == RFX_TASK_REGRESSION;
        // rows per chunk: per-tree outcomes of at most 512 MiB
        const size_t per_row = (size_t)T * (regr ? 4 : 1);
        const int chunk = (int)std::max<size_t>(1, std::min<size_t>((size_t)n, ((size_t)512 << 20) / per_row));
        float* xr = (float*)c.p_X.get((size_t)chunk * p * 4);
        float* xc = (float*)c.p_xc.get((size_t)chunk * p * 4);
        uint8_t* vote = regr ? nullptr : (uint8_t*)c.p_vote.get((size_t)chunk * T);
        float* val = regr ? (float*)c.p_val.get((size_t)chunk * T * 4) : nullptr;
        int* cls = (int*)c.p_cls.get((size_t)chunk * 4);
        float* proba = (float*)c.p_proba.get((size_t)chunk * std::max(nc, 1) * 4);
        float* pred = (float*)c.p_pred.get((size_t)chunk * 4);
        const float* cw = c.f_classwt ? (const float*)c.f_cw.p : nullptr;
        for (int s0 = 0; s0 < n; s0 += chunk) {
            const int m = std::min(chunk, n - s0);
            RFX_CUDA(cudaMemcpyAsync(xr, X_host + (size_t)s0 * p, (size_t)m * p * 4,
                                     cudaMemcpyHostToDevice, st));
            {
                const dim3 grid((unsigned)((m + 31) / 32), (unsigned)((p + 31) / 32));
                rfx::k_transpose<<<grid, dim3(32, 8), 0, st>>>(xr, m, p, xc);
                RFX_LAUNCH("k_transpose");
            }
            const dim3 wg((unsigned)((m + 127) / 128), (unsigned)T);
            rfx::k_predict_walk<<<wg, 128, 0, st>>>((const rfx::PNode*)c.f_nodes.p,
                                                    (const float*)c.f_root.p, c.f_M, T, xc, m, p,
                                                    (const int*)c.f_cat.p, c.f_task, nc, vote, val);
            RFX_LAUNCH("k_predict_walk");
            rfx::k_predict_reduce<<<(m + 127) / 128, 128, 0, st>>>(vote, val, m, T, c.f_task, nc, cw,
                                                                  cls, proba, pred);
            RFX_LAUNCH("k_predict_reduce");
            c.launches += 3;
            if (regr) {
                if (value_out)
                    RFX_CUDA(cudaMemcpyAsync(value_out + s0, pred, (size_t)m * 4, cudaMemcpyDeviceToHost, st));
            } else {
                if (class_out)
                    RFX_CUDA(cudaMemcpyAsync(class_out + s0, cls, (size_t)m * 4, cudaMemcpyDeviceToHost, st));
                if (proba_out)
                    RFX_CUDA(cudaMemcpyAsync(proba_out + (size_t)s0 * nc, proba, (size_t)m * nc * 4,
                                             cudaMemcpyDeviceToHost, st));
            }
            RFX_CUDA(cudaStreamSynchronize(st));
        }
    });
}

}  // extern "C"
