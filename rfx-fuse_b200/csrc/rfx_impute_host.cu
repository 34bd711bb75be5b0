// Host side of the imputation round (kernel in rfx_impute.cu, ABI in include/rfx_b200.h).
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "rfx_ctx.h"
#include "rfx_impute.h"
#include "rfx_kernels.h"

using namespace rfxh;

extern "C" {

int rfx_impute_round(void* ctx, const float* xc_host, const uint8_t* miss_host,
                     const uint8_t* is_cat_host, int n, int p, const int* cells_host, int ncells,
                     float* out_host) {
    return rfx_impute_round_ex(ctx, xc_host, miss_host, is_cat_host, n, p, cells_host, ncells, -1,
                               RFX_IMPUTE_MEAN, out_host);
}

int rfx_impute_round_ex(void* ctx, const float* xc_host, const uint8_t* miss_host,
                        const uint8_t* is_cat_host, int n, int p, const int* cells_host,
                        int ncells, int top_k, int aggregation, float* out_host) {
    return guarded([&] {
        require(top_k >= -1, RFX_ERR_ARG, "top_k must be -1 (none) or >= 0");
        require(aggregation == RFX_IMPUTE_MEAN || aggregation == RFX_IMPUTE_MEDIAN, RFX_ERR_ARG,
                "unknown aggregation");
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.prox, RFX_ERR_STATE, "dense proximity counts are required (fit with compute_proximity)");
        require(n == c.R, RFX_ERR_ARG, "n must equal the proximity rows of the fit");
        require(xc_host && miss_host && is_cat_host && p >= 1 && ncells >= 0, RFX_ERR_ARG, "bad arguments");
        require(ncells == 0 || (cells_host && out_host), RFX_ERR_ARG, "null cells / output");
        if (ncells == 0) return;
        for (int q = 1; q < ncells; ++q)
            require(cells_host[2 * q] >= cells_host[2 * (q - 1)], RFX_ERR_ARG, "cells must be sorted by row");
        cudaStream_t st = c.st;
        const size_t N = n, P = p;
        float* xc = (float*)c.i_x.get(P * N * 4);
        uint8_t* miss = (uint8_t*)c.i_miss.get(P * N);
        uint8_t* cat = (uint8_t*)c.i_cat.get(P);
        RFX_CUDA(cudaMemcpyAsync(xc, xc_host, P * N * 4, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaMemcpyAsync(miss, miss_host, P * N, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaMemcpyAsync(cat, is_cat_host, P, cudaMemcpyHostToDevice, st));
        // rows with missing cells and their ranges of cells
        std::vector<int> rows, row_cells;
        for (int q = 0; q < ncells; ++q) {
            const int i = cells_host[2 * q];
            require(i >= 0 && i < n && cells_host[2 * q + 1] >= 0 && cells_host[2 * q + 1] < p,
                    RFX_ERR_ARG, "cell outside the matrix");
            if (rows.empty() || rows.back() != i) {
                rows.push_back(i);
                row_cells.push_back(q);
            }
        }
        row_cells.push_back(ncells);
        const int nrows = (int)rows.size();
        // finished proximity rows in blocks of at most 4 GiB
        const int rows_per = (int)std::max<long long>(1, ((long long)1 << 32) / ((long long)N * 4));
        float* S = (float*)c.i_S.get((size_t)std::min<long long>(rows_per, n) * N * 4);
        const int max_leaves = n / 32 + 4;
        const long long stride = rfx::impute_scratch_floats(n, max_leaves);
        // 4 blocks of 8 warps per SM, fewer when the per-warp scratch passes 8 GiB in total
        const long long fit = std::max<long long>(1, ((long long)1 << 33) / (stride * 4 * 8));
        const int blocks = (int)std::min<long long>((long long)c.sm_count * 4, fit);
        float* scratch = (float*)c.i_scratch.get((size_t)blocks * 8 * stride * 4);
        int* cells = (int*)c.i_cells.get((size_t)ncells * 8 + (size_t)(2 * nrows + 1) * 4);
        int* drows = cells + 2 * (size_t)ncells;
        int* drow_cells = drows + nrows;
        float* out = (float*)c.i_out.get((size_t)ncells * 4);
        RFX_CUDA(cudaMemcpyAsync(cells, cells_host, (size_t)ncells * 8, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaMemcpyAsync(drows, rows.data(), (size_t)nrows * 4, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaMemcpyAsync(drow_cells, row_cells.data(), (size_t)(nrows + 1) * 4,
                                 cudaMemcpyHostToDevice, st));
        static const bool want_prof = std::getenv("RFX_IMPUTE_PROF") != nullptr;
        unsigned long long* prof = nullptr;
        if (want_prof) {
            prof = (unsigned long long*)c.i_prof.get(16 * 8);
            RFX_CUDA(cudaMemsetAsync(prof, 0, 16 * 8, st));
        }
        int b0 = 0;
        for (int r0 = 0; r0 < n && b0 < nrows; r0 += rows_per) {
            const int r1 = std::min(n, r0 + rows_per);
            int b1 = b0;
            while (b1 < nrows && rows[b1] < r1) ++b1;
            if (b1 == b0) continue;
            // finish only the span of rows that have cells
            const int f0 = rows[b0], f1 = rows[b1 - 1] + 1;
            RFX_CUDA(rfx::launch_prox_finish(c.prox, (const int*)c.nout.p, n, f0, f1, S, st));
            rfx::ImputeArgs a;
            a.S = S;
            a.ldS = n;
            a.r0 = f0;
            a.n = n;
            a.p = p;
            a.xc = xc;
            a.miss = miss;
            a.is_cat = cat;
            a.cells = cells;
            a.rows = drows + b0;
            a.row_cells = drow_cells + b0;
            a.nrows = b1 - b0;
            a.out = out;
            a.scratch = scratch;
            a.scratch_stride = stride;
            a.max_leaves = max_leaves;
            a.top_k = top_k;
            a.median = aggregation == RFX_IMPUTE_MEDIAN ? 1 : 0;
            a.prof = prof;
            const int grid = std::min(blocks, (a.nrows + 7) / 8);
            rfx::k_impute<<<grid, 256, 0, st>>>(a);
            RFX_LAUNCH("k_impute");
            c.launches += 2;
            b0 = b1;
        }
        RFX_CUDA(cudaMemcpyAsync(out_host, out, (size_t)ncells * 4, cudaMemcpyDeviceToHost, st));
        RFX_CUDA(cudaStreamSynchronize(st));
        if (prof) {
            unsigned long long hp[16] = {};
            RFX_CUDA(cudaMemcpy(hp, prof, 16 * 8, cudaMemcpyDeviceToHost));
            std::fprintf(stderr,
                         "impute prof: rows %d sum_m %llu max_m %llu sum_mm %llu | cycles scan %llu "
                         "compact %llu cont %llu cat %llu | cells cont %llu cat %llu distinct %llu\n",
                         nrows, hp[0], hp[7], hp[1], hp[2], hp[3], hp[4], hp[5], hp[8], hp[9], hp[6]);
        }
    });
}

}  // extern "C"
