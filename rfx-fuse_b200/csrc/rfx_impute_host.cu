// Host side of the imputation round (kernel in rfx_impute.cu, ABI in include/rfx_b200.h).
#include <vector>

#include "rfx_ctx.h"
#include "rfx_impute.h"
#include "rfx_kernels.h"

using namespace rfxh;

extern "C" {

int rfx_impute_round(void* ctx, const float* xc_host, const uint8_t* miss_host,
                     const uint8_t* is_cat_host, int n, int p, const int* cells_host, int ncells,
                     float* out_host) {
    return guarded([&] {
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
        // finished proximity rows in blocks of at most 1 GiB
        const int rows_per = (int)std::max<long long>(1, ((long long)1 << 30) / ((long long)N * 4));
        float* S = (float*)c.i_S.get((size_t)std::min<long long>(rows_per, n) * N * 4);
        const int max_leaves = n / 32 + 4;
        const long long stride = rfx::impute_scratch_floats(n, max_leaves);
        const int blocks = c.sm_count * 2;
        float* scratch = (float*)c.i_scratch.get((size_t)blocks * 8 * stride * 4);
        int* cells = (int*)c.i_cells.get((size_t)ncells * 8);
        float* out = (float*)c.i_out.get((size_t)ncells * 4);
        RFX_CUDA(cudaMemcpyAsync(cells, cells_host, (size_t)ncells * 8, cudaMemcpyHostToDevice, st));
        int q0 = 0;
        for (int r0 = 0; r0 < n && q0 < ncells; r0 += rows_per) {
            const int r1 = std::min(n, r0 + rows_per);
            int q1 = q0;
            while (q1 < ncells && cells_host[2 * q1] < r1) ++q1;
            if (q1 == q0) continue;
            RFX_CUDA(rfx::launch_prox_finish(c.prox, (const int*)c.nout.p, n, r0, r1, S, st));
            rfx::ImputeArgs a;
            a.S = S;
            a.ldS = n;
            a.r0 = r0;
            a.n = n;
            a.p = p;
            a.xc = xc;
            a.miss = miss;
            a.is_cat = cat;
            a.cells = cells + 2 * (size_t)q0;
            a.ncells = q1 - q0;
            a.out = out + q0;
            a.scratch = scratch;
            a.scratch_stride = stride;
            a.max_leaves = max_leaves;
            const int grid = std::min(blocks, (a.ncells + 7) / 8);
            rfx::k_impute<<<grid, 256, 0, st>>>(a);
            RFX_LAUNCH("k_impute");
            c.launches += 2;
            q0 = q1;
        }
        RFX_CUDA(cudaMemcpyAsync(out_host, out, (size_t)ncells * 4, cudaMemcpyDeviceToHost, st));
        RFX_CUDA(cudaStreamSynchronize(st));
    });
}

}  // extern "C"
