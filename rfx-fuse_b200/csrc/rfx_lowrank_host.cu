// Host orchestration of the low-rank proximity path (kernels in rfx_lowrank.cu and
// rfx_topk.cu; ABI in include/rfx_b200.h).
//
// Fit: with lowrank_rank > 0 every grown batch stores its trees' leaf groups (row -> group
// code, rows ordered by leaf and in-bag/OOB, group offsets) instead of dense counts.
// Build: randomized range finder on S (Halko, Martinsson & Tropp, SIAM Review 53(2), 2011,
// algorithms 4.3/4.4 with Cholesky-QR twice as the orthonormaliser), then the eigenpairs of
// the r x r projection Q^T S Q; A = Q V_k sqrt(max(lambda_k, 0)) is the best rank-k
// positive semidefinite approximation of S within range(Q); A is stored int8 per row.
#include <cub/cub.cuh>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "rfx_ctx.h"
#include "rfx_lowrank.h"

namespace rfxh {

namespace {

int nq_of(int W) { return W / 32; }

// CZ = C Z over the stored trees, Z / CZ device [R][W] (W a multiple of 32, <= 256).
void apply_counts(Ctx& c, const float* Z, int W, float* CZ) {
    cudaStream_t st = c.st;
    const int R = c.R, N = c.N, G = c.lr_G;
    RFX_CUDA(cudaMemsetAsync(CZ, 0, (size_t)R * W * 4, st));
    if (c.lr_n == 0) return;
    const size_t per_tree = (size_t)G * W * 4;
    const int Tc = (int)std::max<size_t>(1, std::min<size_t>((size_t)c.lr_n, ((size_t)1 << 30) / per_tree));
    float* LS = (float*)c.lr_ls.get((size_t)Tc * per_tree);
    const uint16_t* code = (const uint16_t*)c.lr_code.p;
    const int* order = (const int*)c.lr_order.p;
    const int* goff = (const int*)c.lr_goff.p;
    const int* ng = (const int*)c.lr_ngroups.p;
    const int nq = nq_of(W);
    if (c.profiling) RFX_CUDA(cudaEventRecord(c.ev0, st));
    for (int t0 = 0; t0 < c.lr_n; t0 += Tc) {
        const int T = std::min(Tc, c.lr_n - t0);
        const dim3 g((unsigned)((G - 1 + 7) / 8), (unsigned)T);
        require(rfx::lr_launch_leafsum(nq, g, st, order + (size_t)t0 * N,
                                       goff + (size_t)t0 * G, ng + t0, N, G, T, Z, LS),
                RFX_ERR_ARG, "sketch width out of range");
        RFX_LAUNCH("k_lr_leafsum");
        rfx::lr_launch_scatter(nq, (R + 7) / 8, st, code + (size_t)t0 * N, N, R, T, G, LS, CZ);
        RFX_LAUNCH("k_lr_scatter");
        c.launches += 2;
    }
    if (c.profiling) {
        RFX_CUDA(cudaEventRecord(c.ev1, st));
        RFX_CUDA(cudaEventSynchronize(c.ev1));
        float ms = 0.0f;
        RFX_CUDA(cudaEventElapsedTime(&ms, c.ev0, c.ev1));
        c.sketch_ms += ms;
        // per tree: gather of the R rows of Z into leaf sums, gather of a leaf sum per row
        // (W floats each), plus the row order (4 B) and group code (2 B) of every row
        c.sketch_bytes += (double)c.lr_n * ((double)R * W * 4.0 * 2.0 + (double)R * 6.0);
    }
}

// Y = S X (X, Y device [R][r]); `reduce` sums C [X | D X] over the processes first.
void apply_s(Ctx& c, const float* X, int r, const int* nout, float* Y, rfx_reduce_fn reduce,
             void* user) {
    cudaStream_t st = c.st;
    const int R = c.R;
    const int W = (int)round_up(2 * r, 32);
    float* Z = (float*)c.lr_Z.get((size_t)R * W * 4);
    float* CZ = (float*)c.lr_CZ.get((size_t)R * W * 4);
    rfx::k_lr_prep<<<grid_for((long long)R * W, 256, c.sm_count * 16), 256, 0, st>>>(X, R, r, nout, W, Z);
    RFX_LAUNCH("k_lr_prep");
    apply_counts(c, Z, W, CZ);
    if (reduce) {
        RFX_CUDA(cudaStreamSynchronize(st));
        require(reduce(user, CZ, (int64_t)R * W) == 0, RFX_ERR_DEVICE, "sketch reduction failed");
    }
    rfx::k_lr_combine<<<grid_for((long long)R * r, 256, c.sm_count * 16), 256, 0, st>>>(CZ, W, X, R, r, nout, Y);
    RFX_LAUNCH("k_lr_combine");
    c.launches += 2;
}

void set_smem(const void* f, size_t bytes) {
    RFX_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)std::max<size_t>(bytes, 48 * 1024)));
}

// G = A^T B (fp64 [ra][rb]); sym: symmetrised.
void gram(Ctx& c, const float* A, int ra, const float* B, int rb, int sym, double* G) {
    cudaStream_t st = c.st;
    const int R = c.R;
    const int nblk = (int)std::max(1LL, std::min<long long>((R + 255) / 256, (long long)c.sm_count * 2));
    const int rpb = (int)round_up((R + nblk - 1) / nblk, 32);
    double* part = (double*)c.lr_part.get((size_t)nblk * ra * rb * 8);
    rfx::k_lr_gram<<<nblk, 256, 0, st>>>(A, ra, B, rb, R, rpb, part);
    RFX_LAUNCH("k_lr_gram");
    rfx::k_lr_gram_reduce<<<(ra * rb + 127) / 128, 128, 0, st>>>(part, nblk, ra, rb, sym, G);
    RFX_LAUNCH("k_lr_gram_reduce");
    c.launches += 2;
    if (sym) {
        rfx::k_lr_symmetrize<<<1, 256, 0, st>>>(G, ra);
        RFX_LAUNCH("k_lr_symmetrize");
        c.launches += 1;
    }
}

// Q = orthonormal basis of range(Y) by Cholesky-QR twice; Y is overwritten.
void orth(Ctx& c, float* Y, int r, float* Q, double* G, double* Uinv) {
    cudaStream_t st = c.st;
    const int R = c.R;
    set_smem((const void*)rfx::k_lr_chol_inv, (size_t)2 * r * r * 8);
    set_smem((const void*)rfx::k_lr_rowmat, (size_t)r * r * 8);
    float* src = Y;
    float* dst = Q;
    for (int pass = 0; pass < 2; ++pass) {
        gram(c, src, r, src, r, 1, G);
        rfx::k_lr_chol_inv<<<1, 128, (size_t)2 * r * r * 8, st>>>(G, r, Uinv);
        RFX_LAUNCH("k_lr_chol_inv");
        rfx::k_lr_rowmat<<<c.sm_count * 4, 256, (size_t)r * r * 8, st>>>(src, R, r, Uinv, r, dst);
        RFX_LAUNCH("k_lr_rowmat");
        c.launches += 2;
        std::swap(src, dst);
    }
    // two passes: the result is back in Y; copy to Q
    RFX_CUDA(cudaMemcpyAsync(Q, src, (size_t)R * r * 4, cudaMemcpyDeviceToDevice, st));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::mutex mu;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        RFX_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        require(p != nullptr && q == cudaDriverEntryPointSuccess, RFX_ERR_CUDA,
                "cuTensorMapEncodeTiled is not available");
        fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// Tensor map of the bf16 factor rows [Rpad][64]: boxes of 128 rows x 64 columns, 128-byte
// swizzle (one box row is exactly one 128-byte swizzle span).
CUtensorMap factor_map(Ctx& c, void* rows) {
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    const cuuint64_t dims[2] = {(cuuint64_t)rfx::kLrK, (cuuint64_t)c.lr_Rpad};
    const cuuint64_t strides[1] = {(cuuint64_t)rfx::kLrK * 2};
    const cuuint32_t box[2] = {(cuuint32_t)rfx::kLrK, 128};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, dims, strides,
                                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, RFX_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    return tm;
}

// One launch of the product kernel for original rows [r0, r1).  Top-k (k > 0) runs on the
// rows stored by descending bound factor n (early stop); the dense product (k == 0) on the
// identity order.
void run_product(Ctx& c, int r0, int r1, int k, int* oi, float* ov, float* dense, long long ld,
                 int blk0 = -1, int blk1 = -1) {
    cudaStream_t st = c.st;
    const bool ordered = k > 0;
    const CUtensorMap tm = factor_map(c, ordered ? c.lr_qbp.p : c.lr_qb.p);
    int* err = (int*)c.lr_err.get(16);
    RFX_CUDA(cudaMemsetAsync(err, 0, 16, st));
    rfx::TopkArgs a;
    a.R = c.lr_R;
    a.r0 = r0;
    a.r1 = r1;
    a.ntiles = c.lr_Rpad / rfx::kTkCols;
    a.k = k;
    a.scale = (const float*)(ordered ? c.lr_sp.p : c.lr_s.p);
    a.perm = ordered ? (const int*)c.lr_perm.p : nullptr;
    a.norm = ordered ? (const float*)c.lr_np.p : nullptr;
    a.blocks = nullptr;
    a.out_pos0 = -1;
    int grid = (r1 - r0 + rfx::kTkRows - 1) / rfx::kTkRows;
    if (ordered && blk0 >= 0) {
        // an explicit range of stored-order blocks: every row in them, outputs by position
        std::vector<int> blk;
        for (int b = blk0; b < blk1; ++b) blk.push_back(b);
        int* db = (int*)c.lr_blocks.get(std::max<size_t>(1, blk.size()) * 4);
        RFX_CUDA(cudaMemcpyAsync(db, blk.data(), blk.size() * 4, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaStreamSynchronize(st));
        a.blocks = db;
        a.r0 = 0;
        a.r1 = c.lr_R;
        a.out_pos0 = blk0 * rfx::kTkRows;
        grid = blk1 - blk0;
    } else if (ordered) {
        // the 128-row blocks of the stored order that hold any requested row
        std::vector<int> blk;
        if (r0 == 0 && r1 == c.lr_R) {
            for (int b = 0; b < (c.lr_R + rfx::kTkRows - 1) / rfx::kTkRows; ++b) blk.push_back(b);
        } else {
            std::vector<char> mark((c.lr_R + rfx::kTkRows - 1) / rfx::kTkRows, 0);
            for (int i = r0; i < r1; ++i) mark[c.lr_pos[i] / rfx::kTkRows] = 1;
            for (int b = 0; b < (int)mark.size(); ++b)
                if (mark[b]) blk.push_back(b);
        }
        int* db = (int*)c.lr_blocks.get(blk.size() * 4);
        RFX_CUDA(cudaMemcpyAsync(db, blk.data(), blk.size() * 4, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaStreamSynchronize(st));  // blk is a local vector
        a.blocks = db;
        grid = (int)blk.size();
    }
    a.out_idx = oi;
    a.out_val = ov;
    a.dense = dense;
    a.dense_ld = ld;
    a.err = err;
    a.prof = nullptr;
    unsigned long long* prof = nullptr;
    static const bool want_prof = std::getenv("RFX_TOPK_PROF") != nullptr;
    if (want_prof) {
        prof = (unsigned long long*)c.lr_part.get(64 * 8);
        RFX_CUDA(cudaMemsetAsync(prof, 0, 128, st));
        a.prof = prof;
    }
    const int smem = rfx::tk_layout(k).bytes;
    set_smem((const void*)rfx::k_topk_tc, smem);
    if (c.profiling) RFX_CUDA(cudaEventRecord(c.ev0, st));
    rfx::k_topk_tc<<<grid, rfx::kTkThreads, smem, st>>>(tm, a);
    RFX_LAUNCH("k_topk_tc");
    if (c.profiling) RFX_CUDA(cudaEventRecord(c.ev1, st));
    c.launches += 1;
    int hv[2] = {0, 0};
    RFX_CUDA(cudaMemcpyAsync(hv, err, 8, cudaMemcpyDeviceToHost, st));
    RFX_CUDA(cudaStreamSynchronize(st));
    const int h = hv[0];
    c.topk_tiles += hv[1];
    if (c.profiling) {
        float ms = 0.0f;
        RFX_CUDA(cudaEventElapsedTime(&ms, c.ev0, c.ev1));
        c.topk_ms += ms;
    }
    require(h == 0, RFX_ERR_DEVICE, "product kernel: a pipeline wait timed out (code " + std::to_string(h) + ")");
    if (prof) {
        unsigned long long hp[16] = {};
        RFX_CUDA(cudaMemcpy(hp, prof, 128, cudaMemcpyDeviceToHost));
        std::fprintf(stderr,
                     "[rfx topk] rows=%d chunks=%llu scanned=%llu pushes=%llu finality-cycles=%llu "
                     "polls: readout=%llu mma=%llu load=%llu  cycles: readout wait=%llu "
                     "readout total=%llu mma wait-acc=%llu mma wait-load=%llu load wait-free=%llu tmem=%llu filter=%llu scan=%llu stage=%llu\n",
                     r1 - r0, hp[0], hp[1], hp[2], hp[3], hp[4], hp[5], hp[6], hp[7], hp[8], hp[9],
                     hp[10], hp[11], hp[12], hp[13], hp[14], hp[15]);
    }
}

// The product's stored order of the factors (rows by descending n_i = scale_i |q_i|,
// stable: ties by row id) from lr_q / lr_qb / lr_s of R rows.
void order_factors(Ctx& c, int R, int rank) {
    cudaStream_t st = c.st;
    const int Rpad = (int)round_up(R, rfx::kTkCols);
    const int8_t* q = (const int8_t*)c.lr_q.p;
    const uint16_t* qb = (const uint16_t*)c.lr_qb.p;
    const float* s = (const float*)c.lr_s.p;
    float* nrm = (float*)c.lr_norm.get((size_t)R * 4);
    int* ids = (int*)c.lr_ids.get((size_t)R * 4);
    float* keys = (float*)c.lr_keys.get((size_t)R * 4);
    int* order = (int*)c.lr_order_s.get((size_t)R * 4);
    rfx::k_lr_norms<<<(R + 255) / 256, 256, 0, st>>>(q, s, R, nrm, ids);
    RFX_LAUNCH("k_lr_norms");
    size_t tmp_bytes = 0;
    RFX_CUDA(cub::DeviceRadixSort::SortPairsDescending(nullptr, tmp_bytes, nrm, keys, ids, order,
                                                       R, 0, 32, st));
    void* tmp = c.lr_cub.get(tmp_bytes);
    RFX_CUDA(cub::DeviceRadixSort::SortPairsDescending(tmp, tmp_bytes, nrm, keys, ids, order, R, 0,
                                                       32, st));
    uint16_t* qbp = (uint16_t*)c.lr_qbp.get((size_t)Rpad * rfx::kLrK * 2);
    float* sp = (float*)c.lr_sp.get((size_t)Rpad * 4);
    float* np_ = (float*)c.lr_np.get((size_t)Rpad * 4);
    int* perm = (int*)c.lr_perm.get((size_t)Rpad * 4);
    rfx::k_lr_permute<<<grid_for((long long)Rpad * 8, 256, c.sm_count * 16), 256, 0, st>>>(
        qb, s, nrm, order, R, Rpad, qbp, sp, np_, perm);
    RFX_LAUNCH("k_lr_permute");
    std::vector<int> hp(R);
    RFX_CUDA(cudaMemcpyAsync(hp.data(), perm, (size_t)R * 4, cudaMemcpyDeviceToHost, st));
    c.launches += 2;
    RFX_CUDA(cudaStreamSynchronize(st));
    c.lr_pos.assign(R, 0);
    for (int p = 0; p < R; ++p) c.lr_pos[hp[p]] = p;
    c.lr_k = rank;
    c.lr_Rpad = Rpad;
    c.lr_R = R;
    c.lr_ready = true;
}

}  // namespace

void lr_reserve(Ctx& c, int extra) {
    if (c.lr_rank <= 0) return;
    const int need = c.lr_n + extra;
    if (need <= c.lr_cap) return;
    const size_t N = c.N, G = c.lr_G;
    DBuf code, order, goff, ng;
    code.get((size_t)need * N * 2);
    order.get((size_t)need * N * 4);
    goff.get((size_t)need * G * 4);
    ng.get((size_t)need * 4);
    if (c.lr_n > 0) {
        RFX_CUDA(cudaMemcpyAsync(code.p, c.lr_code.p, (size_t)c.lr_n * N * 2, cudaMemcpyDeviceToDevice, c.st));
        RFX_CUDA(cudaMemcpyAsync(order.p, c.lr_order.p, (size_t)c.lr_n * N * 4, cudaMemcpyDeviceToDevice, c.st));
        RFX_CUDA(cudaMemcpyAsync(goff.p, c.lr_goff.p, (size_t)c.lr_n * G * 4, cudaMemcpyDeviceToDevice, c.st));
        RFX_CUDA(cudaMemcpyAsync(ng.p, c.lr_ngroups.p, (size_t)c.lr_n * 4, cudaMemcpyDeviceToDevice, c.st));
    }
    RFX_CUDA(cudaStreamSynchronize(c.st));
    c.lr_code.release();
    c.lr_order.release();
    c.lr_goff.release();
    c.lr_ngroups.release();
    c.lr_code = code;
    c.lr_order = order;
    c.lr_goff = goff;
    c.lr_ngroups = ng;
    code.p = order.p = goff.p = ng.p = nullptr;
    c.lr_cap = need;
}

void lr_store_batch(Ctx& c, const rfx::Batch& B, int T) {
    lr_reserve(c, T);
    cudaStream_t st = c.st;
    const size_t N = c.N, G = c.lr_G, M = c.M;
    require(N < (1u << 24) && M <= 65535 && T <= 4096, RFX_ERR_UNSUPPORTED,
            "low-rank leaf groups need < 2^24 rows, maxnode < 65536, <= 4096 trees per batch");
    uint16_t* code = (uint16_t*)c.lr_code.p + (size_t)c.lr_n * N;
    int* order = (int*)c.lr_order.p + (size_t)c.lr_n * N;
    int* goff = (int*)c.lr_goff.p + (size_t)c.lr_n * G;
    int* ngroups = (int*)c.lr_ngroups.p + c.lr_n;
    int* tmp = (int*)c.lr_tmp.get((size_t)T * 2 * M * 4 + (size_t)(2 * T + 2) * 4);
    int* lidx = tmp;
    int* opre = tmp + (size_t)T * M;
    int* noob_r = tmp + (size_t)2 * T * M;
    int* nkeys_d = noob_r + T;
    int* obase_d = (int*)c.lr_ids.get((size_t)(T + 1) * 4);
    RFX_CUDA(cudaMemsetAsync(code, 0xFF, (size_t)T * N * 2, st));
    RFX_CUDA(cudaMemsetAsync(nkeys_d, 0, 4, st));
    rfx::k_lr_count<<<T, 1024, 0, st>>>(B, c.N, c.R, c.lr_G, goff, ngroups, lidx, opre, noob_r);
    RFX_LAUNCH("k_lr_count");
    rfx::k_lr_inbag<<<c.sm_count * 8, 256, 0, st>>>(B, c.N, c.R, c.lr_G, T, lidx, goff, code, order);
    RFX_LAUNCH("k_lr_inbag");
    unsigned long long* keys = (unsigned long long*)c.lr_keys.get((size_t)T * N * 8);
    unsigned long long* sorted = (unsigned long long*)c.lr_order_s.get((size_t)T * N * 8);
    rfx::k_lr_oob_keys<<<dim3((unsigned)((N + 255) / 256), (unsigned)T), 256, 0, st>>>(
        B, c.N, c.R, lidx, code, keys, nkeys_d);
    RFX_LAUNCH("k_lr_oob_keys");
    std::vector<int> hv(T + 1);
    RFX_CUDA(cudaMemcpyAsync(hv.data(), noob_r, (size_t)(T + 1) * 4, cudaMemcpyDeviceToHost, st));
    RFX_CUDA(cudaStreamSynchronize(st));
    const int nkeys = hv[T];
    std::vector<int> ob(T);
    for (int t = 0, a = 0; t < T; ++t) {
        ob[t] = a;
        a += hv[t];
    }
    RFX_CUDA(cudaMemcpyAsync(obase_d, ob.data(), (size_t)T * 4, cudaMemcpyHostToDevice, st));
    int end_bit = 41;
    while ((1 << (end_bit - 40)) < T) ++end_bit;
    size_t tmp_bytes = 0;
    RFX_CUDA(cub::DeviceRadixSort::SortKeys(nullptr, tmp_bytes, keys, sorted, nkeys, 0, end_bit, st));
    void* ctmp = c.lr_cub.get(tmp_bytes);
    RFX_CUDA(cub::DeviceRadixSort::SortKeys(ctmp, tmp_bytes, keys, sorted, nkeys, 0, end_bit, st));
    if (nkeys > 0) {
        rfx::k_lr_oob_place<<<(nkeys + 255) / 256, 256, 0, st>>>(sorted, nkeys, c.N, (int)M, c.lr_G,
                                                                 obase_d, opre, goff, order);
        RFX_LAUNCH("k_lr_oob_place");
    }
    RFX_CUDA(cudaStreamSynchronize(st));  // ob is a host vector
    c.launches += 4;
    c.lr_n += T;
    c.lr_ready = false;
}

}  // namespace rfxh

using namespace rfxh;

extern "C" {

int rfx_prox_apply(void* ctx, const float* X_dev, int ncols, const int* nout_dev, float* Y_dev) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.lr_rank > 0, RFX_ERR_STATE, "low-rank mode is not active");
        require(X_dev && Y_dev && ncols >= 1 && ncols <= 128, RFX_ERR_ARG, "bad arguments");
        apply_s(c, X_dev, ncols, nout_dev ? nout_dev : (const int*)c.nout.p, Y_dev, nullptr, nullptr);
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_lowrank_build(void* ctx, int rank, int oversample, int power_iters, uint64_t seed,
                      const int* nout_dev, rfx_reduce_fn reduce, void* reduce_user) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.loaded && c.lr_rank > 0, RFX_ERR_STATE, "low-rank mode is not active");
        require(rank >= 1 && rank <= rfx::kLrK, RFX_ERR_ARG, "rank must be in [1, 64]");
        require(oversample >= 0 && power_iters >= 0 && power_iters <= 8, RFX_ERR_ARG, "bad sketch parameters");
        int r = rank + oversample;
        r += r & 1;  // the Jacobi pairing needs an even size
        require(r <= rfx::kLrMaxR, RFX_ERR_ARG, "rank + oversample must be <= 96");
        cudaStream_t st = c.st;
        const int R = c.R;
        const int* nout = nout_dev ? nout_dev : (const int*)c.nout.p;
        float* X = (float*)c.lr_X.get((size_t)R * r * 4);
        float* Y = (float*)c.lr_Y.get((size_t)R * r * 4);
        float* Q = (float*)c.lr_A.get((size_t)R * r * 4);
        double* sm = (double*)c.lr_small.get((size_t)(3 * r * r + r * rfx::kLrK + r) * 8);
        double* G = sm;
        double* Uinv = sm + r * r;
        double* T = sm + 2 * r * r;
        double* Mk = sm + 3 * r * r;
        double* lam = Mk + r * rfx::kLrK;
        rfx::k_lr_omega<<<grid_for((long long)R * r, 256, c.sm_count * 16), 256, 0, st>>>(X, R, r, seed);
        RFX_LAUNCH("k_lr_omega");
        apply_s(c, X, r, nout, Y, reduce, reduce_user);
        for (int i = 0; i < power_iters; ++i) {
            orth(c, Y, r, Q, G, Uinv);
            apply_s(c, Q, r, nout, Y, reduce, reduce_user);
        }
        orth(c, Y, r, Q, G, Uinv);
        apply_s(c, Q, r, nout, Y, reduce, reduce_user);  // Y = S Q
        gram(c, Q, r, Y, r, 1, T);                        // T = Q^T S Q
        const size_t eig_smem = (size_t)2 * r * r * 8 + (size_t)r * 8 + (size_t)2 * r * 4;
        set_smem((const void*)rfx::k_lr_eig_select, eig_smem);
        rfx::k_lr_eig_select<<<1, 256, eig_smem, st>>>(T, r, rank, Mk, lam);
        RFX_LAUNCH("k_lr_eig_select");
        set_smem((const void*)rfx::k_lr_rowmat, (size_t)r * rank * 8);
        float* A = X;  // R x rank
        rfx::k_lr_rowmat<<<c.sm_count * 4, 256, (size_t)r * rank * 8, st>>>(Q, R, r, Mk, rank, A);
        RFX_LAUNCH("k_lr_rowmat");
        const int Rpad = (int)round_up(R, rfx::kTkCols);
        int8_t* q = (int8_t*)c.lr_q.get((size_t)Rpad * rfx::kLrK);
        uint16_t* qb = (uint16_t*)c.lr_qb.get((size_t)Rpad * rfx::kLrK * 2);
        float* s = (float*)c.lr_s.get((size_t)Rpad * 4);
        rfx::k_lr_quantize<<<c.sm_count * 8, 256, 0, st>>>(A, R, rank, Rpad, q, qb, s);
        RFX_LAUNCH("k_lr_quantize");
        c.launches += 4;
        order_factors(c, R, rank);
    });
}

int rfx_lowrank_set_factors(void* ctx, const int8_t* q_host, const float* scale_host, int rows,
                            int rank) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(q_host && scale_host, RFX_ERR_ARG, "null factors");
        require(rows >= 1 && rank >= 1 && rank <= rfx::kLrK, RFX_ERR_ARG, "bad factor shape");
        for (size_t i = 0; i < (size_t)rows * rank; ++i)
            require(q_host[i] >= -127, RFX_ERR_ARG, "factor values must be in [-127, 127]");
        for (int i = 0; i < rows; ++i)
            require(scale_host[i] >= 0.0f && std::isfinite(scale_host[i]), RFX_ERR_ARG,
                    "scales must be finite and non-negative");
        cudaStream_t st = c.st;
        const int Rpad = (int)round_up(rows, rfx::kTkCols);
        int8_t* qin = (int8_t*)c.lr_X.get((size_t)rows * rank);
        float* sin = (float*)c.lr_Y.get((size_t)rows * 4);
        RFX_CUDA(cudaMemcpyAsync(qin, q_host, (size_t)rows * rank, cudaMemcpyHostToDevice, st));
        RFX_CUDA(cudaMemcpyAsync(sin, scale_host, (size_t)rows * 4, cudaMemcpyHostToDevice, st));
        int8_t* q = (int8_t*)c.lr_q.get((size_t)Rpad * rfx::kLrK);
        uint16_t* qb = (uint16_t*)c.lr_qb.get((size_t)Rpad * rfx::kLrK * 2);
        float* s = (float*)c.lr_s.get((size_t)Rpad * 4);
        rfx::k_lr_load_factors<<<grid_for((long long)Rpad * rfx::kLrK, 256, c.sm_count * 16), 256, 0, st>>>(
            qin, sin, rows, rank, Rpad, q, qb, s);
        RFX_LAUNCH("k_lr_load_factors");
        c.launches += 1;
        order_factors(c, rows, rank);
    });
}

int rfx_lowrank_factors(void* ctx, float* A_host, int8_t* q_host, float* scale_host,
                        int* rank_out, int* rows_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.lr_ready, RFX_ERR_STATE, "low-rank factors have not been built");
        const int R = c.lr_R, k = c.lr_k;
        std::vector<int8_t> qh((size_t)R * rfx::kLrK);
        std::vector<float> sh(R);
        RFX_CUDA(cudaMemcpyAsync(qh.data(), c.lr_q.p, qh.size(), cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaMemcpyAsync(sh.data(), c.lr_s.p, (size_t)R * 4, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
        for (int i = 0; i < R; ++i) {
            for (int j = 0; j < k; ++j) {
                const int8_t v = qh[(size_t)i * rfx::kLrK + j];
                if (q_host) q_host[(size_t)i * k + j] = v;
                if (A_host) A_host[(size_t)i * k + j] = sh[i] * (float)v;
            }
            if (scale_host) scale_host[i] = sh[i];
        }
        if (rank_out) *rank_out = k;
        if (rows_out) *rows_out = R;
    });
}

int rfx_lowrank_topk(void* ctx, int k, int row_begin, int row_end, int* idx_host, float* val_host) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.lr_ready, RFX_ERR_STATE, "low-rank factors have not been built");
        require(k >= 1 && k <= 64, RFX_ERR_ARG, "k must be in [1, 64]");
        require(row_begin >= 0 && row_begin <= row_end && row_end <= c.lr_R, RFX_ERR_ARG, "bad row range");
        require(idx_host && val_host, RFX_ERR_ARG, "null output");
        const int rows = row_end - row_begin;
        if (rows == 0) return;
        int* oi = (int*)c.lr_out_i.get((size_t)rows * k * 4);
        float* ov = (float*)c.lr_out_v.get((size_t)rows * k * 4);
        run_product(c, row_begin, row_end, k, oi, ov, nullptr, 0);
        RFX_CUDA(cudaMemcpyAsync(idx_host, oi, (size_t)rows * k * 4, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaMemcpyAsync(val_host, ov, (size_t)rows * k * 4, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_lowrank_topk_part(void* ctx, int k, int part, int nparts, int* rows_host, int* idx_host,
                          float* val_host, int* nrows_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.lr_ready, RFX_ERR_STATE, "low-rank factors have not been built");
        require(k >= 1 && k <= 64, RFX_ERR_ARG, "k must be in [1, 64]");
        require(nparts >= 1 && part >= 0 && part < nparts && nrows_out, RFX_ERR_ARG, "bad part");
        const int nblk = (c.lr_R + rfx::kTkRows - 1) / rfx::kTkRows;
        const int b0 = (int)((long long)nblk * part / nparts), b1 = (int)((long long)nblk * (part + 1) / nparts);
        const int p0 = b0 * rfx::kTkRows, p1 = std::min(c.lr_R, b1 * rfx::kTkRows);
        const int rows = std::max(0, p1 - p0);
        *nrows_out = rows;
        if (!rows_host || rows == 0) return;
        require(idx_host && val_host, RFX_ERR_ARG, "null output");
        int* oi = (int*)c.lr_out_i.get((size_t)(b1 - b0) * rfx::kTkRows * k * 4);
        float* ov = (float*)c.lr_out_v.get((size_t)(b1 - b0) * rfx::kTkRows * k * 4);
        run_product(c, 0, c.lr_R, k, oi, ov, nullptr, 0, b0, b1);
        RFX_CUDA(cudaMemcpyAsync(idx_host, oi, (size_t)rows * k * 4, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaMemcpyAsync(val_host, ov, (size_t)rows * k * 4, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaMemcpyAsync(rows_host, (const int*)c.lr_perm.p + p0, (size_t)rows * 4,
                                 cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_lowrank_product(void* ctx, int row_begin, int row_end, float* out_host) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.lr_ready, RFX_ERR_STATE, "low-rank factors have not been built");
        require(row_begin >= 0 && row_begin <= row_end && row_end <= c.lr_R, RFX_ERR_ARG, "bad row range");
        require(out_host, RFX_ERR_ARG, "null output");
        const int R = c.lr_R;
        const long long ld = c.lr_Rpad;
        const int chunk = (int)std::max<long long>(rfx::kTkRows,
            (((long long)256 << 20) / (ld * 4)) / rfx::kTkRows * rfx::kTkRows);
        float* buf = (float*)c.lr_out_v.get((size_t)std::min(chunk, row_end - row_begin + rfx::kTkRows) * ld * 4);
        for (int r0 = row_begin; r0 < row_end; r0 += chunk) {
            const int r1 = std::min(row_end, r0 + chunk);
            run_product(c, r0, r1, 0, nullptr, nullptr, buf, ld);
            RFX_CUDA(cudaMemcpy2DAsync(out_host + (size_t)(r0 - row_begin) * R, (size_t)R * 4, buf,
                                       (size_t)ld * 4, (size_t)R * 4, (size_t)(r1 - r0),
                                       cudaMemcpyDeviceToHost, c.st));
            RFX_CUDA(cudaStreamSynchronize(c.st));
        }
    });
}

}  // extern "C"
