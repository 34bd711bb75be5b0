// Low-rank proximity: per-tree leaf groups, the proximity operator applied through leaf
// sums, and the small dense linear algebra of the randomized range finder.
//
// The reference keeps a low-rank factorisation of the proximity matrix updated tree by tree
// (LowRankProximityMatrix, include/rf_proximity_lowrank.hpp:27-439: a rank-1 power
// iteration per tree over an fp16 packed triangle, cuda/rf_proximity_lowrank.cu:414-1340),
// which needs the n x n tree proximity.  Here the counts are never formed.  A tree's
// contribution to the symmetric count matrix C (reference dense branch,
// src/rf_proximity.cpp:99-230: OOB row i and in-bag row j in one leaf add 1 to P[i][j]) is
//     C_t = sum over leaves l of  o_l b_l^T + b_l o_l^T
// with o_l / b_l the indicator vectors of the leaf's OOB / distinct in-bag rows, so
//     (C_t Z)_i = sum_{j in-bag in leaf(i)} Z_j   for an OOB row i, and vice versa.
// One pass over the stored trees therefore applies C to an R x W block Z with two
// gathers per row and tree: leaf sums of Z over each (leaf, in-bag|OOB) group, then every
// row picks up the sum of the opposite group of its leaf.  The finishprox'd matrix is
//     S = (D C + C D) / 4 + I,   D = diag(1/nout)  (1 where nout = 0),
// the matrix rfx_prox_finish produces entry by entry (src/rf_finishprox.cpp:12-74).
//
// All sums run in a fixed order (group order, then tree order), so the results are
// reproducible bit for bit.
#include <cuda_runtime.h>
#include <cstdint>

#include "rfx_device.cuh"
#include "rfx_lowrank.h"

namespace rfx {

namespace {

// Exclusive scan of n ints in place by one block (blockDim.x a multiple of 32, <= 1024);
// returns the total.  `warp_tot` is 32 ints of shared memory.
__device__ int block_scan_inplace(int* a, int n, int* warp_tot) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
    int carry = 0;
    for (int base = 0; base < n; base += blockDim.x) {
        const int i = base + tid;
        const int v = i < n ? a[i] : 0;
        int x = v;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[wid] = x;
        __syncthreads();
        if (wid == 0) {
            int w = lane < nw ? warp_tot[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            if (lane < nw) warp_tot[lane] = w;  // inclusive prefix over warps
        }
        __syncthreads();
        const int before = (wid > 0 ? warp_tot[wid - 1] : 0) + carry;
        if (i < n) a[i] = before + x - v;
        const int tot = warp_tot[nw - 1];
        __syncthreads();
        carry += tot;
    }
    return carry;
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    // splitmix64 finaliser (Steele, Lea, Flood 2014)
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float inv_nout(const int* nout, int i) {
    const int n = nout[i];
    return n > 0 ? 1.0f / (float)n : 1.0f;
}

}  // namespace

// ---------------------------------------------------------------------------------------
// Leaf groups of one batch of trees.  For tree t:
//   code[t][row]  = 2*l (in-bag) or 2*l+1 (OOB) for rows < R, l the leaf's rank among the
//                   tree's terminal nodes in node order; kNoGroup for rows >= R;
//   order[t][...] = rows grouped by code: group g occupies [goff[t][g], goff[t][g+1]);
//                   in-bag rows in their growth-segment order (ascending), OOB rows ascending;
//   ngroups[t]    = 2 * leaves.
// Built by k_lr_count (block per tree: leaf ranks, group sizes, offsets), k_lr_inbag (warp
// per terminal node: the segment's rows), k_lr_oob_keys + a radix sort of the batch's
// (tree, leaf, row) keys + k_lr_oob_place (the OOB rows, ascending inside each group).
// lidx / oprefix: [T][M] ints (leaf rank of every node; exclusive prefix of the OOB group
// sizes over leaves); noob_r[t]: the tree's OOB rows below R.
// ---------------------------------------------------------------------------------------
__global__ void k_lr_count(Batch B, int N, int R, int G, int* __restrict__ goff,
                           int* __restrict__ ngroups, int* __restrict__ lidx_all,
                           int* __restrict__ oprefix_all, int* __restrict__ noob_r) {
    __shared__ int wtot[32];
    const int t = blockIdx.x, M = B.M;
    const int nn = B.nnode[t];
    const int* status = B.status + (size_t)t * M;
    int* lidx = lidx_all + (size_t)t * M;
    int* opre = oprefix_all + (size_t)t * M;
    int* gt = goff + (size_t)t * G;
    for (int m = threadIdx.x; m < nn; m += blockDim.x) lidx[m] = status[m] == -1 ? 1 : 0;
    __syncthreads();
    const int L = block_scan_inplace(lidx, nn, wtot);  // lidx[m] = leaf rank of leaf m
    for (int g = threadIdx.x; g <= 2 * L; g += blockDim.x) gt[g] = 0;
    for (int l = threadIdx.x; l < L; l += blockDim.x) opre[l] = 0;
    __syncthreads();
    for (int m = threadIdx.x; m < nn; m += blockDim.x) {
        if (status[m] != -1) continue;
        const size_t nm = (size_t)t * M + m;
        const int c = B.nd_cnt[nm];
        int k = c;
        if (R < N) {
            const int* seg = B.seg[B.nd_buf[nm]] + (size_t)t * N + B.nd_start[nm];
            k = 0;
            for (int q = 0; q < c; ++q) k += seg[q] < R ? 1 : 0;
        }
        gt[2 * lidx[m]] = k;
    }
    const int noob = B.noob[t];
    const int* oob = B.oob + (size_t)t * N;
    const int* oleaf = B.oob_leaf + (size_t)t * N;
    __syncthreads();
    for (int i = threadIdx.x; i < noob; i += blockDim.x) {
        const int row = oob[i];
        if (row < R) {
            const int l = lidx[oleaf[row]];
            atomicAdd(&gt[2 * l + 1], 1);
            atomicAdd(&opre[l], 1);
        }
    }
    __syncthreads();
    const int tot_oob = block_scan_inplace(opre, L, wtot);
    block_scan_inplace(gt, 2 * L + 1, wtot);  // gt[g] = start of group g, gt[2L] = total
    if (threadIdx.x == 0) {
        ngroups[t] = 2 * L;
        noob_r[t] = tot_oob;
    }
}

// In-bag rows (< R) of every terminal node into its group, segment order kept (grid-stride
// warps over (tree, node)).
__global__ void k_lr_inbag(Batch B, int N, int R, int G, int T, const int* __restrict__ lidx_all,
                           const int* __restrict__ goff, uint16_t* __restrict__ code,
                           int* __restrict__ order) {
    const int M = B.M;
    const int lane = threadIdx.x & 31;
    const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    for (int t = 0; t < T; ++t)
    for (long long mm = wid, nn = B.nnode[t]; mm < nn; mm += nwarps) {
        const int m = (int)mm;
        const size_t nm = (size_t)t * M + m;
        if (B.status[nm] != -1) continue;
        const int l = lidx_all[nm];
        const int* seg = B.seg[B.nd_buf[nm]] + (size_t)t * N + B.nd_start[nm];
        const int c = B.nd_cnt[nm];
        int pos = goff[(size_t)t * G + 2 * l];
        int* ot = order + (size_t)t * N;
        uint16_t* ct = code + (size_t)t * N;
        for (int q0 = 0; q0 < c; q0 += 32) {
            const int q = q0 + lane;
            const int row = q < c ? seg[q] : R;
            const bool keep = row < R;
            const unsigned bal = __ballot_sync(0xffffffffu, keep);
            if (keep) {
                ot[pos + __popc(bal & ((1u << lane) - 1u))] = row;
                ct[row] = (uint16_t)(2 * l);
            }
            pos += __popc(bal);
        }
    }
}

// One key (tree << 40 | leaf rank << 24 | row) per OOB row below R; nkeys counts them.
__global__ void k_lr_oob_keys(Batch B, int N, int R, const int* __restrict__ lidx_all,
                              uint16_t* __restrict__ code, unsigned long long* __restrict__ keys,
                              int* __restrict__ nkeys) {
    const int t = blockIdx.y, M = B.M;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    bool have = false;
    unsigned long long key = 0;
    if (i < B.noob[t]) {
        const int row = B.oob[(size_t)t * N + i];
        if (row < R) {
            const int l = lidx_all[(size_t)t * M + B.oob_leaf[(size_t)t * N + row]];
            code[(size_t)t * N + row] = (uint16_t)(2 * l + 1);
            key = ((unsigned long long)t << 40) | ((unsigned long long)l << 24) | (unsigned long long)row;
            have = true;
        }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, have);
    int base = 0;
    if (lane == 0 && bal) base = atomicAdd(nkeys, __popc(bal));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (have) keys[base + __popc(bal & ((1u << lane) - 1u))] = key;
}

// Sorted keys -> OOB group slots: key i of tree t, leaf l sits at goff[t][2l+1] + its rank
// among the tree's leaf-l keys (i - obase[t] - oprefix[t][l]).
__global__ void k_lr_oob_place(const unsigned long long* __restrict__ keys, int nkeys, int N, int M,
                               int G, const int* __restrict__ obase,
                               const int* __restrict__ oprefix_all, const int* __restrict__ goff,
                               int* __restrict__ order) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nkeys) return;
    const unsigned long long key = keys[i];
    const int t = (int)(key >> 40), l = (int)((key >> 24) & 0xFFFFu), row = (int)(key & 0xFFFFFFu);
    const int rank = i - obase[t] - oprefix_all[(size_t)t * M + l];
    order[(size_t)t * N + goff[(size_t)t * G + 2 * l + 1] + rank] = row;
}

// ---------------------------------------------------------------------------------------
// Applying C.  LS[t][g][:] = sum of Z over group g of tree t (warp per group, lanes over
// columns, rows in group order).  Z is [R][W], W = 32 * NQ.
// ---------------------------------------------------------------------------------------
template <int NQ>
__global__ void k_lr_leafsum(const int* __restrict__ order, const int* __restrict__ goff,
                             const int* __restrict__ ngroups, int N, int G, int T,
                             const float* __restrict__ Z, float* __restrict__ LS) {
    (void)T;
    const int t = blockIdx.y;
    const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (g >= ngroups[t]) return;
    const int* gt = goff + (size_t)t * G;
    const int* ot = order + (size_t)t * N;
    const int a = gt[g], b = gt[g + 1];
    constexpr int W = 32 * NQ;
    float acc[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc[q] = 0.0f;
    int k = a;
    for (; k + 4 <= b; k += 4) {  // four rows in flight, added in group order
        const float* z0 = Z + (size_t)ot[k] * W + lane;
        const float* z1 = Z + (size_t)ot[k + 1] * W + lane;
        const float* z2 = Z + (size_t)ot[k + 2] * W + lane;
        const float* z3 = Z + (size_t)ot[k + 3] * W + lane;
        float v[4][NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            v[0][q] = __ldg(z0 + 32 * q);
            v[1][q] = __ldg(z1 + 32 * q);
            v[2][q] = __ldg(z2 + 32 * q);
            v[3][q] = __ldg(z3 + 32 * q);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int q = 0; q < NQ; ++q) acc[q] += v[u][q];
    }
    for (; k < b; ++k) {
        const float* z = Z + (size_t)ot[k] * W + lane;
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[q] += __ldg(z + 32 * q);
    }
    float* o = LS + ((size_t)t * G + g) * W + lane;
#pragma unroll
    for (int q = 0; q < NQ; ++q) o[32 * q] = acc[q];
}

// Y[row] += sum over the chunk's trees, in tree order, of the leaf sum of the row's
// opposite group (warp per row).
template <int NQ>
__global__ void k_lr_scatter(const uint16_t* __restrict__ code, int N, int R, int T, int G,
                             const float* __restrict__ LS, float* __restrict__ Y) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= R) return;
    constexpr int W = 32 * NQ;
    float acc[NQ];
    float* y = Y + (size_t)row * W + lane;
#pragma unroll
    for (int q = 0; q < NQ; ++q) acc[q] = y[32 * q];
    for (int t = 0; t < T; ++t) {
        const int cd = code[(size_t)t * N + row];
        if (cd == kNoGroup) continue;
        const float* s = LS + ((size_t)t * G + (cd ^ 1)) * W + lane;
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[q] += __ldg(s + 32 * q);
    }
#pragma unroll
    for (int q = 0; q < NQ; ++q) y[32 * q] = acc[q];
}


bool lr_launch_leafsum(int nq, dim3 grid, cudaStream_t st, const int* order, const int* goff,
                       const int* ngroups, int N, int G, int T, const float* Z, float* LS) {
    switch (nq) {
#define RFX_LS(Q) case Q: k_lr_leafsum<Q><<<grid, 256, 0, st>>>(order, goff, ngroups, N, G, T, Z, LS); return true;
        RFX_LS(1) RFX_LS(2) RFX_LS(3) RFX_LS(4) RFX_LS(5) RFX_LS(6) RFX_LS(7) RFX_LS(8)
#undef RFX_LS
        default: return false;
    }
}

bool lr_launch_scatter(int nq, int grid, cudaStream_t st, const uint16_t* code, int N, int R, int T,
                       int G, const float* LS, float* Y) {
    switch (nq) {
#define RFX_SC(Q) case Q: k_lr_scatter<Q><<<grid, 256, 0, st>>>(code, N, R, T, G, LS, Y); return true;
        RFX_SC(1) RFX_SC(2) RFX_SC(3) RFX_SC(4) RFX_SC(5) RFX_SC(6) RFX_SC(7) RFX_SC(8)
#undef RFX_SC
        default: return false;
    }
}

// Z = [X | D X | 0] ([R][W]) from X ([R][r]).
__global__ void k_lr_prep(const float* __restrict__ X, int R, int r, const int* __restrict__ nout,
                          int W, float* __restrict__ Z) {
    const long long total = (long long)R * W;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(k / W), c = (int)(k % W);
        float v = 0.0f;
        if (c < r) v = X[(size_t)i * r + c];
        else if (c < 2 * r) v = inv_nout(nout, i) * X[(size_t)i * r + (c - r)];
        Z[k] = v;
    }
}

// Y = S X = (D (C X) + C (D X)) / 4 + X from CZ = C [X | D X].
__global__ void k_lr_combine(const float* __restrict__ CZ, int W, const float* __restrict__ X,
                             int R, int r, const int* __restrict__ nout, float* __restrict__ Y) {
    const long long total = (long long)R * r;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(k / r), c = (int)(k % r);
        const float* cz = CZ + (size_t)i * W;
        const float a = inv_nout(nout, i) * cz[c];
        Y[k] = 0.25f * (a + cz[r + c]) + X[k];
    }
}

// Random +-1 test matrix [R][r].
__global__ void k_lr_omega(float* __restrict__ X, int R, int r, unsigned long long seed) {
    const long long total = (long long)R * r;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x)
        X[k] = (mix64(seed * 0x100000001B3ull + (uint64_t)k) >> 63) ? 1.0f : -1.0f;
}

// ---------------------------------------------------------------------------------------
// Small dense linear algebra (r <= kLrMaxR), fp64.
// ---------------------------------------------------------------------------------------

// part[b][a][c] = sum over block b's rows of A[i][a] * B[i][c] (A [R][ra], B [R][rb]).
__global__ void k_lr_gram(const float* __restrict__ A, int ra, const float* __restrict__ Bm,
                          int rb, int R, int rows_per_block, double* __restrict__ part) {
    __shared__ float sa[32][kLrMaxR];
    __shared__ float sb[32][kLrMaxR];
    constexpr int kPer = (kLrMaxR * kLrMaxR + 255) / 256;
    double acc[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) acc[e] = 0.0;
    const int r0 = blockIdx.x * rows_per_block;
    const int r1 = min(R, r0 + rows_per_block);
    const int nent = ra * rb;
    for (int base = r0; base < r1; base += 32) {
        const int nr = min(32, r1 - base);
        for (int k = threadIdx.x; k < 32 * kLrMaxR; k += blockDim.x) {
            const int i = k / kLrMaxR, c = k % kLrMaxR;
            sa[i][c] = (i < nr && c < ra) ? A[(size_t)(base + i) * ra + c] : 0.0f;
            sb[i][c] = (i < nr && c < rb) ? Bm[(size_t)(base + i) * rb + c] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            const int idx = threadIdx.x + 256 * e;
            if (idx < nent) {
                const int a = idx / rb, c = idx % rb;
                double s = acc[e];
                for (int i = 0; i < nr; ++i) s += (double)sa[i][a] * (double)sb[i][c];
                acc[e] = s;
            }
        }
        __syncthreads();
    }
    double* o = part + (size_t)blockIdx.x * nent;
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
        const int idx = threadIdx.x + 256 * e;
        if (idx < nent) o[idx] = acc[e];
    }
}

// G = sum of the partials in block order (thread per entry).
__global__ void k_lr_gram_reduce(const double* __restrict__ part, int nblk, int ra, int rb,
                                 int sym, double* __restrict__ G) {
    (void)sym;
    const int nent = ra * rb;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < nent; idx += gridDim.x * blockDim.x) {
        double s = 0.0;
        for (int b = 0; b < nblk; ++b) s += part[(size_t)b * nent + idx];
        G[idx] = s;
    }
}

// G <- (G + G^T) / 2 (one block).
__global__ void k_lr_symmetrize(double* __restrict__ G, int r) {
    for (int idx = threadIdx.x; idx < r * r; idx += blockDim.x) {
        const int a = idx / r, c = idx % r;
        if (a < c) {
            const double m = 0.5 * (G[a * r + c] + G[c * r + a]);
            G[a * r + c] = m;
            G[c * r + a] = m;
        }
    }
}

// Cholesky G = U^T U (U upper) and Uinv = U^{-1}, one block, fp64 in shared memory.  A
// pivot below tol * max diag marks a dependent column: U_jj = 1 and the rest of row j 0,
// which maps that column of Y to its (near-zero) residual.
__global__ void k_lr_chol_inv(const double* __restrict__ Gm, int r, double* __restrict__ Uinv) {
    extern __shared__ double sm[];
    double* U = sm;           // [r][r]
    double* Gs = sm + r * r;  // [r][r]
    __shared__ double piv, dmax;
    for (int k = threadIdx.x; k < r * r; k += blockDim.x) {
        Gs[k] = Gm[k];
        U[k] = 0.0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double m = 0.0;
        for (int j = 0; j < r; ++j) m = fmax(m, Gs[j * r + j]);
        dmax = m;
    }
    __syncthreads();
    const double tol = 1e-13 * dmax;
    for (int j = 0; j < r; ++j) {
        if (threadIdx.x == 0) {
            double s = Gs[j * r + j];
            for (int k = 0; k < j; ++k) s -= U[k * r + j] * U[k * r + j];
            piv = s > tol && s > 0.0 ? sqrt(s) : 0.0;
            U[j * r + j] = piv > 0.0 ? piv : 1.0;
        }
        __syncthreads();
        for (int i = j + 1 + threadIdx.x; i < r; i += blockDim.x) {
            if (piv > 0.0) {
                double s = Gs[j * r + i];
                for (int k = 0; k < j; ++k) s -= U[k * r + j] * U[k * r + i];
                U[j * r + i] = s / piv;
            } else {
                U[j * r + i] = 0.0;
            }
        }
        __syncthreads();
    }
    // inverse of the upper-triangular U, column by column (thread per column)
    for (int j = threadIdx.x; j < r; j += blockDim.x) {
        for (int i = r - 1; i >= 0; --i) {
            double v;
            if (i > j) {
                v = 0.0;
            } else {
                double s = i == j ? 1.0 : 0.0;
                for (int k = i + 1; k <= j; ++k) s -= U[i * r + k] * Uinv[k * r + j];
                v = s / U[i * r + i];
            }
            Uinv[i * r + j] = v;
        }
    }
}

// Out[i][:] = Y[i][:] * Mat (Y [R][rin] fp32, Mat [rin][rout] fp64, Out [R][rout] fp32);
// warp per row, fp64 accumulation.
__global__ void k_lr_rowmat(const float* __restrict__ Y, int R, int rin,
                            const double* __restrict__ Mat, int rout, float* __restrict__ Out) {
    extern __shared__ double smat[];
    for (int k = threadIdx.x; k < rin * rout; k += blockDim.x) smat[k] = Mat[k];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    constexpr int NQ = kLrMaxR / 32;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < R;
         row += gridDim.x * (blockDim.x >> 5)) {
        float y[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int c = lane + 32 * q;
            y[q] = c < rin ? Y[(size_t)row * rin + c] : 0.0f;
        }
        double acc[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[q] = 0.0;
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) {
            for (int ii = 0; ii < 32; ++ii) {
                const int i = 32 * qi + ii;
                const double yi = (double)__shfl_sync(0xffffffffu, y[qi], ii);
                if (i >= rin) break;
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    const int c = lane + 32 * q;
                    if (c < rout) acc[q] += yi * smat[i * rout + c];
                }
            }
        }
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int c = lane + 32 * q;
            if (c < rout) Out[(size_t)row * rout + c] = (float)acc[q];
        }
    }
}

// Symmetric eigendecomposition T = V diag(lam) V^T by parallel cyclic Jacobi (one block,
// round-robin pairing, rotations of Golub & Van Loan, Matrix Computations, sec. 8.5), then
// Mk[:, c] = V[:, idx_c] * sqrt(max(lam_c, 0)) for the k largest eigenvalues (descending).
// r must be even.  lam_out gets the sorted eigenvalues (all r).
__global__ void k_lr_eig_select(const double* __restrict__ Tm, int r, int k, double* __restrict__ Mk,
                                double* __restrict__ lam_out) {
    extern __shared__ double sm[];
    double* A = sm;                 // [r][r]
    double* V = A + r * r;          // [r][r]
    double* cs = V + r * r;         // [r/2][2] rotation (c, s)
    int* pp = (int*)(cs + r);       // [r/2] pair p
    int* pq = pp + r / 2;           // [r/2] pair q
    int* ord = pq + r / 2;          // [r]
    __shared__ double off_s, tot_s;
    for (int e = threadIdx.x; e < r * r; e += blockDim.x) {
        A[e] = Tm[e];
        V[e] = (e / r == e % r) ? 1.0 : 0.0;
    }
    __syncthreads();
    const int h = r / 2;
    for (int sweep = 0; sweep < 60; ++sweep) {
        if (threadIdx.x == 0) {
            double off = 0.0, tot = 0.0;
            for (int e = 0; e < r * r; ++e) {
                const double v = A[e] * A[e];
                tot += v;
                if (e / r != e % r) off += v;
            }
            off_s = off;
            tot_s = tot;
        }
        __syncthreads();
        if (!(off_s > 1e-30 * tot_s)) break;
        for (int round = 0; round < r - 1; ++round) {
            // circle method: position 0 holds player 0, position j >= 1 holds
            // 1 + (j - 1 + round) mod (r - 1); pair positions j and r - 1 - j
            for (int j = threadIdx.x; j < h; j += blockDim.x) {
                const int a = j == 0 ? 0 : 1 + (j - 1 + round) % (r - 1);
                const int b = 1 + (r - 2 - j + round) % (r - 1);
                const int p = min(a, b), q = max(a, b);
                const double apq = A[p * r + q];
                double c = 1.0, s = 0.0;
                if (apq != 0.0) {
                    const double tau = (A[q * r + q] - A[p * r + p]) / (2.0 * apq);
                    const double t = (tau >= 0.0 ? 1.0 : -1.0) / (fabs(tau) + sqrt(1.0 + tau * tau));
                    c = 1.0 / sqrt(1.0 + t * t);
                    s = t * c;
                }
                pp[j] = p;
                pq[j] = q;
                cs[2 * j] = c;
                cs[2 * j + 1] = s;
            }
            __syncthreads();
            // rows p, q of A <- J^T A
            for (int e = threadIdx.x; e < h * r; e += blockDim.x) {
                const int j = e / r, col = e % r;
                const int p = pp[j], q = pq[j];
                const double c = cs[2 * j], s = cs[2 * j + 1];
                const double ap = A[p * r + col], aq = A[q * r + col];
                A[p * r + col] = c * ap - s * aq;
                A[q * r + col] = s * ap + c * aq;
            }
            __syncthreads();
            // columns p, q of A and V <- A J, V J
            for (int e = threadIdx.x; e < h * r; e += blockDim.x) {
                const int j = e / r, row = e % r;
                const int p = pp[j], q = pq[j];
                const double c = cs[2 * j], s = cs[2 * j + 1];
                const double ap = A[row * r + p], aq = A[row * r + q];
                A[row * r + p] = c * ap - s * aq;
                A[row * r + q] = s * ap + c * aq;
                const double vp = V[row * r + p], vq = V[row * r + q];
                V[row * r + p] = c * vp - s * vq;
                V[row * r + q] = s * vp + c * vq;
            }
            __syncthreads();
        }
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < r; ++i) ord[i] = i;
        for (int i = 1; i < r; ++i) {  // insertion sort, eigenvalue descending, index ascending
            const int v = ord[i];
            int j = i - 1;
            while (j >= 0 && A[ord[j] * r + ord[j]] < A[v * r + v]) {
                ord[j + 1] = ord[j];
                --j;
            }
            ord[j + 1] = v;
        }
        for (int i = 0; i < r; ++i) lam_out[i] = A[ord[i] * r + ord[i]];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < r * k; e += blockDim.x) {
        const int i = e / k, c = e % k;
        const int src = ord[c];
        const double lam = A[src * r + src];
        Mk[e] = V[i * r + src] * (lam > 0.0 ? sqrt(lam) : 0.0);
    }
}

// Per-row symmetric int8 quantisation of A [R][k] (warp per row):
//   scale_i = max_c |A_ic| / 127,  q_ic = round-half-even(A_ic / scale_i)  (0 when scale 0);
// writes q [Rpad][kLrK] int8 and qb [Rpad][kLrK] bf16 (the same integers, exact), zero
// padded, and scale [Rpad].
__global__ void k_lr_quantize(const float* __restrict__ A, int R, int k, int Rpad,
                              int8_t* __restrict__ q, uint16_t* __restrict__ qb,
                              float* __restrict__ scale) {
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < Rpad;
         row += gridDim.x * (blockDim.x >> 5)) {
        float a0 = 0.0f, a1 = 0.0f;
        if (row < R) {
            if (lane < k) a0 = A[(size_t)row * k + lane];
            if (lane + 32 < k) a1 = A[(size_t)row * k + lane + 32];
        }
        float m = fmaxf(fabsf(a0), fabsf(a1));
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float s = m / 127.0f;
        int q0 = 0, q1 = 0;
        if (m > 0.0f) {
            q0 = max(-127, min(127, __float2int_rn(a0 / s)));
            q1 = max(-127, min(127, __float2int_rn(a1 / s)));
        }
        int8_t* qr = q + (size_t)row * kLrK;
        uint16_t* br = qb + (size_t)row * kLrK;
        qr[lane] = (int8_t)q0;
        qr[lane + 32] = (int8_t)q1;
        // an integer of magnitude <= 127 is exact in bf16: the top 16 bits of its float
        br[lane] = (uint16_t)(__float_as_uint((float)q0) >> 16);
        br[lane + 32] = (uint16_t)(__float_as_uint((float)q1) >> 16);
        if (lane == 0) scale[row] = s;
    }
}

// Caller-supplied factors q [R][rank] / scale [R] into the padded [Rpad][kLrK] layouts.
__global__ void k_lr_load_factors(const int8_t* __restrict__ qin, const float* __restrict__ sin,
                                  int R, int rank, int Rpad, int8_t* __restrict__ q,
                                  uint16_t* __restrict__ qb, float* __restrict__ scale) {
    const long long total = (long long)Rpad * kLrK;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(k / kLrK), c = (int)(k % kLrK);
        const int v = (i < R && c < rank) ? (int)qin[(size_t)i * rank + c] : 0;
        q[k] = (int8_t)v;
        qb[k] = (uint16_t)(__float_as_uint((float)v) >> 16);
        if (c == 0) scale[i] = i < R ? sin[i] : 0.0f;
    }
}

// n_i = scale_i * |q_i|_2 (the Cauchy-Schwarz bound factor of row i) and ids[i] = i.
__global__ void k_lr_norms(const int8_t* __restrict__ q, const float* __restrict__ scale, int R,
                           float* __restrict__ norm, int* __restrict__ ids) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R) return;
    const int8_t* r = q + (size_t)i * kLrK;
    int ss = 0;
    for (int c = 0; c < kLrK; ++c) ss += (int)r[c] * (int)r[c];
    norm[i] = scale[i] * sqrtf((float)ss);
    ids[i] = i;
}

// Factor rows in the product's stored order: position p holds original row order[p] (rows
// by descending n, so the strongest candidates are met first); positions >= R are zero with
// id INT_MAX.  order == null: identity.
__global__ void k_lr_permute(const uint16_t* __restrict__ qb, const float* __restrict__ scale,
                             const float* __restrict__ norm, const int* __restrict__ order, int R,
                             int Rpad, uint16_t* __restrict__ qbp, float* __restrict__ sp,
                             float* __restrict__ np, int* __restrict__ perm) {
    const long long total = (long long)Rpad * (kLrK / 8);  // 16-byte pieces
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x) {
        const int pos = (int)(k / (kLrK / 8)), piece = (int)(k % (kLrK / 8));
        const int src = pos < R ? (order ? order[pos] : pos) : -1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (src >= 0) v = reinterpret_cast<const uint4*>(qb + (size_t)src * kLrK)[piece];
        reinterpret_cast<uint4*>(qbp + (size_t)pos * kLrK)[piece] = v;
        if (piece == 0) {
            sp[pos] = src >= 0 ? scale[src] : 0.0f;
            np[pos] = src >= 0 ? norm[src] : 0.0f;
            perm[pos] = src >= 0 ? src : 0x7fffffff;
        }
    }
}

}  // namespace rfx
