// After growth: OOB leaf drop, OOB votes / predictions, permutation importance, proximity
// co-membership counts and the finishprox normalisation.
#include <algorithm>

#include "rfx_device.cuh"
#include "rfx_kernels.h"

namespace rfx {

// cpu_testreebag walk (src/rf_testreebag.cpp:37-121): quantitative (cat <= 2) splits go
// left when x <= xbestsplit; categorical ones go right (the histogram grower leaves
// catgoleft empty); at most 1000 steps; a walk that does not end on a terminal node
// reports the root.  `feat_mask` collects the split features met on the way (p <= 256).
__device__ __forceinline__ int walk_oob(const Data& D, const int* st, const int* bv,
                                        const float* xb, const int* tm, int row,
                                        uint32_t* feat_mask) {
    int kt = 0, steps = 0;
    while (st[kt] == 1 && steps < 1000) {
        ++steps;
        const int mv = bv[kt];
        if (feat_mask && mv < 256) feat_mask[mv >> 5] |= 1u << (mv & 31);
        if (D.cat[mv] <= 2) kt = D.xc[(size_t)mv * D.N + row] <= xb[kt] ? tm[2 * kt] : tm[2 * kt + 1];
        else kt = tm[2 * kt + 1];
        if (st[kt] != 1) break;
    }
    return (st[kt] == -1 || st[kt] == 2) ? kt : 0;
}

// OOB leaf of every out-of-bag row of every tree.  grid (rows, trees).
__global__ void k_oob_drop(Data D, Batch B) {
    const int t = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= B.noob[t]) return;
    const size_t mo = (size_t)t * B.M;
    const int row = B.oob[(size_t)t * D.N + j];
    B.oob_leaf[(size_t)t * D.N + row] =
        walk_oob(D, B.status + mo, B.bestvar + mo, B.xbest + mo, B.treemap + 2 * mo, row, nullptr);
}

// Vote / prediction accumulation in tree order (src/rf_random_forest.cpp:1500-1535):
// one thread per row walks the batch's trees in order, so the regression float sum is the
// reference's sequential sum.  Classification keeps integer vote counts.
__global__ void k_votes(Data D, Batch B, int* nout, int* votes, float* oob_sum,
                        float* tree_oob, int tree_oob_stride) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= D.N) return;
    int no = 0;
    float acc = oob_sum ? oob_sum[i] : 0.0f;
    for (int t = 0; t < B.T; ++t) {
        const int leaf = B.oob_leaf[(size_t)t * D.N + i];
        float v = __int_as_float(0x7fc00000);
        if (leaf >= 0) {
            ++no;
            const size_t m = (size_t)t * B.M + leaf;
            if (D.nclass == 1) {
                v = B.nodepred[m];
                acc += v;
            } else {
                const int c = B.nodeclass[m];
                if (c >= 0 && c < D.nclass) votes[(size_t)i * D.nclass + c] += 1;
            }
        }
        if (tree_oob) tree_oob[(size_t)t * tree_oob_stride + i] = v;
    }
    nout[i] += no;
    if (oob_sum) oob_sum[i] = acc;
}

// Features used by the splits of each tree (src/rf_varimp.cpp:265-270).  grid (trees).
__global__ void k_imp_used(Data D, Batch B) {
    const int t = blockIdx.x;
    uint8_t* u = B.used + (size_t)t * D.p;
    for (int k = threadIdx.x; k < D.p; k += blockDim.x) u[k] = 0;
    __syncthreads();
    const size_t mo = (size_t)t * B.M;
    const int nn = B.nnode[t];
    for (int k = threadIdx.x; k < nn; k += blockDim.x)
        if (B.status[mo + k] != -1) u[B.bestvar[mo + k]] = 1;
}

// Permuted walk of cpu_testreeimp_batched (src/rf_varimp.cpp:74-143): feature `mr` is
// read from row prow, the others from row `row`; returns the terminal's class (or -1).
__device__ __forceinline__ int walk_perm_class(const Data& D, const int* st, const int* bv,
                                               const float* xb, const int* tm, const int* ncls,
                                               int nnode, int row, int prow, int mr) {
    int kt = 0;
    for (int k = 0; k < nnode; ++k) {
        if (st[kt] == -1) return ncls[kt];
        const int m = bv[kt];
        if (m < 0 || m >= D.p) break;
        const float v = D.xc[(size_t)m * D.N + (m == mr ? prow : row)];
        if (D.cat[m] <= 2) kt = v <= xb[kt] ? tm[2 * kt] : tm[2 * kt + 1];
        else {
            const int j = (int)(v + 0.5f);
            kt = (j >= 0 && j < D.maxcat) ? tm[2 * kt + 1] : tm[2 * kt];
        }
        if (kt <= 0) return ncls[0];
    }
    return -1;
}

// Permuted walk of cpu_predict_regression (src/rf_varimp.cpp:427-475).
__device__ __forceinline__ float walk_perm_regr(const Data& D, const int* st, const int* bv,
                                                const float* xb, const int* tm, const float* np,
                                                int nnode, int row, int prow, int mr) {
    int kt = 0;
    for (int k = 0; k < nnode; ++k) {
        if (st[kt] == -1) return np[kt];
        const int m = bv[kt];
        if (m < 0 || m >= D.p) break;
        const float v = D.xc[(size_t)m * D.N + (m == mr ? prow : row)];
        if (D.cat[m] <= 2) kt = v <= xb[kt] ? tm[2 * kt] : tm[2 * kt + 1];
        else {
            const int j = (int)(v + 0.5f);
            if (j >= 0 && j < D.maxcat) kt = tm[2 * kt + 1];
            else break;
        }
        if (kt < 0 || kt >= nnode) break;
    }
    return 0.0f;
}

// Classification importance counts (cpu_varimp, src/rf_varimp.cpp:218-427): correct OOB
// votes unpermuted (right) and with each used feature permuted (rightimp).  A feature that
// the row's own path never tests cannot change its terminal node, so only path features
// are re-walked.  grid (rows, trees), 256 threads.
__global__ void __launch_bounds__(256) k_imp_class(Data D, Batch B) {
    const int t = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const int noob = B.noob[t];
    const size_t mo = (size_t)t * B.M;
    const int *st = B.status + mo, *bv = B.bestvar + mo, *tm = B.treemap + 2 * mo, *nc = B.nodeclass + mo;
    const float* xb = B.xbest + mo;
    const bool valid = j < noob;
    uint32_t mask[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int row = 0, lab = 0, cls0 = -1;
    if (valid) {
        row = B.oob[(size_t)t * D.N + j];
        lab = D.lab[row];
        walk_oob(D, st, bv, xb, tm, row, mask);
        cls0 = nc[B.oob_leaf[(size_t)t * D.N + row]];
    }
    const bool wide = D.p > 256 || D.has_cat;
    const int ok0 = valid && cls0 == lab;
    const int s0 = __reduce_add_sync(kFull, ok0);
    if (lane == 0 && s0) atomicAdd(&B.right[t], s0);
    const uint8_t* used = B.used + (size_t)t * D.p;
    const int nn = B.nnode[t];
    const int prow = valid ? D.perm[row] : 0;
    for (int k = 0; k < D.p; ++k) {
        if (!used[k]) continue;
        int ok = ok0;
        if (valid && (wide || ((mask[k >> 5] >> (k & 31)) & 1u)))
            ok = walk_perm_class(D, st, bv, xb, tm, nc, nn, row, prow, k) == lab;
        const int s = __reduce_add_sync(kFull, ok);
        if (lane == 0 && s) atomicAdd(&B.rightimp[(size_t)t * D.p + k], s);
    }
}

// rr = (right - rightimp) / noob per used feature (src/rf_varimp.cpp:345-348).
__global__ void k_imp_class_rr(Data D, Batch B) {
    const int t = blockIdx.x;
    const float noob = (float)B.noob[t];
    for (int k = threadIdx.x; k < D.p; k += blockDim.x) {
        const size_t q = (size_t)t * D.p + k;
        B.rr[q] = B.used[q] ? ((float)B.right[t] - (float)B.rightimp[q]) / noob : 0.0f;
    }
}

// Regression importance, squared errors (cpu_varimp_regression, src/rf_varimp.cpp:477-597):
// d0[j] for the unpermuted prediction, d2[j][k] with feature k permuted, per OOB rank j.
// The squared errors of OOB rank j of tree t into out[k * os], k in [0, p).
// The walks read a node as one 16-byte record (B.imp_node, written by k_imp_pack).
__device__ __forceinline__ int pk_status(const int4& n) { return (int)(int8_t)((unsigned)n.x >> 24); }
__device__ __forceinline__ int pk_feature(const int4& n) { return n.x & 0xFFFFFF; }

__device__ __forceinline__ float walk_perm_regr_pk(const Data& D, const int4* nd, int nnode,
                                                   int row, int prow, int mr) {
    int kt = 0;
    for (int k = 0; k < nnode; ++k) {
        const int4 n = nd[kt];
        if (pk_status(n) == -1) return __int_as_float(n.y);
        const int m = pk_feature(n);
        if (m >= D.p) break;
        const float v = D.xc[(size_t)m * D.N + (m == mr ? prow : row)];
        if (D.cat[m] <= 2) kt = v <= __int_as_float(n.y) ? n.z : n.w;
        else {
            const int j = (int)(v + 0.5f);
            if (j >= 0 && j < D.maxcat) kt = n.w;
            else break;
        }
        if (kt < 0 || kt >= nnode) break;
    }
    return 0.0f;
}

__device__ void imp_regr_row(const Data& D, const Batch& B, int t, int j, float* out, size_t os) {
    const int4* nd = B.imp_node + (size_t)t * B.M;
    const int row = B.oob[(size_t)t * D.N + j];
    // (nodepred itself: a walk that did not end on a terminal node reports the root)
    const float pred = B.nodepred[(size_t)t * B.M + B.oob_leaf[(size_t)t * D.N + row]];
    const float y = D.yreg[row];
    const float d = pred - y;
    const float dd = 1.0f * d * d;
    B.d0[(size_t)t * D.N + j] = dd;
    const int prow = D.perm[row];
    const int nn = B.nnode[t];
    // The permuted walk for feature k follows the row's own path up to the first node that
    // tests k; features never tested on the path keep the unpermuted error.  Along the path
    // only the nodes testing k can turn the walk, so one pass down the row's path checks, at
    // every node, the permuted value of the node's feature (unless that feature's walk has
    // already left the path) and walks the tree from where a permuted walk leaves it.
    for (int k = 0; k < D.p; ++k) out[k * os] = dd;
    bool deep = D.has_cat != 0 || D.p > 64;
    if (!deep) {
        constexpr int kMaxPath = 48;
        unsigned long long tested = 0, left = 0;  // features on the path / walks that left it
        int kt = 0, steps = 0, depth = 0;
        int4 n = nd[0];
        while (pk_status(n) == 1 && steps < 1000) {
            ++steps;
            if (depth == kMaxPath) { deep = true; break; }
            const int f = pk_feature(n);
            if (f >= D.p) { deep = true; break; }
            const float th = __int_as_float(n.y);
            const int l = n.z, r = n.w;
            const int nx = D.xc[(size_t)f * D.N + row] <= th ? l : r;
            tested |= 1ull << f;
            if (!((left >> f) & 1ull)) {
                int pk_kt = D.xc[(size_t)f * D.N + prow] <= th ? l : r;
                if (pk_kt != nx) {
                    left |= 1ull << f;
                    // the rest of the walk, with the step budget the full walk from the
                    // feature's first node has left after this node
                    float pk = 0.0f;
                    if (pk_kt >= 0 && pk_kt < nn) {
                        for (int k = depth + 1; k < nn; ++k) {
                            const int4 q = nd[pk_kt];
                            if (pk_status(q) == -1) { pk = __int_as_float(q.y); break; }
                            const int m = pk_feature(q);
                            const float v = D.xc[(size_t)m * D.N + (m == f ? prow : row)];
                            pk_kt = v <= __int_as_float(q.y) ? q.z : q.w;
                            if (pk_kt < 0 || pk_kt >= nn) break;
                        }
                    }
                    const float dk = pk - y;
                    out[f * os] = 1.0f * dk * dk;
                }
            }
            ++depth;
            kt = nx;
            n = nd[kt];
            if (pk_status(n) != 1) break;
        }
        // walks that never left the path end at the row's own terminal node
        const unsigned long long stay = tested & ~left;
        if (!deep && stay) {
            if (kt >= 0 && kt < nn && pk_status(n) == -1) {
                const float dk = __int_as_float(n.y) - y;
                const float e = 1.0f * dk * dk;
                for (int k = 0; k < D.p; ++k)
                    if ((stay >> k) & 1ull) out[k * os] = e;
            } else {
                deep = true;
            }
        }
    }
    if (deep) {
        for (int k = 0; k < D.p; ++k) {
            const float dk = walk_perm_regr_pk(D, nd, nn, row, prow, k) - y;
            out[k * os] = 1.0f * dk * dk;
        }
    }
}

// The batch's nodes as 16-byte records for the regression importance walks.  grid (M/256, T).
__global__ void k_imp_pack(Batch B) {
    const int t = blockIdx.y;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= B.M) return;
    const size_t m = (size_t)t * B.M + k;
    const int st = B.status[m];
    const float v = st == -1 ? B.nodepred[m] : B.xbest[m];
    B.imp_node[m] = make_int4((int)(((unsigned)st & 0xFFu) << 24 | ((unsigned)B.bestvar[m] & 0xFFFFFFu)),
                              __float_as_int(v), B.treemap[2 * m], B.treemap[2 * m + 1]);
}

// One thread per OOB rank; d2 is feature-major, so a warp's stores of one feature are
// consecutive ranks.
__global__ void __launch_bounds__(256) k_imp_regr(Data D, Batch B) {
    const int t = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= B.noob[t]) return;
    imp_regr_row(D, B, t, j, B.d2 + (size_t)t * D.p * D.N + j, (size_t)D.N);
}

// Serial sums over the OOB rows in row order (the reference's loop order).  One warp per
// (tree, column k): k < p the permuted errors of feature k, k == p the unpermuted errors.
// The warp loads 8 x 32 consecutive ranks at a time (coalesced) and every lane runs the
// same serial chain over them through shuffles.  rsum[t][k] = the sums.
__global__ void __launch_bounds__(256) k_imp_regr_sum(Data D, Batch B) {
    constexpr int U = 8;
    const int p = D.p, P1 = D.p + 1;
    const int g = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (g >= B.T * P1) return;
    const int t = g / P1, k = g - t * P1;
    const int noob = B.noob[t];
    const float* src = k < p ? B.d2 + ((size_t)t * p + k) * D.N : B.d0 + (size_t)t * D.N;
    float s = 0.0f;
    for (int b0 = 0; b0 < noob; b0 += 32 * U) {
        float x[U];
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const int i = b0 + q * 32 + lane;
            x[q] = i < noob ? src[i] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const int n = min(32, noob - (b0 + q * 32));
            if (n == 32) {
#pragma unroll
                for (int e = 0; e < 32; ++e) s += __shfl_sync(kFull, x[q], e);
            } else {
                for (int e = 0; e < n; ++e) s += __shfl_sync(kFull, x[q], e);
            }
        }
    }
    if (lane == 0) B.rsum[(size_t)t * P1 + k] = s;
}

// rr = mse_perm - mse_orig per (tree, feature), 0 for a tree without OOB rows.
__global__ void k_imp_regr_rr(Data D, Batch B) {
    const int t = blockIdx.x, p = D.p;
    const int noob = B.noob[t];
    const float* sum = B.rsum + (size_t)t * (p + 1);
    for (int k = threadIdx.x; k < p; k += blockDim.x) {
        if (noob == 0) {
            B.rr[(size_t)t * p + k] = 0.0f;
        } else {
            const float mse0 = sum[p] / (float)noob;
            B.rr[(size_t)t * p + k] = sum[k] / (float)noob - mse0;
        }
    }
}

// avimp += rr, sqsd += rr*rr over the batch's trees in order (src/rf_random_forest.cpp:1903-1906).
__global__ void k_imp_fold(Data D, Batch B, float* avimp, float* sqsd) {
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < D.p; k += gridDim.x * blockDim.x) {
        float a = avimp[k], s = sqsd[k];
        for (int t = 0; t < B.T; ++t) {
            const float r = B.rr[(size_t)t * D.p + k];
            a += r;
            s += r * r;
        }
        avimp[k] = a;
        sqsd[k] = s;
    }
}

// ---------------------------------------------------------------------------------------
// Proximity counts (cpu_proximity dense branch, src/rf_proximity.cpp:99-230, integer
// weights): every OOB row i in terminal node k meets every distinct in-bag row j of k,
// C[min(i,j), max(i,j)] += 1 in the packed upper triangle over rows [0, R).  The in-bag
// rows of a terminal node are its segment from growth.  grid (rows, trees).
// ---------------------------------------------------------------------------------------
__global__ void k_prox(Data D, Batch B, int R, int* __restrict__ C) {
    const int t = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= B.noob[t]) return;
    const int row = B.oob[(size_t)t * D.N + j];
    if (row >= R) return;
    const int leaf = B.oob_leaf[(size_t)t * D.N + row];
    const size_t m = (size_t)t * B.M + leaf;
    if (B.status[m] != -1) return;
    const int st = B.nd_start[m], c = B.nd_cnt[m];
    const int* seg = B.seg[B.nd_buf[m]] + (size_t)t * D.N + st;
    const long long R2 = 2LL * R;
    unsigned long long done = 0;
    for (int q = 0; q < c; ++q) {
        const int col = seg[q];
        if (col >= R) continue;
        const long long a = min(row, col), b = max(row, col);
        atomicAdd(&C[a * (R2 - a - 1) / 2 + (b - a - 1)], 1);
        ++done;
    }
    if (B.prox_pairs && done) atomicAdd(B.prox_pairs, done);
}

// ---------------------------------------------------------------------------------------
// The same counts pulled tile by tile.  Give every row of tree t the 16-bit code
// 2 * (terminal node) + (1 if OOB): rows i and j add one pair in tree t exactly when their
// codes differ in the last bit only.  k_prox_codes writes the codes of a batch ([T][R],
// rows >= R and padding trees 0xFFFF, which never pair) and counts the pairs the batch
// adds (sum over terminal nodes of OOB rows x in-bag rows, both below R), which decides
// between pushing (k_prox) and pulling (k_prox_pull).  Block per tree; ocnt: [T][M] ints.
// ---------------------------------------------------------------------------------------
__global__ void k_prox_codes(Batch B, int N, int R, uint16_t* __restrict__ code,
                             int* __restrict__ ocnt, unsigned long long* __restrict__ pairs) {
    __shared__ unsigned long long red[32];
    const int t = blockIdx.x, M = B.M;
    const int nn = B.nnode[t];
    const int* status = B.status + (size_t)t * M;
    uint16_t* ct = code + (size_t)t * R;
    int* oc = ocnt + (size_t)t * M;
    for (int m = threadIdx.x; m < nn; m += blockDim.x) oc[m] = 0;
    __syncthreads();
    const int noob = B.noob[t];
    const int* oob = B.oob + (size_t)t * N;
    const int* oleaf = B.oob_leaf + (size_t)t * N;
    for (int i = threadIdx.x; i < noob; i += blockDim.x) {
        const int row = oob[i];
        if (row >= R) continue;
        const int leaf = oleaf[row];
        atomicAdd(&oc[leaf], 1);
        ct[row] = (uint16_t)(2 * leaf + 1);
    }
    __syncthreads();
    unsigned long long mine = 0;
    for (int m = threadIdx.x; m < nn; m += blockDim.x) {
        if (status[m] != -1) continue;
        const size_t nm = (size_t)t * M + m;
        const int* seg = B.seg[B.nd_buf[nm]] + (size_t)t * N + B.nd_start[nm];
        const int c = B.nd_cnt[nm];
        int k = 0;
        for (int q = 0; q < c; ++q) {
            const int row = seg[q];
            if (row >= R) continue;
            ct[row] = (uint16_t)(2 * m);
            ++k;
        }
        mine += (unsigned long long)k * (unsigned long long)oc[m];
    }
    for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long tot = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        atomicAdd(pairs, tot);
    }
}

// C[i][j] (i < j < R) += #{trees t of the batch : code_t(i) ^ code_t(j) == 1}.  Block per
// 128 x 128 tile of the upper triangle (tile id k enumerates block pairs bi <= bj row by
// row); thread (tx, ty) owns rows i0 + 8 ty .. +7 and columns j0 + 8 tx .. +7.  Codes of two
// trees travel packed in one word; the column codes are staged with the OOB bit flipped, so
// a pair is a 16-bit half-word equality (__vcmpeq2: 0xFFFF per equal half).  Tp is even.
constexpr int kPullTile = 128;
constexpr int kPullChunk = 32;  // tree pairs staged per pass

__global__ void __launch_bounds__(256) k_prox_pull(const uint16_t* __restrict__ code, int Tp,
                                                   int R, int nb, int* __restrict__ C) {
    __shared__ __align__(16) uint32_t si[kPullChunk][kPullTile];
    __shared__ __align__(16) uint32_t sj[kPullChunk][kPullTile];
    // tile id -> (bi, bj), bi <= bj; row bi holds nb - bi tiles
    long long k = blockIdx.x;
    int bi = 0;
    {
        // first tile of row b is b*nb - b*(b-1)/2; invert with a square root and fix up
        const double nbd = nb + 0.5;
        int g = (int)(nbd - sqrt(nbd * nbd - 2.0 * (double)k));
        g = max(0, min(nb - 1, g));
        while (g > 0 && (long long)g * nb - (long long)g * (g - 1) / 2 > k) --g;
        while (g + 1 < nb && (long long)(g + 1) * nb - (long long)(g + 1) * g / 2 <= k) ++g;
        bi = g;
    }
    const int bj = bi + (int)(k - ((long long)bi * nb - (long long)bi * (bi - 1) / 2));
    const int i0 = bi * kPullTile, j0 = bj * kPullTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    int acc[8][8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int v = 0; v < 8; ++v) acc[u][v] = 0;
    for (int tp0 = 0; tp0 < Tp / 2; tp0 += kPullChunk) {
        const int ntp = min(kPullChunk, Tp / 2 - tp0);
        for (int e = threadIdx.x; e < kPullChunk * kPullTile; e += blockDim.x) {
            const int tp = e / kPullTile, r = e % kPullTile;
            uint32_t wi = 0xFFFFFFFFu, wj = 0xFFFFFFFFu;
            if (tp < ntp) {
                const size_t t0 = (size_t)(2 * (tp0 + tp));
                const int ri = i0 + r, rj = j0 + r;
                if (ri < R) wi = (uint32_t)code[t0 * R + ri] | ((uint32_t)code[(t0 + 1) * R + ri] << 16);
                if (rj < R) wj = (uint32_t)code[t0 * R + rj] | ((uint32_t)code[(t0 + 1) * R + rj] << 16);
            }
            si[tp][r] = wi;
            sj[tp][r] = wj ^ 0x00010001u;
        }
        __syncthreads();
        for (int tp = 0; tp < ntp; ++tp) {
            const uint4 a0 = *reinterpret_cast<const uint4*>(&si[tp][8 * ty]);
            const uint4 a1 = *reinterpret_cast<const uint4*>(&si[tp][8 * ty + 4]);
            const uint4 b0 = *reinterpret_cast<const uint4*>(&sj[tp][8 * tx]);
            const uint4 b1 = *reinterpret_cast<const uint4*>(&sj[tp][8 * tx + 4]);
            const uint32_t a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const uint32_t b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int v = 0; v < 8; ++v) acc[u][v] += __popc(__vcmpeq2(a[u], b[v]));
        }
        __syncthreads();
    }
    const long long R2 = 2LL * R;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int i = i0 + 8 * ty + u;
        if (i >= R) continue;
        int* row = C + (long long)i * (R2 - i - 1) / 2 - i - 1;  // row[j] for j > i
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const int j = j0 + 8 * tx + v;
            if (j > i && j < R) row[j] += acc[u][v] >> 4;
        }
    }
}

// finishprox (src/rf_finishprox.cpp:12-74) of rows [r0, r1): with C the symmetric count,
// S_ij = 0.5 * (C/2 * (1/nout_i) + C/2 * (1/nout_j)) in double (a row with nout 0 is left
// unscaled), diagonal 1, returned as float32 like get_proximity_matrix
// (python/randomforest_py.cpp:2129-2155).  Block per 64 x 64 output tile: a tile above the
// diagonal reads its counts row by row from the packed upper triangle, a tile below it reads
// the mirrored tile (again row by row) and transposes it through shared memory, so every
// global access is contiguous; tiles crossing the diagonal read entry by entry.
constexpr int kFinTile = 64;

__device__ __forceinline__ long long upper_index(long long a, long long b, long long R2) {
    return a * (R2 - a - 1) / 2 + (b - a - 1);  // a < b
}

__global__ void __launch_bounds__(256) k_prox_finish(const int* __restrict__ C,
                                                     const int* __restrict__ nout, int R,
                                                     int r0, int r1, float* __restrict__ out) {
    __shared__ int tile[kFinTile][kFinTile + 1];  // tile[ii][jj] = C of (i0 + ii, j0 + jj)
    __shared__ double sc_i[kFinTile], sc_j[kFinTile];
    const int i0 = r0 + blockIdx.y * kFinTile, j0 = blockIdx.x * kFinTile;
    const long long R2 = 2LL * R;
    const int tid = threadIdx.x;
    if (tid < kFinTile) {
        const int i = i0 + tid;
        const int ni = i < r1 ? nout[i] : 0;
        sc_i[tid] = ni > 0 ? 1.0 / (double)ni : 1.0;
    } else if (tid < 2 * kFinTile) {
        const int j = j0 + tid - kFinTile;
        const int nj = j < R ? nout[j] : 0;
        sc_j[tid - kFinTile] = nj > 0 ? 1.0 / (double)nj : 1.0;
    }
    const bool upper = i0 + kFinTile <= j0;  // every i < every j
    const bool lower = j0 + kFinTile <= i0;  // every j < every i
    if (upper) {
        for (int e = tid; e < kFinTile * kFinTile; e += blockDim.x) {
            const int ii = e / kFinTile, jj = e % kFinTile;
            const int i = i0 + ii, j = j0 + jj;
            tile[ii][jj] = (i < r1 && j < R) ? C[upper_index(i, j, R2)] : 0;
        }
    } else if (lower) {
        for (int e = tid; e < kFinTile * kFinTile; e += blockDim.x) {
            const int jj = e / kFinTile, ii = e % kFinTile;  // consecutive threads: row j, ascending i
            const int i = i0 + ii, j = j0 + jj;
            tile[ii][jj] = (i < r1 && j < R) ? C[upper_index(j, i, R2)] : 0;
        }
    } else {
        for (int e = tid; e < kFinTile * kFinTile; e += blockDim.x) {
            const int ii = e / kFinTile, jj = e % kFinTile;
            const int i = i0 + ii, j = j0 + jj;
            int v = 0;
            if (i < r1 && j < R && i != j) v = C[upper_index(min(i, j), max(i, j), R2)];
            tile[ii][jj] = v;
        }
    }
    __syncthreads();
    for (int e = tid; e < kFinTile * kFinTile; e += blockDim.x) {
        const int ii = e / kFinTile, jj = e % kFinTile;
        const int i = i0 + ii, j = j0 + jj;
        if (i >= r1 || j >= R) continue;
        float v;
        if (i == j) {
            v = 1.0f;
        } else {
            const double h = (double)tile[ii][jj] / 2.0;
            const double si = h * sc_i[ii];
            const double sj = h * sc_j[jj];
            v = (float)(0.5 * (si + sj));
        }
        out[(size_t)(i - r0) * R + j] = v;
    }
}

cudaError_t launch_prox_finish(const int* C, const int* nout, int R, int r0, int r1, float* out,
                               cudaStream_t st) {
    if (r1 <= r0) return cudaSuccess;
    const dim3 grid((unsigned)((R + kFinTile - 1) / kFinTile),
                    (unsigned)((r1 - r0 + kFinTile - 1) / kFinTile));
    k_prox_finish<<<grid, 256, 0, st>>>(C, nout, R, r0, r1, out);
    return cudaGetLastError();
}

// 1 / nout (1 where nout is 0): the row scales of finishprox.
__global__ void k_inv_nout(const int* __restrict__ nout, int R, double* __restrict__ inv) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < R; i += gridDim.x * blockDim.x)
        inv[i] = nout[i] > 0 ? 1.0 / (double)nout[i] : 1.0;
}

// The whole R x R finished matrix from tile pairs: block (bi <= bj) reads the counts of the
// upper tile (rows of tile bi, columns of tile bj) once -- rows of the packed triangle, so
// the loads coalesce -- and writes them finished to both the tile and its mirror (the
// mirror's rows through a shared-memory transpose); diagonal tiles fill both halves and the
// unit diagonal.  Per element the double operations of k_prox_finish; inv = 1 / nout.
__global__ void __launch_bounds__(256) k_prox_finish_full(const int* __restrict__ C,
                                                          const double* __restrict__ inv, int R,
                                                          int nb, float* __restrict__ out) {
    __shared__ float tile[kFinTile][kFinTile + 1];
    __shared__ double sc_i[kFinTile], sc_j[kFinTile];
    __shared__ long long rowbase[kFinTile];
    // pair index -> (bi, bj), bi <= bj, row-major over the upper triangle of tiles
    const long long pidx = blockIdx.x;
    int bi = (int)((2.0 * nb + 1 - sqrt((2.0 * nb + 1) * (2.0 * nb + 1) - 8.0 * (double)pidx)) / 2.0);
    bi = max(0, min(bi, nb - 1));
    auto first = [&](int b) { return (long long)b * nb - (long long)b * (b - 1) / 2; };
    while (bi > 0 && first(bi) > pidx) --bi;
    while (bi + 1 < nb && first(bi + 1) <= pidx) ++bi;
    const int bj = bi + (int)(pidx - first(bi));
    const int i0 = bi * kFinTile, j0 = bj * kFinTile;
    const long long R2 = 2LL * R;
    const int tid = threadIdx.x;
    if (tid < kFinTile) {
        const int i = i0 + tid;
        sc_i[tid] = i < R ? inv[i] : 1.0;
        rowbase[tid] = (long long)i * (R2 - i - 1) / 2 - i - 1;  // + j = packed index of (i, j)
    } else if (tid < 2 * kFinTile) {
        const int j = j0 + tid - kFinTile;
        sc_j[tid - kFinTile] = j < R ? inv[j] : 1.0;
    }
    __syncthreads();
    const bool diag = bi == bj;
    for (int e = tid; e < kFinTile * kFinTile; e += blockDim.x) {
        const int ii = e / kFinTile, jj = e % kFinTile;
        const int i = i0 + ii, j = j0 + jj;
        if (i >= R || j >= R) continue;
        float v;
        if (i == j) {
            v = 1.0f;
        } else if (diag && j < i) {
            continue;  // written as the mirror of (j, i)
        } else {
            const double h = (double)C[rowbase[ii] + j] / 2.0;
            v = (float)(0.5 * (h * sc_i[ii] + h * sc_j[jj]));
        }
        tile[ii][jj] = v;
        out[(size_t)i * R + j] = v;
    }
    __syncthreads();
    for (int e = tid; e < kFinTile * kFinTile; e += blockDim.x) {
        const int jj = e / kFinTile, ii = e % kFinTile;  // consecutive threads: row j, ascending i
        const int i = i0 + ii, j = j0 + jj;
        if (i >= R || j >= R || i >= j) continue;
        out[(size_t)j * R + i] = tile[ii][jj];
    }
}

cudaError_t launch_prox_finish_full(const int* C, const int* nout, int R, double* inv, float* out,
                                    cudaStream_t st) {
    if (R <= 0) return cudaSuccess;
    k_inv_nout<<<(R + 255) / 256, 256, 0, st>>>(nout, R, inv);
    const int nb = (R + kFinTile - 1) / kFinTile;
    const long long pairs = (long long)nb * (nb + 1) / 2;
    k_prox_finish_full<<<(unsigned)pairs, 256, 0, st>>>(C, inv, R, nb, out);
    return cudaGetLastError();
}


// Finished values of the packed upper-triangle elements [e0, e0 + len), element e = (i, j),
// e = i (2R - i - 1) / 2 + (j - i - 1): the same double operations as k_prox_finish, which
// only need C_ij and the two row scales -- so a rank finishes its own slice of a
// reduce-scattered triangle.  C and out hold the slice (index e - e0).  A warp covers 32 x
// kPackRun consecutive elements, lane-interleaved so that loads and stores coalesce.
constexpr int kPackRun = 8;
__global__ void __launch_bounds__(256) k_prox_finish_packed(const int* __restrict__ C, long long e0,
                                                            long long len, const double* __restrict__ inv,
                                                            int R, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long long R2 = 2LL * R;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long w = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
         w * 32 * kPackRun < len; w += warps) {
        const long long b = w * 32 * kPackRun + lane;  // first element of this lane
        if (b >= len) continue;
        const long long e = e0 + b;
        // row of e: the largest i with i (2R - i - 1) / 2 <= e (double estimate, then exact)
        const double a = (double)(R2 - 1);
        long long i = (long long)((a - sqrt(fmax(a * a - 8.0 * (double)e, 0.0))) * 0.5);
        i = max(0LL, min(i, (long long)R - 2));
        while (i > 0 && i * (R2 - i - 1) / 2 > e) --i;
        while (i < R - 2 && (i + 1) * (R2 - i - 2) / 2 <= e) ++i;
        long long j = e - i * (R2 - i - 1) / 2 + i + 1;
        double si = inv[i];
#pragma unroll
        for (int k = 0; k < kPackRun; ++k) {
            const long long q = b + (long long)k * 32;
            if (q >= len) break;
            const double h = (double)C[q] / 2.0;
            out[q] = (float)(0.5 * (h * si + h * inv[j]));
            j += 32;  // the lane's next element
            while (j >= R && i < R - 2) {
                j -= R - i - 2;  // continue on row i + 1, whose first column is i + 2
                ++i;
                si = inv[i];
            }
        }
    }
}

cudaError_t launch_prox_finish_packed(const int* C, long long e0, long long len, const int* nout,
                                      int R, double* inv, float* out, cudaStream_t st) {
    k_inv_nout<<<(R + 255) / 256, 256, 0, st>>>(nout, R, inv);
    if (len > 0) {
        const long long per_block = 8LL * 32 * kPackRun;
        const unsigned grid = (unsigned)std::min<long long>((len + per_block - 1) / per_block, 148LL * 16);
        k_prox_finish_packed<<<grid, 256, 0, st>>>(C, e0, len, inv, R, out);
    }
    return cudaGetLastError();
}

// q[i][c] = classwt[c] added votes[i][c] times, sequentially (src/rf_random_forest.cpp:1506-1520).
__global__ void k_votes_to_q(const int* __restrict__ votes, const float* __restrict__ w, int N,
                             int nclass, float* __restrict__ q) {
    const long long total = (long long)N * nclass;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(k % nclass);
        const float wc = w ? 1.0f * w[c] : 1.0f;
        float a = 0.0f;
        for (int r = votes[k]; r > 0; --r) a += wc;
        q[k] = a;
    }
}

// vec[i] += per-tree OOB predictions in tree order (NaN marks in-bag).
__global__ void k_oob_fold(const float* __restrict__ tree_oob, int ntrees, int N,
                           float* __restrict__ vec) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    float a = vec[i];
    for (int t = 0; t < ntrees; ++t) {
        const float v = tree_oob[(size_t)t * N + i];
        if (!isnan(v)) a += v;
    }
    vec[i] = a;
}

}  // namespace rfx
