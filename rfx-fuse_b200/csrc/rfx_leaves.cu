// Leaf assignments and the queries built on them: top-k similar training rows, the leaf
// proximity of a pair, leaf assignments and top-k similar rows for new data, Breiman-Cutler
// outlier scores and their anchors (include/rf_random_forest.hpp:296-365,
// src/rf_random_forest.cpp:1543-1610, 4110-4420, 4605-4850).
//
// Layout on the device: leaf [tree][N] int16 (the reference's leaf_assignments_ layout),
// OOB flags [tree][ceil(N/32)] bit words, and the inverted index: (tree, leaf) keys sorted
// with their rows (a stable radix sort keeps rows ascending inside a group, as the
// reference's index lists them) and per-group [start, end) offsets.
//
// Counting runs on the device (a warp per query walks the query's groups, a lane per member;
// the members of one group are distinct rows, so the increments never collide).  Rankings
// whose tie order the reference leaves to std::partial_sort / std::sort are made by the same
// library calls on the host from the device counts (only the nonzero entries for training
// queries), so the order of tied rows is the reference's.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <map>
#include <numeric>
#include <random>
#include <vector>

#include <cub/cub.cuh>

#include "rfx_ctx.h"
#include "rfx_kernels.h"
#include "rfx_predict.h"

using namespace rfxh;

namespace rfx {

namespace {

__device__ __forceinline__ int x86_float_to_int_leaf(float y) {
    if (!(y >= -2147483648.0f && y < 2147483648.0f)) return (int)0x80000000;
    return (int)y;
}

}  // namespace

// Terminal node of every grown row in each tree of a batch (find_terminal_node,
// src/rf_random_forest.cpp:3724-3770, numeric features), and the tree's OOB flags.
__global__ void k_leaf_assign(Data D, Batch B, int16_t* __restrict__ leaf,
                              uint32_t* __restrict__ oobw, int words) {
    const int t = blockIdx.y;
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    bool oob = false;
    if (row < D.N) {
        const size_t mo = (size_t)t * B.M;
        const int *st = B.status + mo, *bv = B.bestvar + mo, *tm = B.treemap + 2 * mo;
        const float* xb = B.xbest + mo;
        int kt = 0;
        for (int k = 0; k < B.M; ++k) {
            if (st[kt] == -1) break;
            const int m = bv[kt];
            if (m < 0 || m >= D.p) break;  // the reference's loop stays on this node
            const int nx = D.xc[(size_t)m * D.N + row] <= xb[kt] ? tm[2 * kt] : tm[2 * kt + 1];
            if (nx < 0 || nx >= B.M) break;
            kt = nx;
        }
        leaf[(size_t)t * D.N + row] = (int16_t)kt;
        oob = B.nin[(size_t)t * D.N + row] == 0;
    }
    const unsigned bal = __ballot_sync(kFull, oob);
    if ((threadIdx.x & 31) == 0 && row < D.N) oobw[(size_t)t * words + (row >> 5)] = bal;
}

// Inverted index keys: (tree, leaf) -> t * W + (uint16)leaf, value = row.
__global__ void k_leaf_keys(const int16_t* __restrict__ leaf, int T, int N, int W,
                            uint32_t* __restrict__ keys, int* __restrict__ rows) {
    const size_t total = (size_t)T * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / N);
        keys[i] = (uint32_t)t * (uint32_t)W + (uint32_t)(uint16_t)leaf[i];
        rows[i] = (int)(i - (size_t)t * N);
    }
}

// Group offsets from the sorted keys (gs/ge zeroed before).
__global__ void k_leaf_offsets(const uint32_t* __restrict__ keys, size_t total, int* __restrict__ gs,
                               int* __restrict__ ge) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t k = keys[i];
        if (i == 0 || keys[i - 1] != k) gs[k] = (int)i;
        if (i + 1 == total || keys[i + 1] != k) ge[k] = (int)(i + 1);
    }
}

// Training queries: cnt[qi][m] = trees where query q was OOB and row m shares its leaf (the
// query itself skipped with exclude_self); noob[qi] = the query's OOB trees.  Warp per query.
__global__ void k_leaf_query(const int16_t* __restrict__ leaf, const uint32_t* __restrict__ oobw,
                             int words, const int* __restrict__ gs, const int* __restrict__ ge,
                             const int* __restrict__ rows, int N, int T, int W,
                             const int* __restrict__ queries, int nq, int exclude_self,
                             int* __restrict__ cnt, int* __restrict__ noob) {
    const int lane = threadIdx.x & 31;
    const int qi = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    if (qi >= nq) return;
    const int q = queries[qi];
    int* c = cnt + (size_t)qi * N;
    int no = 0;
    for (int t = 0; t < T; ++t) {
        if (!((oobw[(size_t)t * words + (q >> 5)] >> (q & 31)) & 1u)) continue;
        ++no;
        const uint32_t g = (uint32_t)t * (uint32_t)W + (uint32_t)(uint16_t)leaf[(size_t)t * N + q];
        for (int i = gs[g] + lane; i < ge[g]; i += 32) {
            const int m = rows[i];
            if (!(exclude_self && m == q)) c[m] += 1;
        }
        __syncwarp();
    }
    if (lane == 0) noob[qi] = no;
}

// New rows: cnt[qi][m] = trees where training row m shares the new row's leaf.  Warp per row.
__global__ void k_leaf_query_new(const int16_t* __restrict__ newleaf, const int* __restrict__ gs,
                                 const int* __restrict__ ge, const int* __restrict__ rows, int N,
                                 int T, int W, int nq, int* __restrict__ cnt) {
    const int lane = threadIdx.x & 31;
    const int qi = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    if (qi >= nq) return;
    int* c = cnt + (size_t)qi * N;
    for (int t = 0; t < T; ++t) {
        const uint32_t g = (uint32_t)t * (uint32_t)W + (uint32_t)(uint16_t)newleaf[(size_t)qi * T + t];
        for (int i = gs[g] + lane; i < ge[g]; i += 32) c[rows[i]] += 1;
        __syncwarp();
    }
}

// Nonzero counts of each query in ascending row order: block per query.
__global__ void __launch_bounds__(1024) k_leaf_compact(const int* __restrict__ cnt, int N,
                                                       int* __restrict__ cidx,
                                                       int* __restrict__ cval,
                                                       int* __restrict__ nnz) {
    using Scan = cub::BlockScan<int, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ int base;
    const int qi = blockIdx.x;
    const int* c = cnt + (size_t)qi * N;
    if (threadIdx.x == 0) base = 0;
    __syncthreads();
    for (int i0 = 0; i0 < N; i0 += 1024) {
        const int i = i0 + threadIdx.x;
        const int v = i < N ? c[i] : 0;
        int pos, tot;
        Scan(tmp).ExclusiveSum(v > 0 ? 1 : 0, pos, tot);
        if (v > 0) {
            cidx[(size_t)qi * N + base + pos] = i;
            cval[(size_t)qi * N + base + pos] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) base += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) nnz[qi] = base;
}

// compute_proximity_from_leaves for one pair: out[0] = matches, out[1] = OOB trees of i.
__global__ void k_leaf_pair(const int16_t* __restrict__ leaf, const uint32_t* __restrict__ oobw,
                            int words, int N, int T, int i, int j, int* __restrict__ out) {
    int match = 0, no = 0;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        if (!((oobw[(size_t)t * words + (i >> 5)] >> (i & 31)) & 1u)) continue;
        ++no;
        match += leaf[(size_t)t * N + i] == leaf[(size_t)t * N + j];
    }
    for (int o = 16; o > 0; o >>= 1) {
        match += __shfl_xor_sync(kFull, match, o);
        no += __shfl_xor_sync(kFull, no, o);
    }
    if (threadIdx.x == 0) {
        out[0] = match;
        out[1] = no;
    }
}

// predict_leaf_assignments walk over the device forest: out[s * T + t].  xc [p][n].
__global__ void k_leaf_predict(const PNode* __restrict__ forest, int M, int T,
                               const float* __restrict__ xc, int n, int p,
                               const int* __restrict__ cat, int16_t* __restrict__ out) {
    const int t = blockIdx.y;
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const PNode* nodes = forest + (size_t)t * M;
    int kt = 0;
    for (int k = 0; k < M; ++k) {
        const PNode nd = nodes[kt];
        if (nd.feat == -1) break;
        const int m = nd.feat;
        if (m < 0 || m >= p) break;  // no move: the walk stays here
        const float x = xc[(size_t)m * n + s];
        int nx;
        if (cat[m] == 1) {
            nx = x <= nd.val ? nd.left : nd.right;
        } else {
            const int jcat = x86_float_to_int_leaf(x + 0.5f);
            if (!(jcat >= 0 && jcat < cat[m])) break;  // no move
            nx = nd.right;  // catgoleft is empty for histogram-grown trees
        }
        if (nx < 0 || nx >= M) break;
        kt = nx;
    }
    out[(size_t)s * T + t] = (int16_t)kt;
}

// Greedy outlier measure: raw[n] = n_anchors / sum over anchors a != n of (shared / T)^2.
__global__ void k_outlier_greedy(const int16_t* __restrict__ leaf, int T, int N,
                                 const int* __restrict__ anchors, int na, int n_anchors,
                                 float* __restrict__ raw) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float s = 0.0f;
    for (int ai = 0; ai < na; ++ai) {
        const int a = anchors[ai];
        if (a == n) continue;
        int shared = 0;
        for (int t = 0; t < T; ++t) shared += leaf[(size_t)t * N + n] == leaf[(size_t)t * N + a];
        const float prox = (float)shared / (float)T;
        s += prox * prox;
    }
    raw[n] = s > 1e-10f ? (float)n_anchors / s : (float)n_anchors * 1e10f;
}

// Full outlier measure: per row n, sum over the other rows m of c_m^2 (c_m = trees where m
// shares n's leaf), exact in integers: each increment c -> c + 1 adds 2c + 1.  Warp per row
// with a zeroed per-warp count array of N ints (restored to zero afterwards).
__global__ void k_outlier_full(const int16_t* __restrict__ leaf, const int* __restrict__ gs,
                               const int* __restrict__ ge, const int* __restrict__ rows, int N,
                               int T, int W, int* __restrict__ scratch,
                               float* __restrict__ raw) {
    const int lane = threadIdx.x & 31;
    const int wid = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int nw = (int)((gridDim.x * (size_t)blockDim.x) >> 5);
    int* c = scratch + (size_t)wid * N;
    for (int n = wid; n < N; n += nw) {
        unsigned long long S = 0;
        for (int t = 0; t < T; ++t) {
            const uint32_t g = (uint32_t)t * (uint32_t)W + (uint32_t)(uint16_t)leaf[(size_t)t * N + n];
            for (int i = gs[g] + lane; i < ge[g]; i += 32) {
                const int m = rows[i];
                if (m != n) {
                    const int v = c[m];
                    c[m] = v + 1;
                    S += 2ull * (unsigned long long)v + 1ull;
                }
            }
            __syncwarp();
        }
        for (int t = 0; t < T; ++t) {
            const uint32_t g = (uint32_t)t * (uint32_t)W + (uint32_t)(uint16_t)leaf[(size_t)t * N + n];
            for (int i = gs[g] + lane; i < ge[g]; i += 32) c[rows[i]] = 0;
        }
        __syncwarp();
        for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(kFull, S, o);
        if (lane == 0) {
            const float pss = (float)((double)S / ((double)T * (double)T));
            raw[n] = pss > 1e-10f ? (float)(N - 1) / pss : (float)N * 1e10f;
        }
    }
}

// New-row outlier measures (predict_outlier_scores): per new row q, from cnt[q][i] = trees
// where training row i shares its leaf, raw = n / sum of (cnt / T)^2 over the positive
// entries -- full: all of them in row order; greedy: the n_anchors largest, in descending
// order (from hist[q][c] = rows with count c; equal values, so the order among them is
// immaterial).  Thread per new row.
__global__ void k_outlier_new(const int* __restrict__ cnt, const int* __restrict__ hist, int N,
                              int T, int nq, int greedy, int n_anchors, float* __restrict__ raw) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    float ss = 0.0f;
    int used = 0;
    if (greedy && n_anchors > 0) {
        const int* h = hist + (size_t)q * (T + 1);
        int left = n_anchors;
        for (int v = T; v >= 1 && left > 0; --v) {
            const int k = min(h[v], left);
            const float pr = (float)v / (float)T;
            for (int e = 0; e < k; ++e) ss += pr * pr;
            used += k;
            left -= k;
        }
    } else {
        const int* c = cnt + (size_t)q * N;
        for (int i = 0; i < N; ++i) {
            const int v = c[i];
            if (v > 0) {
                const float pr = (float)v / (float)T;
                ss += pr * pr;
                ++used;
            }
        }
    }
    raw[q] = (ss > 1e-10f && used > 0) ? (float)used / ss : (float)N * 1e10f;
}

// hist[q][c] += 1 for every training row with count c > 0.
__global__ void k_outlier_new_hist(const int* __restrict__ cnt, int N, int T, int nq,
                                   int* __restrict__ hist) {
    const int q = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) {
        const int v = cnt[(size_t)q * N + i];
        if (v > 0) atomicAdd(&hist[(size_t)q * (T + 1) + v], 1);
    }
}

// Diverse anchors, one step: mn[n] = min(mn[n], proximity of n to the last anchor).
__global__ void k_anchor_update(const int16_t* __restrict__ leaf, int T, int N, int last,
                                float* __restrict__ mn) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    int shared = 0;
    for (int t = 0; t < T; ++t) shared += leaf[(size_t)t * N + n] == leaf[(size_t)t * N + last];
    const float prox = (float)shared / (float)T;
    mn[n] = std::min(mn[n], prox);
}

// The first row (ascending) of smallest mn[] below 2 that is not an anchor yet; -1 if none.
__global__ void __launch_bounds__(1024) k_anchor_pick(const float* __restrict__ mn,
                                                      const uint8_t* __restrict__ taken, int N,
                                                      int* __restrict__ best) {
    float bv = 2.0f;
    int bi = -1;
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
        if (taken[n]) continue;
        if (mn[n] < bv) {
            bv = mn[n];
            bi = n;
        }
    }
    __shared__ float sv[1024];
    __shared__ int si[1024];
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = 512; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = sv[threadIdx.x + s];
            const int oi = si[threadIdx.x + s];
            const bool take = oi >= 0 && (si[threadIdx.x] < 0 || ov < sv[threadIdx.x] ||
                                          (ov == sv[threadIdx.x] && oi < si[threadIdx.x]));
            if (take) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) best[0] = si[0];
}

}  // namespace rfx

namespace rfxh {

void leaves_reset(Ctx& c) {
    c.l_T = 0;
    c.l_index = false;
    c.l_anchors.clear();
    c.l_words = (int)((c.N + 31) / 32);
    c.l_W = c.M <= 32768 ? c.M : 65536;
}

void leaves_store_batch(Ctx& c, const rfx::Batch& B, int T) {
    const size_t N = c.N, words = c.l_words;
    const int need = c.l_T + T;
    if (need > c.l_cap) {
        const int cap = std::max(need, 2 * c.l_cap);
        DBuf leaf, oob;
        leaf.get((size_t)cap * N * 2);
        oob.get((size_t)cap * words * 4);
        if (c.l_T > 0) {
            RFX_CUDA(cudaMemcpyAsync(leaf.p, c.l_leaf.p, (size_t)c.l_T * N * 2, cudaMemcpyDeviceToDevice, c.st));
            RFX_CUDA(cudaMemcpyAsync(oob.p, c.l_oob.p, (size_t)c.l_T * words * 4, cudaMemcpyDeviceToDevice, c.st));
        }
        RFX_CUDA(cudaStreamSynchronize(c.st));
        c.l_leaf.release();
        c.l_oob.release();
        c.l_leaf = leaf;
        c.l_oob = oob;
        leaf.p = oob.p = nullptr;
        c.l_cap = cap;
    }
    const dim3 grid((unsigned)((N + 255) / 256), (unsigned)T);
    rfx::k_leaf_assign<<<grid, 256, 0, c.st>>>(c.D, B, (int16_t*)c.l_leaf.p + (size_t)c.l_T * N,
                                              (uint32_t*)c.l_oob.p + (size_t)c.l_T * words,
                                              (int)words);
    RFX_LAUNCH("k_leaf_assign");
    c.launches += 1;
    c.l_T += T;
    c.l_index = false;
}

namespace {

void require_leaves(Ctx& c) {
    require(c.loaded && c.prm.keep_leaves && c.l_T > 0, RFX_ERR_STATE,
            "leaf assignments not available: fit with compute_leaf_assignments=True");
}

void build_index(Ctx& c) {
    require_leaves(c);
    if (c.l_index) return;
    const size_t N = c.N, T = c.l_T, total = N * T;
    require(total < (size_t)INT32_MAX, RFX_ERR_UNSUPPORTED, "leaf index limited to 2^31 entries");
    require((size_t)T * (size_t)c.l_W < (size_t)UINT32_MAX, RFX_ERR_UNSUPPORTED, "too many trees");
    uint32_t* keys = (uint32_t*)c.l_keys.get(total * 8);  // keys in, then sorted keys
    uint32_t* skeys = keys + total;
    int* rows_in = (int*)c.l_q.get(total * 4);
    int* rows = (int*)c.l_rows.get(total * 4);
    const size_t groups = T * (size_t)c.l_W;
    int* gs = (int*)c.l_gs.get(groups * 4);
    int* ge = (int*)c.l_ge.get(groups * 4);
    cudaStream_t st = c.st;
    rfx::k_leaf_keys<<<grid_for((long long)total, 256, c.sm_count * 32), 256, 0, st>>>(
        (const int16_t*)c.l_leaf.p, (int)T, (int)N, c.l_W, keys, rows_in);
    RFX_LAUNCH("k_leaf_keys");
    int end_bit = 1;
    while (end_bit < 32 && ((size_t)1 << end_bit) < groups) ++end_bit;
    size_t tb = 0;
    RFX_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, keys, skeys, rows_in, rows, (int)total, 0,
                                             end_bit, st));
    void* tmp = c.l_cub.get(tb);
    RFX_CUDA(cub::DeviceRadixSort::SortPairs(tmp, tb, keys, skeys, rows_in, rows, (int)total, 0,
                                             end_bit, st));
    RFX_CUDA(cudaMemsetAsync(gs, 0, groups * 4, st));
    RFX_CUDA(cudaMemsetAsync(ge, 0, groups * 4, st));
    rfx::k_leaf_offsets<<<grid_for((long long)total, 256, c.sm_count * 32), 256, 0, st>>>(skeys, total, gs, ge);
    RFX_LAUNCH("k_leaf_offsets");
    RFX_CUDA(cudaStreamSynchronize(st));
    c.launches += 3;
    c.l_index = true;
}

// X_host [n][p] row-major -> device [p][n] in c.p_xc (through c.p_X).
float* upload_columns(Ctx& c, const float* X_host, int n, int p) {
    float* X = (float*)c.p_X.get((size_t)n * p * 4);
    float* xc = (float*)c.p_xc.get((size_t)n * p * 4);
    RFX_CUDA(cudaMemcpyAsync(X, X_host, (size_t)n * p * 4, cudaMemcpyHostToDevice, c.st));
    const dim3 grid((unsigned)((n + 31) / 32), (unsigned)((p + 31) / 32));
    rfx::k_transpose<<<grid, dim3(32, 8), 0, c.st>>>(X, n, p, xc);
    RFX_LAUNCH("k_transpose");
    return xc;
}

}  // namespace
}  // namespace rfxh

extern "C" {

int rfx_leaf_assignments(void* ctx, int16_t* out, int* ntree_out, int* nrows_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require_leaves(c);
        if (ntree_out) *ntree_out = c.l_T;
        if (nrows_out) *nrows_out = (int)c.N;
        if (out) {
            RFX_CUDA(cudaMemcpyAsync(out, c.l_leaf.p, (size_t)c.l_T * c.N * 2, cudaMemcpyDeviceToHost, c.st));
            RFX_CUDA(cudaStreamSynchronize(c.st));
        }
    });
}

int rfx_leaf_index(void* ctx) {
    return guarded([&] { build_index(*as_ctx(ctx)); });
}

int rfx_leaf_top_k_similar(void* ctx, const int* queries, int nq, int k, int exclude_self,
                           int* idx_out, float* sim_out, int* counts_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(nq >= 0 && k >= 0 && (nq == 0 || (queries && counts_out)), RFX_ERR_ARG, "bad arguments");
        require(nq == 0 || k == 0 || (idx_out && sim_out), RFX_ERR_ARG, "null outputs");
        build_index(c);
        const int N = (int)c.N;
        cudaStream_t st = c.st;
        const int QB = 64;  // queries per pass
        std::vector<int> valid, pos;
        for (int q = 0; q < nq; ++q) {
            counts_out[q] = 0;
            if (queries[q] >= 0 && queries[q] < N) {
                valid.push_back(queries[q]);
                pos.push_back(q);
            }
        }
        int* cnt = (int*)c.l_cnt.get((size_t)QB * N * 4);
        int* cidx = (int*)c.l_cidx.get((size_t)QB * N * 4);
        int* cval = (int*)c.l_cval.get((size_t)QB * N * 4);
        int* dq = (int*)c.l_nnz.get((size_t)QB * 3 * 4);
        int* nnz = dq + QB;
        int* noob = dq + 2 * QB;
        std::vector<int> hn(QB), ho(QB), hi, hv;
        for (size_t b0 = 0; b0 < valid.size(); b0 += QB) {
            const int nb = (int)std::min<size_t>(QB, valid.size() - b0);
            RFX_CUDA(cudaMemcpyAsync(dq, valid.data() + b0, (size_t)nb * 4, cudaMemcpyHostToDevice, st));
            RFX_CUDA(cudaMemsetAsync(cnt, 0, (size_t)nb * N * 4, st));
            rfx::k_leaf_query<<<(nb * 32 + 255) / 256, 256, 0, st>>>(
                (const int16_t*)c.l_leaf.p, (const uint32_t*)c.l_oob.p, c.l_words,
                (const int*)c.l_gs.p, (const int*)c.l_ge.p, (const int*)c.l_rows.p, N, c.l_T,
                c.l_W, dq, nb, exclude_self, cnt, noob);
            RFX_LAUNCH("k_leaf_query");
            rfx::k_leaf_compact<<<nb, 1024, 0, st>>>(cnt, N, cidx, cval, nnz);
            RFX_LAUNCH("k_leaf_compact");
            c.launches += 2;
            RFX_CUDA(cudaMemcpyAsync(hn.data(), nnz, (size_t)nb * 4, cudaMemcpyDeviceToHost, st));
            RFX_CUDA(cudaMemcpyAsync(ho.data(), noob, (size_t)nb * 4, cudaMemcpyDeviceToHost, st));
            RFX_CUDA(cudaStreamSynchronize(st));
            for (int qi = 0; qi < nb; ++qi) {
                const int q = pos[b0 + qi];
                if (ho[qi] == 0 || hn[qi] == 0 || k == 0) continue;
                hi.resize(hn[qi]);
                hv.resize(hn[qi]);
                RFX_CUDA(cudaMemcpyAsync(hi.data(), cidx + (size_t)qi * N, (size_t)hn[qi] * 4, cudaMemcpyDeviceToHost, st));
                RFX_CUDA(cudaMemcpyAsync(hv.data(), cval + (size_t)qi * N, (size_t)hn[qi] * 4, cudaMemcpyDeviceToHost, st));
                RFX_CUDA(cudaStreamSynchronize(st));
                // the reference's ranking: (index, count) in index order, partial_sort on count
                std::vector<std::pair<int, int>> ic(hn[qi]);
                for (int e = 0; e < hn[qi]; ++e) ic[e] = {hi[e], hv[e]};
                const int kk = std::min<int>(k, (int)ic.size());
                std::partial_sort(ic.begin(), ic.begin() + kk, ic.end(),
                                  [](const std::pair<int, int>& a, const std::pair<int, int>& b) {
                                      return a.second > b.second;
                                  });
                const float norm = 1.0f / (float)ho[qi];
                for (int e = 0; e < kk; ++e) {
                    idx_out[(size_t)q * k + e] = ic[e].first;
                    sim_out[(size_t)q * k + e] = (float)ic[e].second * norm;
                }
                counts_out[q] = kk;
            }
        }
    });
}

int rfx_leaf_proximity(void* ctx, int i, int j, float* out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(out != nullptr, RFX_ERR_ARG, "null output");
        require_leaves(c);
        *out = 0.0f;
        const int N = (int)c.N;
        if (i < 0 || i >= N || j < 0 || j >= N) return;
        int* d = (int*)c.l_out.get(16);
        rfx::k_leaf_pair<<<1, 32, 0, c.st>>>((const int16_t*)c.l_leaf.p, (const uint32_t*)c.l_oob.p,
                                            c.l_words, N, c.l_T, i, j, d);
        RFX_LAUNCH("k_leaf_pair");
        c.launches += 1;
        int h[2];
        RFX_CUDA(cudaMemcpyAsync(h, d, 8, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
        if (h[1] > 0) *out = (float)h[0] / (float)h[1];
    });
}

int rfx_predict_leaves(void* ctx, const float* X_host, int n, int p, int16_t* out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.f_T > 0, RFX_ERR_STATE, "no forest on the device (fit with keep_forest)");
        require(X_host && out && n >= 0 && p == c.f_p, RFX_ERR_ARG, "X must have the fit's feature count");
        if (n == 0) return;
        float* xc = upload_columns(c, X_host, n, p);
        int16_t* d = (int16_t*)c.l_f.get((size_t)n * c.f_T * 2);
        const dim3 grid((unsigned)((n + 255) / 256), (unsigned)c.f_T);
        rfx::k_leaf_predict<<<grid, 256, 0, c.st>>>((const rfx::PNode*)c.f_nodes.p, c.f_M, c.f_T, xc,
                                                   n, p, (const int*)c.f_cat.p, d);
        RFX_LAUNCH("k_leaf_predict");
        c.launches += 1;
        RFX_CUDA(cudaMemcpyAsync(out, d, (size_t)n * c.f_T * 2, cudaMemcpyDeviceToHost, c.st));
        RFX_CUDA(cudaStreamSynchronize(c.st));
    });
}

int rfx_predict_top_k_similar(void* ctx, const float* X_host, int n, int p, int k, int* idx_out,
                              float* sim_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.f_T > 0, RFX_ERR_STATE, "no forest on the device (fit with keep_forest)");
        build_index(c);
        require(c.f_T == c.l_T, RFX_ERR_STATE, "the device forest and the leaf store differ");
        const int N = (int)c.N, T = c.l_T;
        require(X_host && n >= 0 && p == c.f_p && k >= 0 && k <= N, RFX_ERR_ARG, "bad arguments (k <= training rows)");
        require(n == 0 || k == 0 || (idx_out && sim_out), RFX_ERR_ARG, "null outputs");
        if (n == 0 || k == 0) return;
        float* xc = upload_columns(c, X_host, n, p);
        int16_t* nl = (int16_t*)c.l_f.get((size_t)n * T * 2);
        const dim3 grid((unsigned)((n + 255) / 256), (unsigned)T);
        rfx::k_leaf_predict<<<grid, 256, 0, c.st>>>((const rfx::PNode*)c.f_nodes.p, c.f_M, T, xc, n,
                                                   p, (const int*)c.f_cat.p, nl);
        RFX_LAUNCH("k_leaf_predict");
        const int QB = 64;
        int* cnt = (int*)c.l_cnt.get((size_t)QB * N * 4);
        std::vector<int> hc((size_t)QB * N), order(N);
        std::vector<float> sims(N);
        for (int b0 = 0; b0 < n; b0 += QB) {
            const int nb = std::min(QB, n - b0);
            RFX_CUDA(cudaMemsetAsync(cnt, 0, (size_t)nb * N * 4, c.st));
            rfx::k_leaf_query_new<<<(nb * 32 + 255) / 256, 256, 0, c.st>>>(
                nl + (size_t)b0 * T, (const int*)c.l_gs.p, (const int*)c.l_ge.p,
                (const int*)c.l_rows.p, N, T, c.l_W, nb, cnt);
            RFX_LAUNCH("k_leaf_query_new");
            c.launches += 1;
            RFX_CUDA(cudaMemcpyAsync(hc.data(), cnt, (size_t)nb * N * 4, cudaMemcpyDeviceToHost, c.st));
            RFX_CUDA(cudaStreamSynchronize(c.st));
            for (int qi = 0; qi < nb; ++qi) {
                // similarity = (1.0f added per shared tree) / ntree, as the reference forms it;
                // then its partial_sort of every training row by similarity
                for (int i = 0; i < N; ++i) sims[i] = (float)hc[(size_t)qi * N + i] / (float)T;
                std::iota(order.begin(), order.end(), 0);
                std::partial_sort(order.begin(), order.begin() + k, order.end(),
                                  [&sims](int a, int b) { return sims[a] > sims[b]; });
                for (int e = 0; e < k; ++e) {
                    idx_out[(size_t)(b0 + qi) * k + e] = order[e];
                    sim_out[(size_t)(b0 + qi) * k + e] = sims[order[e]];
                }
            }
        }
        c.launches += 1;
    });
}

int rfx_leaf_select_anchors(void* ctx, int n_anchors, int method, uint32_t iseed, int* anchors_out,
                            int* count_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require_leaves(c);
        require(anchors_out && count_out && n_anchors >= 0 && (method == 0 || method == 1), RFX_ERR_ARG,
                "bad arguments");
        const int N = (int)c.N;
        std::vector<int> anchors;
        if (n_anchors >= N) {
            anchors.resize(N);
            std::iota(anchors.begin(), anchors.end(), 0);
        } else if (method == 1) {
            std::mt19937 rng(iseed);
            std::uniform_int_distribution<int> dist(0, N - 1);
            anchors.push_back(dist(rng));
            float* mn = (float*)c.l_out.get((size_t)N * 4 + (size_t)N + 64);
            uint8_t* taken = reinterpret_cast<uint8_t*>(mn + N);
            int* best = reinterpret_cast<int*>(taken + ((N + 15) / 16) * 16);
            std::vector<float> ones(N, 1.0f);
            RFX_CUDA(cudaMemcpyAsync(mn, ones.data(), (size_t)N * 4, cudaMemcpyHostToDevice, c.st));
            RFX_CUDA(cudaMemsetAsync(taken, 0, N, c.st));
            const uint8_t one = 1;
            RFX_CUDA(cudaMemcpyAsync(taken + anchors[0], &one, 1, cudaMemcpyHostToDevice, c.st));
            while ((int)anchors.size() < n_anchors) {
                rfx::k_anchor_update<<<(N + 255) / 256, 256, 0, c.st>>>(
                    (const int16_t*)c.l_leaf.p, c.l_T, N, anchors.back(), mn);
                rfx::k_anchor_pick<<<1, 1024, 0, c.st>>>(mn, taken, N, best);
                RFX_LAUNCH("outlier anchors");
                c.launches += 2;
                int b = -1;
                RFX_CUDA(cudaMemcpyAsync(&b, best, 4, cudaMemcpyDeviceToHost, c.st));
                RFX_CUDA(cudaStreamSynchronize(c.st));
                if (b < 0) break;
                anchors.push_back(b);
                RFX_CUDA(cudaMemcpyAsync(taken + b, &one, 1, cudaMemcpyHostToDevice, c.st));
            }
            RFX_CUDA(cudaStreamSynchronize(c.st));
        } else {
            std::vector<int> all(N);
            std::iota(all.begin(), all.end(), 0);
            std::mt19937 rng(iseed);
            std::shuffle(all.begin(), all.end(), rng);
            anchors.assign(all.begin(), all.begin() + n_anchors);
        }
        std::copy(anchors.begin(), anchors.end(), anchors_out);
        *count_out = (int)anchors.size();
        c.l_anchors = anchors;
    });
}

int rfx_leaf_outlier_scores(void* ctx, int mode, const int* anchors, int n_used, int n_anchors,
                            const int* labels, float* scores_out, float* raw_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(scores_out && (mode == 0 || mode == 1), RFX_ERR_ARG, "bad arguments");
        require(mode == 0 || (anchors && n_used >= 0), RFX_ERR_ARG, "greedy mode needs anchors");
        require_leaves(c);
        const int N = (int)c.N, T = c.l_T;
        cudaStream_t st = c.st;
        float* raw = (float*)c.l_out.get((size_t)N * 4 + 64);
        if (mode == 1) {
            int* da = (int*)c.l_q.get((size_t)std::max(1, n_used) * 4);
            if (n_used > 0) RFX_CUDA(cudaMemcpyAsync(da, anchors, (size_t)n_used * 4, cudaMemcpyHostToDevice, st));
            rfx::k_outlier_greedy<<<(N + 255) / 256, 256, 0, st>>>((const int16_t*)c.l_leaf.p, T, N, da,
                                                                  n_used, n_anchors, raw);
            RFX_LAUNCH("k_outlier_greedy");
        } else {
            build_index(c);
            // one count array of N ints per warp, at most 2 GiB in total
            const long long per = (long long)N * 4;
            const int warps = (int)std::max<long long>(32, std::min<long long>((long long)c.sm_count * 32,
                                                                              (2LL << 30) / per));
            const int blocks = (warps + 7) / 8;
            int* scratch = (int*)c.l_cnt.get((size_t)blocks * 8 * N * 4);
            RFX_CUDA(cudaMemsetAsync(scratch, 0, (size_t)blocks * 8 * N * 4, st));
            rfx::k_outlier_full<<<blocks, 256, 0, st>>>((const int16_t*)c.l_leaf.p, (const int*)c.l_gs.p,
                                                       (const int*)c.l_ge.p, (const int*)c.l_rows.p, N, T,
                                                       c.l_W, scratch, raw);
            RFX_LAUNCH("k_outlier_full");
        }
        c.launches += 1;
        std::vector<float> r(N);
        RFX_CUDA(cudaMemcpyAsync(r.data(), raw, (size_t)N * 4, cudaMemcpyDeviceToHost, st));
        RFX_CUDA(cudaStreamSynchronize(st));
        if (raw_out) std::copy(r.begin(), r.end(), raw_out);
        // normalisation (src/rf_random_forest.cpp:4201-4272): median and MAD, per class when
        // labels are given
        auto normalise = [&](const std::vector<int>& idx) {
            std::vector<float> v;
            v.reserve(idx.size());
            for (int i : idx) v.push_back(r[i]);
            std::vector<float> s = v;
            std::sort(s.begin(), s.end());
            const float median = s[s.size() / 2];
            std::vector<float> dev;
            dev.reserve(v.size());
            for (float x : v) dev.push_back(std::abs(x - median));
            std::sort(dev.begin(), dev.end());
            float mad = dev[dev.size() / 2];
            if (mad < 1e-10f) mad = 1.0f;
            for (size_t e = 0; e < idx.size(); ++e) scores_out[idx[e]] = (r[idx[e]] - median) / mad;
            return std::make_pair(median, mad);
        };
        c.l_norm.clear();
        if (labels) {
            std::map<int, std::vector<int>> by_class;
            for (int i = 0; i < N; ++i) by_class[labels[i]].push_back(i);
            for (auto& kv : by_class) c.l_norm[kv.first] = normalise(kv.second);
        } else {
            std::vector<int> all(N);
            std::iota(all.begin(), all.end(), 0);
            c.l_norm[-1] = normalise(all);
        }
    });
}

int rfx_predict_outlier_scores(void* ctx, const float* X_host, int n, int p, int mode,
                               int n_anchors, const int* classes, float* scores_out) {
    return guarded([&] {
        Ctx& c = *as_ctx(ctx);
        require(c.f_T > 0, RFX_ERR_STATE, "no forest on the device (fit with keep_forest)");
        require_leaves(c);
        require(!c.l_norm.empty(), RFX_ERR_STATE,
                "outlier normalisation not available: compute the training outlier scores first");
        build_index(c);
        require(c.f_T == c.l_T, RFX_ERR_STATE, "the device forest and the leaf store differ");
        require(X_host && scores_out && n >= 0 && p == c.f_p && (mode == 0 || mode == 1), RFX_ERR_ARG,
                "bad arguments");
        if (n == 0) return;
        const int N = (int)c.N, T = c.l_T;
        cudaStream_t st = c.st;
        float* xc = upload_columns(c, X_host, n, p);
        int16_t* nl = (int16_t*)c.l_f.get((size_t)n * T * 2);
        const dim3 grid((unsigned)((n + 255) / 256), (unsigned)T);
        rfx::k_leaf_predict<<<grid, 256, 0, st>>>((const rfx::PNode*)c.f_nodes.p, c.f_M, T, xc, n, p,
                                                 (const int*)c.f_cat.p, nl);
        RFX_LAUNCH("k_leaf_predict");
        const int QB = 64;
        int* cnt = (int*)c.l_cnt.get((size_t)QB * N * 4);
        int* hist = (int*)c.l_cidx.get((size_t)QB * (T + 1) * 4);
        float* raw = (float*)c.l_out.get((size_t)QB * 4 + 64);
        std::vector<float> r(n);
        for (int b0 = 0; b0 < n; b0 += QB) {
            const int nb = std::min(QB, n - b0);
            RFX_CUDA(cudaMemsetAsync(cnt, 0, (size_t)nb * N * 4, st));
            rfx::k_leaf_query_new<<<(nb * 32 + 255) / 256, 256, 0, st>>>(
                nl + (size_t)b0 * T, (const int*)c.l_gs.p, (const int*)c.l_ge.p,
                (const int*)c.l_rows.p, N, T, c.l_W, nb, cnt);
            if (mode == 1) {
                RFX_CUDA(cudaMemsetAsync(hist, 0, (size_t)nb * (T + 1) * 4, st));
                rfx::k_outlier_new_hist<<<dim3((unsigned)std::min(64, (N + 255) / 256), (unsigned)nb), 256, 0, st>>>(
                    cnt, N, T, nb, hist);
            }
            rfx::k_outlier_new<<<(nb + 63) / 64, 64, 0, st>>>(cnt, hist, N, T, nb, mode, n_anchors, raw);
            RFX_LAUNCH("new-row outlier kernels");
            c.launches += mode == 1 ? 3 : 2;
            RFX_CUDA(cudaMemcpyAsync(r.data() + b0, raw, (size_t)nb * 4, cudaMemcpyDeviceToHost, st));
        }
        RFX_CUDA(cudaStreamSynchronize(st));
        c.launches += 1;
        // the training statistics: per predicted class for a classifier, else over all rows
        for (int s = 0; s < n; ++s) {
            const int key = classes ? classes[s] : -1;
            auto it = c.l_norm.find(key);
            const float median = it != c.l_norm.end() ? it->second.first : 0.0f;
            const float mad = it != c.l_norm.end() ? it->second.second : 1.0f;
            scores_out[s] = (r[s] - median) / mad;
        }
    });
}

int rfx_rank_scores_desc(const float* scores, int n, int k, int* idx_out, float* val_out) {
    return guarded([&] {
        require(n >= 0 && k >= 0 && (n == 0 || scores) && (k == 0 || (idx_out && val_out)), RFX_ERR_ARG,
                "bad arguments");
        std::vector<std::pair<int, float>> v(n);
        for (int i = 0; i < n; ++i) v[i] = {i, scores[i]};
        std::sort(v.begin(), v.end(),
                  [](const std::pair<int, float>& a, const std::pair<int, float>& b) { return a.second > b.second; });
        const int kk = std::min(k, n);
        for (int e = 0; e < kk; ++e) {
            idx_out[e] = v[e].first;
            val_out[e] = v[e].second;
        }
    });
}

}  // extern "C"
