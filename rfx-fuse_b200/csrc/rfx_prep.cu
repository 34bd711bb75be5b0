// Input preparation on the device: column transpose, quantile binning, packed rows,
// bootstrap weights, the importance permutation, per-tree bootstrap and in/out-of-bag lists.
#include "rfx_device.cuh"
#include "rfx_kernels.h"

namespace rfx {

// ---------------------------------------------------------------------------------------
// X row-major [N][p] -> xc column-major [p][N] (32x32 tiles through shared memory).
// ---------------------------------------------------------------------------------------
__global__ void k_transpose(const float* __restrict__ X, int N, int p, float* __restrict__ xc) {
    __shared__ float tile[32][33];
    const int r0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int r = r0 + k, c = c0 + threadIdx.x;
        if (r < N && c < p) tile[k][threadIdx.x] = X[(size_t)r * p + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int c = c0 + k, r = r0 + threadIdx.x;
        if (r < N && c < p) xc[(size_t)c * N + r] = tile[threadIdx.x][k];
    }
}

// ---------------------------------------------------------------------------------------
// Per-column sort of the raw values (stable LSD radix sort on order-preserving 32-bit keys,
// 8-bit digits, one 1024-thread block per column).  Only the sorted values are used (for
// the unique values of compute_bin_edges_quantile, src/rf_histogram.cpp:60-77), so equal
// keys are interchangeable; stability is what makes the LSD passes correct.
// ---------------------------------------------------------------------------------------
constexpr int kSortThreads = 1024;

__global__ void __launch_bounds__(kSortThreads)
k_sort_columns(const float* __restrict__ xc, int N, const int* __restrict__ cat,
               uint32_t* __restrict__ ka, uint32_t* __restrict__ kb) {
    __shared__ int wcnt[32][kBins];
    __shared__ int base[kBins];
    const int f = blockIdx.x;
    if (cat[f] > 2) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float* col = xc + (size_t)f * N;
    uint32_t* A = ka + (size_t)f * N;
    uint32_t* B = kb + (size_t)f * N;
    for (int k = tid; k < 32 * kBins; k += kSortThreads) (&wcnt[0][0])[k] = 0;
    const uint32_t lt = (1u << lane) - 1u;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 8 * pass;
        const uint32_t* src = pass == 0 ? nullptr : (pass & 1 ? A : B);
        uint32_t* dst = pass & 1 ? B : A;
        if (tid < kBins) base[tid] = 0;
        __syncthreads();
        for (int i = tid; i < N; i += kSortThreads) {
            const uint32_t key = src ? src[i] : ord_of(col[i]);
            atomicAdd(&base[(key >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int run = 0;
            for (int d = 0; d < kBins; ++d) { const int c = base[d]; base[d] = run; run += c; }
        }
        __syncthreads();
        for (int t0 = 0; t0 < N; t0 += kSortThreads) {
            const int i = t0 + tid;
            const bool valid = i < N;
            const uint32_t key = valid ? (src ? src[i] : ord_of(col[i])) : 0u;
            const int d = valid ? (int)((key >> shift) & 255u) : kBins;
            const uint32_t peers = __match_any_sync(kFull, d);
            const int rank = __popc(peers & lt);
            if (valid && rank == 0) wcnt[warp][d] = __popc(peers);
            __syncthreads();
            if (tid < kBins) {
                int run = base[tid];
                for (int w = 0; w < 32; ++w) { const int c = wcnt[w][tid]; wcnt[w][tid] = run; run += c; }
                base[tid] = run;
            }
            __syncthreads();
            if (valid) dst[wcnt[warp][d] + rank] = key;
            __syncthreads();
            if (tid < kBins)
                for (int w = 0; w < 32; ++w) wcnt[w][tid] = 0;
            __syncthreads();
        }
    }
}

// ---------------------------------------------------------------------------------------
// Unique values and bin edges per column: compute_bin_edges_quantile,
// src/rf_histogram.cpp:36-128.  Sorted keys in `sorted`; unique values compacted into
// `uniq` (same shape).  One block per column.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
k_edges(const uint32_t* __restrict__ sorted, int N, const int* __restrict__ cat, int nbins,
        float* __restrict__ uniq, float* __restrict__ edges, int* __restrict__ nb,
        int* __restrict__ kind) {
    __shared__ int woff[32];
    __shared__ int carry;
    const int f = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* e = edges + (size_t)f * 257;
    if (cat[f] > 2) {
        if (tid == 0) { nb[f] = cat[f]; kind[f] = 2; }
        for (int b = tid; b < 257; b += blockDim.x) e[b] = 0.0f;
        return;
    }
    const uint32_t* s = sorted + (size_t)f * N;
    float* u = uniq + (size_t)f * N;
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int t0 = 0; t0 < N; t0 += blockDim.x) {
        const int i = t0 + tid;
        bool flag = false;
        float v = 0.0f;
        if (i < N) {
            v = float_of(s[i]);
            flag = (i == 0) || (v != float_of(s[i - 1]));
        }
        const uint32_t bal = __ballot_sync(kFull, flag);
        if (lane == 0) woff[warp] = __popc(bal);
        __syncthreads();
        if (tid == 0) {
            int run = carry;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { const int c = woff[w]; woff[w] = run; run += c; }
            carry = run;
        }
        __syncthreads();
        if (flag) u[woff[warp] + __popc(bal & ((1u << lane) - 1u))] = v;
        __syncthreads();
    }
    if (tid != 0) return;
    const int nu = carry;
    if (nu <= 2) {
        const float lo = u[0], hi = u[nu - 1];
        e[0] = lo - 1.0f;
        e[1] = (lo + hi) / 2.0f;
        e[2] = hi + 1.0f;
        for (int b = 3; b <= 256; ++b) e[b] = e[2];
        nb[f] = 2;
        kind[f] = 1;
        return;
    }
    const int ab = min(nbins, nu);
    e[0] = u[0] - 1.0f;
    for (int b = 1; b <= ab; ++b) {
        int q = (b * nu) / ab;
        if (q >= nu) q = nu - 1;
        e[b] = u[q];
    }
    for (int b = ab + 1; b <= 256; ++b) e[b] = e[ab];
    for (int b = 1; b <= ab; ++b)
        if (e[b] <= e[b - 1]) e[b] = e[b - 1] + 1e-7f;
    nb[f] = ab;
    kind[f] = 0;
}

// find_bin: src/rf_histogram.cpp:13-31.
__device__ __forceinline__ int find_bin(float v, const float* e, int nb) {
    if (v <= e[0]) return 0;
    if (v >= e[nb]) return nb - 1;
    int lo = 0, hi = nb;
    while (lo < hi) {
        const int mid = (lo + hi) / 2;
        if (v < e[mid]) hi = mid; else lo = mid + 1;
    }
    return max(0, lo - 1);
}

// Packed rows [N][rs]: bin_data_cpu (src/rf_histogram.cpp:134-160) for every feature,
// then the target at byte `ro`.  One thread per (row, feature), features fastest.
__global__ void k_pack_rows(Data D) {
    const long long total = (long long)D.N * D.p;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < total;
         k += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(k / D.p), f = (int)(k % D.p);
        const float v = D.xc[(size_t)f * D.N + i];
        const float* e = D.edges + (size_t)f * 257;
        const int kd = D.kind[f], nbf = D.nb[f];
        int b;
        if (kd == 2) {
            int c = (int)(v + 0.5f);
            b = max(0, min(c, nbf - 1));
        } else if (kd == 1) {
            b = v > e[1] ? 1 : 0;
        } else {
            b = find_bin(v, e, nbf);
        }
        uint8_t* row = const_cast<uint8_t*>(D.rows) + (size_t)i * D.rs;
        row[f] = (uint8_t)b;
        if (f == 0) {
            if (D.nclass == 1) {
                const float val = D.yv[i];
                *reinterpret_cast<float2*>(row + D.ro) = make_float2(val, val * val);
            } else {
                *reinterpret_cast<int*>(row + D.ro) = D.lab[i];
            }
        }
    }
}

// Regression targets: lab = (int)(y * 1000.0f), yv = (float)lab / 1000.0f
// (src/rf_random_forest.cpp:1356-1364, src/rf_growtree.cpp:741-751).
__global__ void k_regr_targets(const float* __restrict__ y, int N, int* __restrict__ lab,
                               float* __restrict__ yv) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) {
        const int q = (int)(y[i] * 1000.0f);
        lab[i] = q;
        yv[i] = (float)q / 1000.0f;
    }
}

// Running float sum of the bootstrap weights in row order (src/rf_bootstrap.cpp:31-37).
__global__ void k_cumw(const float* __restrict__ w, int N, float* __restrict__ cum,
                       float* __restrict__ total) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    float t = 0.0f;
    for (int i = 0; i < N; ++i) { t += w[i]; cum[i] = t; }
    *total = t;
}

// Fisher-Yates permutation of PreShuffledPermutation::initialize (src/rf_varimp.cpp:45-61):
// MT19937(seed); for j = N-1..1: k = (int)(randomu() * (j+1)), clamp, swap.  The block
// generates the swap targets in parallel; one thread then applies the swaps in order.
__global__ void __launch_bounds__(256)
k_permutation(int N, uint32_t seed, int* __restrict__ ks, int* __restrict__ perm) {
    __shared__ uint32_t s[624];
    if (threadIdx.x == 0) mt_seed_serial(s, seed);
    for (int i = threadIdx.x; i < N; i += blockDim.x) perm[i] = i;
    __syncthreads();
    mt_generate(s, 624, (long long)max(N - 1, 0), [&](long long d, uint32_t y) {
        const int j = N - 1 - (int)d;
        int k = (int)(mt_uniform(y) * (float)(j + 1));
        if (k > j) k = j;
        ks[d] = k;
    });
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int d = 0; d < N - 1; ++d) {
        const int j = N - 1 - d, k = ks[d];
        const int a = perm[j];
        perm[j] = perm[k];
        perm[k] = a;
    }
}

// ---------------------------------------------------------------------------------------
// Bootstrap of every tree in the batch: cpu_bootstrap, src/rf_bootstrap.cpp:15-84.  Tree
// t draws N uniforms from MT19937(boot_seed + tree0 + t); draw i -> row (int)(u * N), or
// the first row whose running weight is >= u * total when weights are given.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_bootstrap(Data D, Batch B) {
    __shared__ uint32_t s[624];
    const int t = blockIdx.x;
    if (threadIdx.x == 0) mt_seed_serial(s, (uint32_t)(B.boot_seed + B.tree0 + t));
    __syncthreads();
    int* nin = B.nin + (size_t)t * D.N;
    const int N = D.N;
    const float* cw = D.cumw;
    const float tot = D.totw;
    mt_generate(s, 624, (long long)N, [&](long long, uint32_t y) {
        const float u = mt_uniform(y);
        int i;
        if (cw) {
            const float target = u * tot;
            int lo = 0, hi = N;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (cw[mid] < target) lo = mid + 1; else hi = mid;
            }
            i = lo >= N ? N - 1 : lo;
        } else {
            i = (int)(u * (float)N);
            if (i >= N) i = N - 1;
            if (i < 0) i = 0;
        }
        atomicAdd(&nin[i], 1);
    });
}

// In-bag (ascending, distinct) and out-of-bag row lists of every tree, the root node, and
// the grower's MT19937(iseed + tree) state.
__global__ void __launch_bounds__(1024) k_compact(Data D, Batch B) {
    __shared__ int win[32], wout[32];
    __shared__ int cin, cout_;
    __shared__ uint32_t s[624];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = D.N;
    const int* nin = B.nin + (size_t)t * N;
    int* inb = B.seg[0] + (size_t)t * N;
    int* oob = B.oob + (size_t)t * N;
    if (tid == 0) { cin = 0; cout_ = 0; mt_seed_serial(s, (uint32_t)(B.iseed + B.tree0 + t)); }
    __syncthreads();
    const uint32_t lt = (1u << lane) - 1u;
    for (int t0 = 0; t0 < N; t0 += blockDim.x) {
        const int i = t0 + tid;
        const bool valid = i < N;
        const bool in = valid && nin[i] > 0;
        const bool out = valid && !in;
        const uint32_t bi = __ballot_sync(kFull, in), bo = __ballot_sync(kFull, out);
        if (lane == 0) { win[warp] = __popc(bi); wout[warp] = __popc(bo); }
        __syncthreads();
        if (tid == 0) {
            int ri = cin, ro = cout_;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                const int a = win[w], b = wout[w];
                win[w] = ri; wout[w] = ro; ri += a; ro += b;
            }
            cin = ri; cout_ = ro;
        }
        __syncthreads();
        if (in) inb[win[warp] + __popc(bi & lt)] = i;
        if (out) oob[wout[warp] + __popc(bo & lt)] = i;
        __syncthreads();
    }
    uint32_t* g = B.mt + (size_t)t * 624;
    for (int k = tid; k < 624; k += blockDim.x) g[k] = s[k];
    if (tid == 0) {
        B.ninbag[t] = cin;
        B.noob[t] = cout_;
        B.mt_pos[t] = 624;
        const size_t m0 = (size_t)t * B.M;
        B.nd_start[m0] = 0;
        B.nd_cnt[m0] = cin;
        B.status[m0] = 2;
        B.lvl_lo[t] = 0;
        B.lvl_hi[t] = 1;
        B.nxt_lo[t] = 0;
        B.nxt_hi[t] = 1;
        B.nnode[t] = 1;
    }
}

}  // namespace rfx
