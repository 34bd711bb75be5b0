// Proximity imputation round (the loop body of rfx_impute_proximity,
// python/rfx_impute.py:730-775), bit for bit, for every aggregation and top_k.
//
// For a missing cell (i, j) the reference takes the finishprox'd proximity row i as float32,
// zeroes the row's own entry and the rows missing in column j, keeps the rows with positive
// proximity (ascending), and
//   continuous:  w = p / sum(p);  x_ij = sum(w * x_kj)       (float32 throughout)
//   categorical: x_ij = the value v (ascending, first maximum) with the largest sum(p[x == v])
// where every sum is numpy's pairwise float32 summation (blocks of <= 128 elements summed with
// 8 accumulators, longer ranges split in halves rounded down to a multiple of 8).  Cells of
// one round are independent (a cell reads only rows observed in its column).  A row's cells
// share its proximity row, so each warp takes one row and reads that row once; per cell it
// compacts the selected (p, x) pairs into its scratch in index order, the lanes sum the
// leaves of the pairwise tree, and lane 0 combines them in the tree's order.
//
// top_k (rfx_impute.py:744-748): when more rows qualify, only the top_k by proximity are kept,
// in ascending (proximity, row) order -- the stable order; the reference's np.argsort leaves
// the order of equal proximities to numpy's sort implementation.  A radix select over the
// proximity bits finds the k-th value, the rows above it and the last rows equal to it are
// kept, and each kept pair is placed by counting the kept pairs before it.
// median (rfx_impute.py:754-762): np.median of the values (the middle one, or the float32
// mean of the two middle ones, both found by radix select); categorical: the value that
// occurs most often (ascending values, first maximum).
#include <cuda_runtime.h>
#include <cstdint>

#include "rfx_impute.h"

namespace rfx {

namespace {

constexpr int kLeafMax = 128;

// Element sources for the sums.  Buffers start on 16 bytes and every leaf of the pairwise
// tree starts on a multiple of 8 elements, so a leaf's groups of 8 load as two float4.
struct Plain {
    const float* a;
    __device__ float at(int i) const { return a[i]; }
    __device__ void at8(int i, float (&x)[8]) const {
        const float4 u = *reinterpret_cast<const float4*>(a + i);
        const float4 v = *reinterpret_cast<const float4*>(a + i + 4);
        x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
        x[4] = v.x; x[5] = v.y; x[6] = v.z; x[7] = v.w;
    }
};

// (w[i] / tot) * v[i]: the normalised weight times the value, as the reference forms it
struct Scaled {
    const float* w;
    const float* v;
    float tot;
    __device__ float at(int i) const { return (w[i] / tot) * v[i]; }
    __device__ void at8(int i, float (&x)[8]) const {
        float a[8], b[8];
        Plain{w}.at8(i, a);
        Plain{v}.at8(i, b);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = (a[k] / tot) * b[k];
    }
};

// numpy's pairwise sum of one leaf [lo, lo + n), n <= 128: n < 8 sequentially from 0,
// otherwise eight strided accumulators, combined ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then
// the tail.
template <class F>
__device__ float leaf_sum(const F& f, int lo, int n) {
    if (n < 8) {
        float r = 0.0f;
        for (int i = 0; i < n; ++i) r += f.at(lo + i);
        return r;
    }
    float r[8];
    f.at8(lo, r);
    int i = 8;
    const int n8 = n - (n % 8);
    for (; i + 8 < n8; i += 16) {  // two groups in flight
        float x[8], y[8];
        f.at8(lo + i, x);
        f.at8(lo + i + 8, y);
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] = (r[k] + x[k]) + y[k];
    }
    for (; i < n8; i += 8) {
        float x[8];
        f.at8(lo + i, x);
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] += x[k];
    }
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += f.at(lo + i);
    return res;
}

// Leaves of the pairwise tree of [lo, lo + len) in left-to-right order (numpy's splitting
// rule: ranges above 128 split at half rounded down to a multiple of 8).
__device__ void pairwise_leaves(int lo, int len, int2* leaves, int& cnt) {
    if (len <= kLeafMax) {
        leaves[cnt++] = make_int2(lo, len);
        return;
    }
    int n2 = len / 2;
    n2 -= n2 % 8;
    pairwise_leaves(lo, n2, leaves, cnt);
    pairwise_leaves(lo + n2, len - n2, leaves, cnt);
}

// The leaf sums combined in the same tree: sum(left half) + sum(right half).
__device__ float pairwise_combine(int len, const float* leafsum, int& leaf) {
    if (len <= kLeafMax) return leafsum[leaf++];
    int n2 = len / 2;
    n2 -= n2 % 8;
    const float l = pairwise_combine(n2, leafsum, leaf);
    const float r = pairwise_combine(len - n2, leafsum, leaf);
    return l + r;
}

// Pairwise sum of f over [0, n) by one warp (leaves by the lanes, combination by lane 0).
// `fresh` = false reuses the leaf list of the previous call of the same n.
template <class F>
__device__ float warp_pairwise(const F& f, int n, int2* leaves, float* leafsum, int lane,
                               bool fresh = true) {
    float r = 0.0f;
    if (n <= kLeafMax) {
        if (lane == 0) r = leaf_sum(f, 0, n);
        return __shfl_sync(0xffffffffu, r, 0);
    }
    if (fresh && lane == 0) {
        int cnt = 0;
        pairwise_leaves(0, n, leaves, cnt);
        leaves[kImpLeafCountSlot].x = cnt;
    }
    __syncwarp();
    const int nl = leaves[kImpLeafCountSlot].x;
    for (int l = lane; l < nl; l += 32) leafsum[l] = leaf_sum(f, leaves[l].x, leaves[l].y);
    __syncwarp();
    if (lane == 0) {
        int leaf = 0;
        r = pairwise_combine(n, leafsum, leaf);
    }
    return __shfl_sync(0xffffffffu, r, 0);
}

// Order-preserving key of a float (a larger float has a larger key; -0 counts as +0, so a
// zero median is +0) and its inverse.
__device__ __forceinline__ uint32_t fkey(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u << 1) == 0u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Key of rank r (0 = largest) among the keys of src[0, m) by one warp: four 8-bit radix
// passes over the keys that share the digits found so far, with the warp's 256-bin
// histogram in shared memory.  *above = keys strictly larger than the result.
__device__ uint32_t warp_select_desc(const float* src, int m, int r, unsigned* hist, int lane,
                                     int* above) {
    uint32_t prefix = 0, mask = 0;
    int need = r, ab = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (int q = lane; q < m; q += 32) {
            const uint32_t k = fkey(src[q]);
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncwarp();
        // lane l holds bins 255 - 8l down to 248 - 8l; counts from the top
        unsigned c[8], tot = 0;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            c[t] = hist[255 - 8 * lane - t];
            tot += c[t];
        }
        unsigned incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const unsigned excl = incl - tot;
        const bool mine = excl <= (unsigned)need && (unsigned)need < incl;
        const unsigned bal = __ballot_sync(0xffffffffu, mine);
        int digit = 0;
        unsigned before = 0;
        if (mine) {
            unsigned acc = excl;
            for (int t = 0; t < 8; ++t) {
                if ((unsigned)need < acc + c[t]) {
                    digit = 255 - 8 * lane - t;
                    before = acc;
                    break;
                }
                acc += c[t];
            }
        }
        const int owner = __ffs(bal) - 1;
        digit = __shfl_sync(0xffffffffu, digit, owner);
        before = __shfl_sync(0xffffffffu, before, owner);
        need -= (int)before;
        ab += (int)before;
        prefix |= (uint32_t)digit << shift;
        mask |= 255u << shift;
        __syncwarp();
    }
    *above = ab;
    return prefix;
}

}  // namespace

// One warp per row that has missing cells (grid-stride over rows).  The warp first compacts
// the row's usable neighbours (k != i, proximity > 0; ascending k) from the finished
// proximity row, then serves each of the row's cells from that short list: it drops the
// neighbours missing in the cell's column (order kept) and aggregates.  S: finished
// proximity rows [r0, r0 + rows) of width n (row stride ldS); xc: current values [p][n];
// miss: [p][n] 1 = missing; rows/row_cells: the rows of this block and their ranges of
// cells; out[c]: new value, or NaN when the cell has no usable neighbour (the reference
// leaves it unchanged).
__global__ void __launch_bounds__(256, 4) k_impute(ImputeArgs a) {
    constexpr int U = 8;  // row chunks of 32 in flight per lane
    constexpr int V = 4;  // neighbour chunks of 32 in flight per lane
    const int lane = threadIdx.x & 31;
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const int n = a.n;
    const int nn = impute_row_floats(n);
    float* base = a.scratch + (size_t)wid * a.scratch_stride;
    int* ridx = reinterpret_cast<int*>(base);  // neighbours of the row: index, proximity
    float* rs = base + nn;
    float* wbuf = rs + nn;                      // the cell's selection: weight, value
    float* vbuf = wbuf + nn;
    float* tbuf = vbuf + nn;                    // per-category subsequence
    float* selw = tbuf + nn;                    // the top_k selection in row order
    float* selv = selw + nn;
    int2* leaves = reinterpret_cast<int2*>(selv + nn) + 1;  // [-1] carries the leaf count
    __shared__ unsigned s_hist[8][256];
    unsigned* hist = s_hist[threadIdx.x >> 5];
    float* leafsum = reinterpret_cast<float*>(leaves + a.max_leaves + 1);
    const unsigned lt = (1u << lane) - 1u;
    for (int r = wid; r < a.nrows; r += nwarps) {
        const int i = a.rows[r];
        long long tp = clock64();
        const float* srow = a.S + (size_t)(i - a.r0) * a.ldS;
        int m = 0;
        for (int k0 = 0; k0 < n; k0 += 32 * U) {
            float s[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k = k0 + u * 32 + lane;
                s[u] = k < n ? __ldcs(srow + k) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k = k0 + u * 32 + lane;
                const bool sel = s[u] > 0.0f && k != i;
                const unsigned bal = __ballot_sync(0xffffffffu, sel);
                if (sel) {
                    const int pos = m + __popc(bal & lt);
                    ridx[pos] = k;
                    rs[pos] = s[u];
                }
                m += __popc(bal);
            }
        }
        __syncwarp();
        if (a.prof && lane == 0) {
            atomicAdd(a.prof + 0, (unsigned long long)m);
            atomicMax(a.prof + 7, (unsigned long long)m);
            atomicAdd(a.prof + 2, (unsigned long long)(clock64() - tp));
        }
        for (int c = a.row_cells[r]; c < a.row_cells[r + 1]; ++c) {
            tp = clock64();
            const int j = a.cells[2 * c + 1];
            const uint8_t* mj = a.miss + (size_t)j * n;
            const float* xj = a.xc + (size_t)j * n;
            int mm = 0;
            for (int t0 = 0; t0 < m; t0 += 32 * V) {
                int k[V];
                bool sel[V];
                float sv[V], xv[V];
#pragma unroll
                for (int u = 0; u < V; ++u) {
                    const int t = t0 + u * 32 + lane;
                    k[u] = t < m ? ridx[t] : -1;
                }
#pragma unroll
                for (int u = 0; u < V; ++u) sel[u] = k[u] >= 0 && !mj[k[u]];
#pragma unroll
                for (int u = 0; u < V; ++u) {
                    const int t = t0 + u * 32 + lane;
                    sv[u] = sel[u] ? rs[t] : 0.0f;
                    xv[u] = sel[u] ? xj[k[u]] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < V; ++u) {
                    const unsigned bal = __ballot_sync(0xffffffffu, sel[u]);
                    if (sel[u]) {
                        const int pos = mm + __popc(bal & lt);
                        wbuf[pos] = sv[u];
                        vbuf[pos] = xv[u];
                    }
                    mm += __popc(bal);
                }
            }
            __syncwarp();
            if (a.prof && lane == 0) {
                atomicAdd(a.prof + 1, (unsigned long long)mm);
                atomicAdd(a.prof + 3, (unsigned long long)(clock64() - tp));
                tp = clock64();
            }
            if (mm > 0 && a.top_k >= 0 && mm > a.top_k) {
                // the top kk by (proximity, row), placed in ascending order
                const int kk = a.top_k == 0 ? mm : a.top_k;
                int above;
                const uint32_t K = warp_select_desc(wbuf, mm, kk - 1, hist, lane, &above);
                int eqc = 0;
                for (int q = lane; q < mm; q += 32) eqc += fkey(wbuf[q]) == K ? 1 : 0;
                for (int o = 16; o > 0; o >>= 1) eqc += __shfl_xor_sync(0xffffffffu, eqc, o);
                const int skip = eqc - (kk - above);  // the first rows equal to the k-th drop
                int ms = 0, eqseen = 0;
                for (int q0 = 0; q0 < mm; q0 += 32) {
                    const int q = q0 + lane;
                    const uint32_t key = q < mm ? fkey(wbuf[q]) : 0u;
                    const bool eq = q < mm && key == K;
                    const unsigned beq = __ballot_sync(0xffffffffu, eq);
                    const bool keep = q < mm && (key > K || (eq && eqseen + __popc(beq & lt) >= skip));
                    const unsigned bk = __ballot_sync(0xffffffffu, keep);
                    if (keep) {
                        selw[ms + __popc(bk & lt)] = wbuf[q];
                        selv[ms + __popc(bk & lt)] = vbuf[q];
                    }
                    ms += __popc(bk);
                    eqseen += __popc(beq);
                }
                __syncwarp();
                for (int t = lane; t < kk; t += 32) {
                    const float wt = selw[t];
                    int rank = 0;
                    for (int u = 0; u < kk; ++u) {
                        const float wu = selw[u];
                        rank += (wu < wt || (wu == wt && u < t)) ? 1 : 0;
                    }
                    wbuf[rank] = wt;
                    vbuf[rank] = selv[t];
                }
                __syncwarp();
                mm = kk;
            }
            float result = __int_as_float(0x7fc00000);
            if (mm > 0 && a.median && !a.is_cat[j]) {
                int above;
                if (mm & 1) {
                    result = fkey_inv(warp_select_desc(vbuf, mm, (mm - 1) / 2, hist, lane, &above));
                } else {
                    const float hi = fkey_inv(warp_select_desc(vbuf, mm, mm / 2 - 1, hist, lane, &above));
                    const float lo = fkey_inv(warp_select_desc(vbuf, mm, mm / 2, hist, lane, &above));
                    result = (lo + hi) / 2.0f;
                }
            } else if (mm > 0) {
                if (!a.is_cat[j]) {
                    const float tot = warp_pairwise(Plain{wbuf}, mm, leaves, leafsum, lane);
                    result = warp_pairwise(Scaled{wbuf, vbuf, tot}, mm, leaves, leafsum, lane, false);
                } else {
                    // distinct values ascending; weight of each = pairwise sum of its subsequence
                    float prev = -__int_as_float(0x7f800000);
                    bool first = true;
                    float best = 0.0f, best_v = 0.0f;
                    for (;;) {
                        float nxt = __int_as_float(0x7f800000);
                        for (int q = lane; q < mm; q += 32) {
                            const float v = vbuf[q];
                            if ((first || v > prev) && v < nxt) nxt = v;
                        }
                        for (int o = 16; o > 0; o >>= 1) nxt = fminf(nxt, __shfl_xor_sync(0xffffffffu, nxt, o));
                        bool any = false;
                        for (int q = lane; q < mm; q += 32) any |= vbuf[q] == nxt;
                        if (!__any_sync(0xffffffffu, any)) break;
                        int mc = 0;
                        for (int q0 = 0; q0 < mm; q0 += 32) {
                            const int q = q0 + lane;
                            const bool selc = q < mm && vbuf[q] == nxt;
                            const unsigned bal = __ballot_sync(0xffffffffu, selc);
                            if (selc) tbuf[mc + __popc(bal & lt)] = wbuf[q];
                            mc += __popc(bal);
                        }
                        __syncwarp();
                        const float cntw = a.median ? (float)mc
                                                    : warp_pairwise(Plain{tbuf}, mc, leaves, leafsum, lane);
                        if (first || cntw > best) {
                            best = cntw;
                            best_v = nxt;
                        }
                        first = false;
                        prev = nxt;
                        if (a.prof && lane == 0) atomicAdd(a.prof + 6, 1ull);
                    }
                    result = best_v;
                }
            }
            if (a.prof && lane == 0) {
                const int cat = a.is_cat[j] ? 1 : 0;
                atomicAdd(a.prof + 4 + cat, (unsigned long long)(clock64() - tp));
                atomicAdd(a.prof + 8 + cat, 1ull);
            }
            if (lane == 0) a.out[c] = result;
            __syncwarp();
        }
    }
}

}  // namespace rfx
