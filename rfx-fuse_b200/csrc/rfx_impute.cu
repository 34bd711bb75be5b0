// Proximity-weighted imputation round (the loop body of rfx_impute_proximity,
// python/rfx_impute.py:730-775, aggregation 'mean', top_k None), bit for bit.
//
// For a missing cell (i, j) the reference takes the finishprox'd proximity row i as float32,
// zeroes the row's own entry and the rows missing in column j, keeps the rows with positive
// proximity (ascending), and
//   continuous:  w = p / sum(p);  x_ij = sum(w * x_kj)       (float32 throughout)
//   categorical: x_ij = the value v (ascending, first maximum) with the largest sum(p[x == v])
// where every sum is numpy's pairwise float32 summation (blocks of <= 128 elements summed with
// 8 accumulators, longer ranges split in halves rounded down to a multiple of 8).  Cells of
// one round are independent (a cell reads only rows observed in its column), so each warp
// takes one cell: it compacts the selected (p, x) pairs into its scratch in index order, the
// lanes sum the leaves of the pairwise tree, and lane 0 combines them in the tree's order.
#include <cuda_runtime.h>
#include <cstdint>

#include "rfx_impute.h"

namespace rfx {

namespace {

constexpr int kLeafMax = 128;

// numpy's pairwise sum of one leaf (n <= 128): n < 8 sequentially from 0, otherwise eight
// strided accumulators, combined ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the tail.
__device__ float leaf_sum(const float* a, int n) {
    if (n < 8) {
        float r = 0.0f;
        for (int i = 0; i < n; ++i) r += a[i];
        return r;
    }
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = a[k];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] += a[i + k];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += a[i];
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

// Pairwise sum of buf[0, n) by one warp (leaves by the lanes, combination by lane 0).
__device__ float warp_pairwise(const float* buf, int n, int2* leaves, float* leafsum, int lane) {
    float r = 0.0f;
    if (n <= kLeafMax) {
        if (lane == 0) r = leaf_sum(buf, n);
        return __shfl_sync(0xffffffffu, r, 0);
    }
    if (lane == 0) {
        int cnt = 0;
        pairwise_leaves(0, n, leaves, cnt);
        leaves[kImpLeafCountSlot].x = cnt;
    }
    __syncwarp();
    const int nl = leaves[kImpLeafCountSlot].x;
    for (int l = lane; l < nl; l += 32) leafsum[l] = leaf_sum(buf + leaves[l].x, leaves[l].y);
    __syncwarp();
    if (lane == 0) {
        int leaf = 0;
        r = pairwise_combine(n, leafsum, leaf);
    }
    return __shfl_sync(0xffffffffu, r, 0);
}

}  // namespace

// One warp per missing cell (grid-stride).  S: finished proximity rows [r0, r0 + rows) of
// width n (row stride ldS); xc: current values [p][n]; miss: [p][n] 1 = missing; cells:
// (row, column) of the missing cells whose row lies in this block; out[c]: new value, or NaN
// when the cell has no usable neighbour (the reference leaves it unchanged).
__global__ void k_impute(ImputeArgs a) {
    const int lane = threadIdx.x & 31;
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const size_t n = a.n;
    float* wbuf = a.scratch + (size_t)wid * a.scratch_stride;
    float* vbuf = wbuf + n;
    float* tbuf = vbuf + n;  // per-category subsequence
    float* lp = tbuf + n;
    if (reinterpret_cast<uintptr_t>(lp) & 7) ++lp;         // int2 alignment
    int2* leaves = reinterpret_cast<int2*>(lp) + 1;         // [-1] carries the leaf count
    float* leafsum = reinterpret_cast<float*>(leaves + a.max_leaves + 1);
    const unsigned lt = (1u << lane) - 1u;
    for (int c = wid; c < a.ncells; c += nwarps) {
        const int i = a.cells[2 * c], j = a.cells[2 * c + 1];
        const float* srow = a.S + (size_t)(i - a.r0) * a.ldS;
        const uint8_t* mj = a.miss + (size_t)j * n;
        const float* xj = a.xc + (size_t)j * n;
        int m = 0;
        for (size_t k0 = 0; k0 < n; k0 += 32) {
            const size_t k = k0 + lane;
            float s = 0.0f;
            bool sel = false;
            if (k < n && (int)k != i && !mj[k]) {
                s = srow[k];
                sel = s > 0.0f;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, sel);
            if (sel) {
                const int pos = m + __popc(bal & lt);
                wbuf[pos] = s;
                vbuf[pos] = xj[k];
            }
            m += __popc(bal);
        }
        __syncwarp();
        float result = __int_as_float(0x7fc00000);
        if (m > 0) {
            if (!a.is_cat[j]) {
                const float tot = warp_pairwise(wbuf, m, leaves, leafsum, lane);
                for (int q = lane; q < m; q += 32) wbuf[q] = (wbuf[q] / tot) * vbuf[q];
                __syncwarp();
                result = warp_pairwise(wbuf, m, leaves, leafsum, lane);
            } else {
                // distinct values ascending; weight of each = pairwise sum of its subsequence
                float prev = -__int_as_float(0x7f800000);
                bool first = true;
                float best = 0.0f, best_v = 0.0f;
                for (;;) {
                    float nxt = __int_as_float(0x7f800000);
                    for (int q = lane; q < m; q += 32) {
                        const float v = vbuf[q];
                        if ((first || v > prev) && v < nxt) nxt = v;
                    }
                    for (int o = 16; o > 0; o >>= 1) nxt = fminf(nxt, __shfl_xor_sync(0xffffffffu, nxt, o));
                    bool any = false;
                    for (int q = lane; q < m; q += 32) any |= vbuf[q] == nxt;
                    if (!__any_sync(0xffffffffu, any)) break;
                    int mc = 0;
                    for (int q0 = 0; q0 < m; q0 += 32) {
                        const int q = q0 + lane;
                        const bool selc = q < m && vbuf[q] == nxt;
                        const unsigned bal = __ballot_sync(0xffffffffu, selc);
                        if (selc) tbuf[mc + __popc(bal & lt)] = wbuf[q];
                        mc += __popc(bal);
                    }
                    __syncwarp();
                    const float cntw = warp_pairwise(tbuf, mc, leaves, leafsum, lane);
                    if (first || cntw > best) {
                        best = cntw;
                        best_v = nxt;
                    }
                    first = false;
                    prev = nxt;
                }
                result = best_v;
            }
        }
        if (lane == 0) a.out[c] = result;
        __syncwarp();
    }
}

}  // namespace rfx
