// Level-wise histogram tree growth of a batch of trees: cpu_growtree's histogram path
// (src/rf_growtree.cpp:616-1161) restructured so that every node of one tree level, in
// every tree of the batch, is processed by one launch of each kernel below.
//
// The reference visits nodes one at a time in creation order (breadth first), so the
// nodes of level d are exactly the ids [lvl_lo, lvl_hi) and are all visited before any
// node of level d+1.  Everything order-dependent in the reference is reproduced:
//   * split-variable draws: one MT19937 stream per tree, consumed by the searched nodes of
//     the level in node-id order, mtry draws each (k_draw);
//   * child ids: the parents that split, in node-id order, take nnode, nnode+2, ... until
//     the maxnode cap stops all later ones (k_commit);
//   * node members: every node owns a contiguous segment of its tree's distinct in-bag
//     rows in ascending row order (k_partition is a stable partition), which is the order
//     in which the reference accumulates its float sums.
#include "rfx_device.cuh"
#include "rfx_kernels.h"

namespace rfx {

// ---------------------------------------------------------------------------------------
// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ int block_excl_scan(int v, int* wsum, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? wsum[lane] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) wsum[lane] = w;
    }
    __syncthreads();
    const int excl = x - v + (warp > 0 ? wsum[warp - 1] : 0);
    total = wsum[nw - 1];
    __syncthreads();
    return excl;
}

// Level ranges of every tree, their prefix (flattened task index -> tree) and total width.
__global__ void __launch_bounds__(1024) k_level_begin(Batch B, int level) {
    __shared__ int ws[32];
    int carry = 0;
    for (int t0 = 0; t0 < B.T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int w = 0;
        if (t < B.T) {
            const int lo = B.nxt_lo[t], hi = B.nxt_hi[t];
            B.lvl_lo[t] = lo;
            B.lvl_hi[t] = hi;
            w = hi - lo;
        }
        int tot;
        const int ex = block_excl_scan(w, ws, tot);
        if (t < B.T) B.lvl_off[t] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) {
        B.lvl_off[B.T] = carry;
        B.counters[0] = carry;
        B.counters[20] = 0;
        B.counters[21] = 0;
        B.counters[22] = 0;
        if (carry > 0) B.counters[7] = level + 1;  // levels that had nodes
        B.counters[2] = 0;
        B.counters[5] = 0;
    }
}

// ---------------------------------------------------------------------------------------
// Node evaluation (classification: one warp per node of the level; regression: one lane
// per node of at most kEvalLaneNode rows, one warp per larger node): member count, class
// counts and majority, or the serial float sums of y; the size, purity and variance tests that
// decide whether the node is searched (src/rf_growtree.cpp:700-774); crit0 (:783-795).
// Nodes that are not searched become terminal here.
// ---------------------------------------------------------------------------------------
// Node record and stop tests from the node's sums (regression ts/ts2) or class counts.
__device__ __forceinline__ void node_finalize(const Batch& B, size_t m, int c, int cur, bool regr,
                                              float ts, float ts2, int maj, int nz) {
    B.nd_buf[m] = (uint8_t)cur;
    bool searched = c >= B.minsplit;
    float crit0 = 0.0f;
    if (regr) {
        const float tw = (float)c;
        B.nd_sum[m] = ts;
        if (searched) {
            if (tw > 1.0e-5f) {
                const float mean = ts / tw;
                const float var = ts2 / tw - mean * mean;
                if (var < 1.0e-6f) searched = false;
                crit0 = var;
            } else {
                searched = false;
            }
        }
    } else {
        B.nd_maj[m] = maj;
        if (searched && nz <= 1) searched = false;
    }
    B.nd_crit0[m] = crit0;
    B.nd_flag[m] = searched ? 1 : 0;
    if (!searched) {
        B.status[m] = -1;
        B.nodeclass[m] = regr ? 0 : maj;
        if (regr) {
            B.nodepred[m] = c > 0 ? ts / (float)c : 0.0f;
            B.tnodewt[m] = c > 0 ? 1.0f : 0.0f;
        }
    }
}

// Regression nodes up to this many rows are summed by one lane (32 nodes per warp).
constexpr int kEvalLaneNode = 64;

__global__ void __launch_bounds__(256) k_node_eval(Data D, Batch B, int cur) {
    __shared__ int ccount[8][kMaxClass];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int total = B.counters[0];
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const bool regr = D.nclass == 1;
    if (regr) {
        // G level nodes per warp (G = nodes per warp of the grid, 1..32, so that every
        // warp has work at the top levels): a lane sums a small node's rows serially (row
        // order); the larger ones are summed by the whole warp, one after another
        const int G = max(1, min(32, total / nwarps));
        for (int w0 = (blockIdx.x * (blockDim.x >> 5) + wib) * G; w0 < total; w0 += nwarps * G) {
            const int w = w0 + lane;
            size_t m = 0;
            int c = 0, start = 0, t = 0;
            if (lane < G && w < total) {
                t = tree_of(B.lvl_off, B.T, w);
                m = (size_t)t * B.M + B.lvl_lo[t] + (w - B.lvl_off[t]);
                start = B.nd_start[m];
                c = B.nd_cnt[m];
            }
            const bool mine = lane < G && w < total && c <= kEvalLaneNode;
            if (mine) {
                const int* seg = B.seg[cur] + (size_t)t * D.N + start;
                float ts = 0.0f, ts2 = 0.0f;
                constexpr int U = 8;
                for (int i0 = 0; i0 < c; i0 += U) {
                    float v[U];
#pragma unroll
                    for (int q = 0; q < U; ++q) v[q] = i0 + q < c ? D.yv[seg[i0 + q]] : 0.0f;
#pragma unroll
                    for (int q = 0; q < U; ++q) {
                        if (i0 + q < c) {
                            ts += v[q] * 1.0f;
                            ts2 += v[q] * v[q] * 1.0f;
                        }
                    }
                }
                node_finalize(B, m, c, cur, true, ts, ts2, 0, 0);
            }
            unsigned big = __ballot_sync(kFull, lane < G && w < total && !mine);
            while (big) {
                const int src = __ffs(big) - 1;
                big &= big - 1;
                const size_t mb = __shfl_sync(kFull, (unsigned long long)m, src);
                const int cb = __shfl_sync(kFull, c, src);
                const int sb = __shfl_sync(kFull, start, src);
                const int tb = __shfl_sync(kFull, t, src);
                const int* seg = B.seg[cur] + (size_t)tb * D.N + sb;
                // serial sums in row order (lane 0's copy is the one kept); 8 x 32 values
                // are gathered per step so their loads are in flight together
                float ts = 0.0f, ts2 = 0.0f;
                constexpr int U = 8;
                for (int b0 = 0; b0 < cb; b0 += 32 * U) {
                    float v[U];
#pragma unroll
                    for (int q = 0; q < U; ++q) {
                        const int i = b0 + q * 32 + lane;
                        v[q] = i < cb ? D.yv[seg[i]] : 0.0f;
                    }
#pragma unroll
                    for (int q = 0; q < U; ++q) {
                        const int k = min(32, cb - (b0 + q * 32));
                        if (k == 32) {  // unrolled: the shuffles issue ahead of the chain
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                const float x = __shfl_sync(kFull, v[q], j);
                                ts += x * 1.0f;
                                ts2 += x * x * 1.0f;
                            }
                        } else {
                            for (int j = 0; j < k; ++j) {
                                const float x = __shfl_sync(kFull, v[q], j);
                                ts += x * 1.0f;
                                ts2 += x * x * 1.0f;
                            }
                        }
                    }
                }
                if (lane == 0) node_finalize(B, mb, cb, cur, true, ts, ts2, 0, 0);
                __syncwarp();
            }
        }
        return;
    }
    for (int w = blockIdx.x * (blockDim.x >> 5) + wib; w < total; w += nwarps) {
        const int t = tree_of(B.lvl_off, B.T, w);
        const int node = B.lvl_lo[t] + (w - B.lvl_off[t]);
        const size_t m = (size_t)t * B.M + node;
        const int start = B.nd_start[m], c = B.nd_cnt[m];
        const int* seg = B.seg[cur] + (size_t)t * D.N + start;
        int maj = 0, nz = 0;
        if (lane < kMaxClass) ccount[wib][lane] = 0;
        __syncwarp();
        for (int i = lane; i < c; i += 32) atomicAdd(&ccount[wib][D.lab[seg[i]]], 1);
        __syncwarp();
        int mx = 0;
        for (int j = 0; j < D.nclass; ++j) {
            const int k = ccount[wib][j];
            if (k > 0) { ++nz; if (k > mx) { mx = k; maj = j; } }
        }
        __syncwarp();
        if (lane == 0) node_finalize(B, m, c, cur, false, 0.0f, 0.0f, maj, nz);
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------
// Split-variable draws (one block per tree): the searched nodes of the level in node
// order, mtry draws each, mvar = (int)(randomu() * mdim) clamped to mdim-1
// (src/rf_growtree.cpp:808, 930).  Trees whose node count already prevents any split get
// no histogram tasks (their searched nodes still consume their draws).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_draw(Data D, Batch B) {
    __shared__ uint32_t s[624];
    __shared__ int ws[32];
    const int t = blockIdx.x;
    const int lo = B.lvl_lo[t], hi = B.lvl_hi[t];
    int* srch = B.srch + (size_t)t * B.M;
    int* big = B.srch_big + (size_t)t * B.M;
    int* sml = B.srch_sml + (size_t)t * B.M;
    const int lim = small_node_limit(D.nclass, B.mtry);
    int carry = 0, bcarry = 0;
    for (int k0 = lo; k0 < hi; k0 += blockDim.x) {
        const int node = k0 + threadIdx.x;
        const bool f = node < hi && B.nd_flag[(size_t)t * B.M + node];
        const bool fb = f && B.nd_cnt[(size_t)t * B.M + node] > lim;
        int tot, btot;
        const int ex = block_excl_scan(f ? 1 : 0, ws, tot);
        const int bex = block_excl_scan(fb ? 1 : 0, ws, btot);
        if (f) {
            srch[carry + ex] = node;
            B.nd_key[(size_t)t * B.M + node] = kNoKey;
        }
        if (fb) big[bcarry + bex] = node;
        if (f && !fb) sml[(carry - bcarry) + (ex - bex)] = node;
        carry += tot;
        bcarry += btot;
    }
    __syncthreads();
    const int S = carry;
    if (S > 0) {
        uint32_t* g = B.mt + (size_t)t * 624;
        for (int k = threadIdx.x; k < 624; k += blockDim.x) s[k] = g[k];
        __syncthreads();
        const int mtry = B.mtry, p = D.p;
        uint16_t* feat = B.feat + (size_t)t * B.M * mtry;
        const int pos = mt_generate(s, B.mt_pos[t], (long long)S * mtry, [&](long long d, uint32_t y) {
            int mv = (int)(mt_uniform(y) * (float)p);
            if (mv >= p) mv = p - 1;
            const int node = srch[d / mtry];
            feat[(size_t)node * mtry + (d % mtry)] = (uint16_t)mv;
        });
        for (int k = threadIdx.x; k < 624; k += blockDim.x) g[k] = s[k];
        if (threadIdx.x == 0) B.mt_pos[t] = pos;
    }
    if (threadIdx.x == 0) {
        const bool open = B.nnode[t] + 2 <= B.M;
        B.srch_cnt[t] = open ? S : 0;
        B.srch_big_cnt[t] = open ? bcarry : 0;
        B.srch_sml_cnt[t] = open ? S - bcarry : 0;
    }
}

__global__ void __launch_bounds__(1024) k_srch_scan(Batch B) {
    __shared__ int ws[32];
    int carry = 0;
    for (int t0 = 0; t0 < B.T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        const int w = t < B.T ? B.srch_cnt[t] : 0;
        int tot;
        const int ex = block_excl_scan(w, ws, tot);
        if (t < B.T) B.srch_off[t] = carry + ex;
        carry += tot;
    }
    int bcarry = 0;
    for (int t0 = 0; t0 < B.T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        const int w = t < B.T ? B.srch_big_cnt[t] : 0;
        int tot;
        const int ex = block_excl_scan(w, ws, tot);
        if (t < B.T) B.srch_big_off[t] = bcarry + ex;
        bcarry += tot;
    }
    int scarry = 0;
    for (int t0 = 0; t0 < B.T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        const int w = t < B.T ? B.srch_sml_cnt[t] : 0;
        int tot;
        const int ex = block_excl_scan(w, ws, tot);
        if (t < B.T) B.srch_sml_off[t] = scarry + ex;
        scarry += tot;
    }
    if (threadIdx.x == 0) {
        B.srch_off[B.T] = carry;
        B.srch_big_off[B.T] = bcarry;
        B.srch_sml_off[B.T] = scarry;
        B.counters[1] = carry;
        B.counters[4] = bcarry;
        B.counters[6] = scarry;
    }
}

// Flat task records of the level's big and small searched nodes (one block per tree), so
// that the histogram kernels find a task's tree, node, segment start and size with one load.
// True when the small list feeds k_hist_lane (regression): its records are split by size.
__device__ __forceinline__ bool lane_split_list(const Batch& B) { return B.lane_split != 0; }

__global__ void __launch_bounds__(256) k_task_records(Batch B) {
    const int t = blockIdx.x;
    const size_t base = (size_t)t * B.M;
    const int nb = B.srch_big_cnt[t], ns = B.srch_sml_cnt[t];
    for (int i = threadIdx.x; i < nb + ns; i += blockDim.x) {
        const bool big = i < nb;
        const int node = big ? B.srch_big[base + i] : B.srch_sml[base + (i - nb)];
        const int4 r = make_int4(t, node, B.nd_start[base + node], B.nd_cnt[base + node]);
        if (big) {
            B.big_rec[B.srch_big_off[t] + i] = r;
        } else if (lane_split_list(B)) {
            // regression small list, by size for the three k_hist_lane instantiations: nodes
            // of at most kLaneTiny rows from the front of sml_rec, those above kLaneSmall
            // from its back, the others in sml2_rec
            if (r.w <= kLaneTiny) B.sml_rec[atomicAdd(&B.counters[20], 1)] = r;
            else if (r.w <= kLaneSmall) B.sml2_rec[atomicAdd(&B.counters[22], 1)] = r;
            else B.sml_rec[B.counters[6] - 1 - atomicAdd(&B.counters[21], 1)] = r;
        } else {
            B.sml_rec[B.srch_sml_off[t] + (i - nb)] = r;
        }
    }
}

// ---------------------------------------------------------------------------------------
// Commit the level (one block per tree, nodes in id order): accept rule
// (src/rf_growtree.cpp:1000-1028), child ids under the maxnode cap (:1030-1045, :1066-1073),
// split value = midpoint of the winning bin's edges, or the bin for categorical features
// (:95-101, :177-183).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_commit(Data D, Batch B) {
    __shared__ int ws[32];
    const int t = blockIdx.x;
    const int lo = B.lvl_lo[t], hi = B.lvl_hi[t];
    const bool regr = D.nclass == 1;
    int nn = B.nnode[t];
    const int M = B.M;
    int carry = 0;
    for (int k0 = lo; k0 < hi; k0 += blockDim.x) {
        const int node = k0 + threadIdx.x;
        const size_t m = (size_t)t * M + node;
        bool searched = false, wants = false;
        unsigned long long key = kNoKey;
        if (node < hi && B.nd_flag[m]) {
            searched = true;
            key = B.nd_key[m];
            if (key != kNoKey) {
                const float best = float_of((uint32_t)(key >> 32));
                if (regr) {
                    const float crit0 = B.nd_crit0[m];
                    const float red = crit0 - best;
                    wants = !(red < 1.0e-6f) && best < crit0;
                } else {
                    wants = (-best) > -1.0f;
                }
            }
        }
        int tot;
        const int rank = block_excl_scan(wants ? 1 : 0, ws, tot);
        if (searched) {
            const int child = nn + 2 * (carry + rank);
            if (wants && child + 2 <= M) {
                const int mv = (int)((key >> 8) & 0xffffffu);
                const int bin = (int)(key & 0xffu);
                const int f = B.feat[(size_t)t * M * B.mtry + (size_t)node * B.mtry + mv];
                const float* e = D.edges + (size_t)f * 257;
                const float split = D.kind[f] == 2 ? (float)bin : (e[bin] + e[bin + 1]) / 2.0f;
                B.status[m] = 1;
                B.bestvar[m] = f;
                B.xbest[m] = split;
                B.treemap[2 * m] = child;
                B.treemap[2 * m + 1] = child + 1;
                if (B.nd_cnt[m] > kBigSegment) B.part_big[atomicAdd(&B.counters[5], 1)] = (long long)m;
                B.status[(size_t)t * M + child] = 2;
                B.status[(size_t)t * M + child + 1] = 2;
            } else {
                const int c = B.nd_cnt[m];
                B.status[m] = -1;
                B.nodeclass[m] = regr ? 0 : B.nd_maj[m];
                if (regr) {
                    B.nodepred[m] = c > 0 ? B.nd_sum[m] / (float)c : 0.0f;
                    B.tnodewt[m] = c > 0 ? 1.0f : 0.0f;
                }
            }
        }
        carry += tot;
    }
    if (threadIdx.x == 0) {
        const int splits = min(carry, max(0, (M - nn) / 2));
        const int nn2 = nn + 2 * splits;
        B.nnode[t] = nn2;
        B.nxt_lo[t] = hi;
        B.nxt_hi[t] = nn2;
        atomicAdd(&B.counters[2], nn2 - hi);
    }
}

// ---------------------------------------------------------------------------------------
// Stable partition of the split nodes' segments (one warp per node of the level): rows
// with x <= split (raw value, src/rf_growtree.cpp:1051-1061) keep their order on the left,
// the others on the right, into the other segment buffer.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_partition(Data D, Batch B, int cur) {
    __shared__ uint32_t bits[8][64];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int total = B.counters[0];
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const uint32_t lt = (1u << lane) - 1u;
    for (int w = blockIdx.x * (blockDim.x >> 5) + wib; w < total; w += nwarps) {
        const int t = tree_of(B.lvl_off, B.T, w);
        const int node = B.lvl_lo[t] + (w - B.lvl_off[t]);
        const size_t m = (size_t)t * B.M + node;
        if (B.status[m] != 1) continue;
        const int start = B.nd_start[m], c = B.nd_cnt[m];
        const int f = B.bestvar[m];
        const float split = B.xbest[m];
        const float* x = D.xc + (size_t)f * D.N;
        const int* src = B.seg[cur] + (size_t)t * D.N + start;
        int* dst = B.seg[cur ^ 1] + (size_t)t * D.N + start;
        if (c > kBigSegment) continue;  // k_partition_big
        const bool cache = c <= 32 * 64;
        int nl = 0;
        for (int b0 = 0, q = 0; b0 < c; b0 += 32, ++q) {
            const int i = b0 + lane;
            const bool left = i < c && x[src[i]] <= split;
            const uint32_t bal = __ballot_sync(kFull, left);
            if (cache && lane == 0) bits[wib][q] = bal;
            nl += __popc(bal);
        }
        __syncwarp();
        int lo = 0, ro = 0;
        for (int b0 = 0, q = 0; b0 < c; b0 += 32, ++q) {
            const int i = b0 + lane;
            const bool valid = i < c;
            const int sid = valid ? src[i] : 0;
            uint32_t bal;
            if (cache) bal = bits[wib][q];
            else bal = __ballot_sync(kFull, valid && x[sid] <= split);
            const uint32_t vmask = __ballot_sync(kFull, valid);
            const bool left = (bal >> lane) & 1u;
            if (valid) {
                if (left) dst[lo + __popc(bal & lt)] = sid;
                else dst[nl + ro + __popc(~bal & vmask & lt)] = sid;
            }
            lo += __popc(bal);
            ro += __popc(~bal & vmask);
        }
        __syncwarp();
        if (lane == 0) {
            const int l = B.treemap[2 * m], r = B.treemap[2 * m + 1];
            const size_t ml = (size_t)t * B.M + l, mr = (size_t)t * B.M + r;
            B.nd_start[ml] = start;
            B.nd_cnt[ml] = nl;
            B.nd_start[mr] = start + nl;
            B.nd_cnt[mr] = c - nl;
        }
    }
}

// Stable partition of the large split segments (c > kBigSegment), one block per node.
// Pass 1 evaluates x <= split for every row (8 consecutive rows per thread, gathers in
// flight together) and keeps the outcome as a bitmask in shared memory; pass 2 scatters
// with a block-wide scan per 2048-row tile.  Segments longer than the bitmask (384,000
// rows) re-evaluate the comparison in pass 2.
constexpr int kPartItems = 8;
constexpr int kPartBitWords = 12000;  // ~47 KiB of flags (static shared memory limit)

__global__ void __launch_bounds__(256) k_partition_big(Data D, Batch B, int cur) {
    __shared__ uint32_t flags[kPartBitWords];
    __shared__ int ws[32];
    __shared__ int red;
    const int total = B.counters[5];
    const int tile = kPartItems * blockDim.x;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
        const size_t m = (size_t)B.part_big[w];
        const int t = (int)(m / B.M);
        const int c = B.nd_cnt[m];
        const int start = B.nd_start[m];
        const int f = B.bestvar[m];
        const float split = B.xbest[m];
        const float* x = D.xc + (size_t)f * D.N;
        const int* src = B.seg[cur] + (size_t)t * D.N + start;
        int* dst = B.seg[cur ^ 1] + (size_t)t * D.N + start;
        const bool cached = c <= kPartBitWords * 32;
        if (threadIdx.x == 0) red = 0;
        __syncthreads();
        int mine = 0;
        for (int b0 = 0; b0 < c; b0 += tile) {
            const int i0 = b0 + threadIdx.x * kPartItems;
            uint32_t bitsv = 0;
#pragma unroll
            for (int k = 0; k < kPartItems; ++k) {
                const int i = i0 + k;
                if (i < c && x[src[i]] <= split) bitsv |= 1u << k;
            }
            mine += __popc(bitsv);
            if (cached && i0 < c) reinterpret_cast<uint8_t*>(flags)[i0 >> 3] = (uint8_t)bitsv;
        }
        atomicAdd(&red, mine);
        __syncthreads();
        const int nl = red;
        int lcarry = 0, rcarry = 0;
        for (int b0 = 0; b0 < c; b0 += tile) {
            const int i0 = b0 + threadIdx.x * kPartItems;
            uint32_t bitsv = 0;
            if (cached) {
                bitsv = i0 < c ? reinterpret_cast<const uint8_t*>(flags)[i0 >> 3] : 0u;
            } else {
#pragma unroll
                for (int k = 0; k < kPartItems; ++k) {
                    const int i = i0 + k;
                    if (i < c && x[src[i]] <= split) bitsv |= 1u << k;
                }
            }
            const int nvalid = max(0, min(kPartItems, c - i0));
            const int lcnt = __popc(bitsv);
            int ltot, rtot;
            const int lex = block_excl_scan(lcnt, ws, ltot);
            const int rex = block_excl_scan(nvalid - lcnt, ws, rtot);
            int lp = lcarry + lex, rp = nl + rcarry + rex;
#pragma unroll
            for (int k = 0; k < kPartItems; ++k) {
                const int i = i0 + k;
                if (i < c) {
                    const int sid = src[i];
                    if ((bitsv >> k) & 1u) dst[lp++] = sid;
                    else dst[rp++] = sid;
                }
            }
            lcarry += ltot;
            rcarry += rtot;
        }
        if (threadIdx.x == 0) {
            const int l = B.treemap[2 * m], r = B.treemap[2 * m + 1];
            const size_t ml = (size_t)t * B.M + l, mr = (size_t)t * B.M + r;
            B.nd_start[ml] = start;
            B.nd_cnt[ml] = nl;
            B.nd_start[mr] = start + nl;
            B.nd_cnt[mr] = c - nl;
        }
        __syncthreads();
    }
}

}  // namespace rfx
