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
__global__ void __launch_bounds__(1024) k_level_begin(Batch B) {
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
        B.counters[2] = 0;
    }
}

// ---------------------------------------------------------------------------------------
// Node evaluation (one warp per node of the level): member count, class counts and
// majority, or the serial float sums of y; the size, purity and variance tests that
// decide whether the node is searched (src/rf_growtree.cpp:700-774); crit0 (:783-795).
// Nodes that are not searched become terminal here.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_node_eval(Data D, Batch B, int cur) {
    __shared__ int ccount[8][kMaxClass];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int total = B.counters[0];
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const bool regr = D.nclass == 1;
    for (int w = blockIdx.x * (blockDim.x >> 5) + wib; w < total; w += nwarps) {
        const int t = tree_of(B.lvl_off, B.T, w);
        const int node = B.lvl_lo[t] + (w - B.lvl_off[t]);
        const size_t m = (size_t)t * B.M + node;
        const int start = B.nd_start[m], c = B.nd_cnt[m];
        const int* seg = B.seg[cur] + (size_t)t * D.N + start;
        float ts = 0.0f, ts2 = 0.0f;
        int maj = 0, nz = 0;
        if (regr) {
            for (int b0 = 0; b0 < c; b0 += 32) {
                const int i = b0 + lane;
                const float v = i < c ? D.yv[seg[i]] : 0.0f;
                const int k = min(32, c - b0);
                for (int j = 0; j < k; ++j) {
                    const float x = __shfl_sync(kFull, v, j);
                    ts += x * 1.0f;
                    ts2 += x * x * 1.0f;
                }
            }
        } else {
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
        }
        if (lane == 0) {
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
    int carry = 0;
    for (int k0 = lo; k0 < hi; k0 += blockDim.x) {
        const int node = k0 + threadIdx.x;
        const bool f = node < hi && B.nd_flag[(size_t)t * B.M + node];
        int tot;
        const int ex = block_excl_scan(f ? 1 : 0, ws, tot);
        if (f) {
            srch[carry + ex] = node;
            B.nd_key[(size_t)t * B.M + node] = kNoKey;
        }
        carry += tot;
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
    if (threadIdx.x == 0) B.srch_cnt[t] = (B.nnode[t] + 2 <= B.M) ? S : 0;
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
    if (threadIdx.x == 0) {
        B.srch_off[B.T] = carry;
        B.counters[1] = carry;
    }
}

// ---------------------------------------------------------------------------------------
// Histogram split search (one block per searched node, one warp per drawn feature):
// histogram_find_best_split_classification / _regression (src/rf_growtree.cpp:22-184)
// and the per-node comparison across the mtry draws (:820-836, :929-955).
//
// The node's packed rows (bins + target) are staged through shared memory in chunks, so
// each row crosses L2 once per level however many features are drawn.  Each warp builds
// its feature's histogram: classification as integer class counts (the reference's float
// counts are small integers, so exact); regression as float sums that must equal the
// reference's row-order serial sums bin by bin -- rows that hit the same bin within a
// 32-row step are added one rank at a time, in row order.
//
// Only non-empty bins can win (an empty bin repeats the previous bin's criterion, and
// the reference keeps the first of equal values), so the scan runs over the compacted
// list of non-empty bins.  The running left/right sums of the scan are serial float
// chains in the reference; lanes 0..2 compute them in bin order, then all lanes evaluate
// the criterion of every candidate bin in parallel and the first minimum wins.
//
// Per-node winner: key = (order-preserving bits of the criterion, draw index, bin); the
// smallest key is the reference's choice (regression: lowest MSE, first draw wins ties;
// classification: highest 2 - gini, i.e. lowest -(2 - gini), first draw wins ties).
// ---------------------------------------------------------------------------------------
struct HistLayout {
    int warp_bytes;   // per-warp scratch
    int stage_rows;   // rows staged per chunk
};

__device__ __forceinline__ void warp_compact_bins(uint32_t* mask, uint8_t* bl, int lane, int& m) {
    // bl[0..m) = ascending list of set bits of mask[0..8).
    uint32_t w = lane < 8 ? mask[lane] : 0u;
    int cnt = __popc(w), x = cnt;
    for (int o = 1; o < 8; o <<= 1) {
        const int y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    int off = x - cnt;
    m = __shfl_sync(kFull, x, 7);
    if (lane < 8) {
        while (w) {
            const int b = __ffs(w) - 1;
            w &= w - 1;
            bl[off++] = (uint8_t)(lane * 32 + b);
        }
        mask[lane] = 0u;
    }
    __syncwarp();
}

__global__ void __launch_bounds__(512) k_hist(Data D, Batch B, int cur, int nwarp_blk,
                                              int stage_rows, int warp_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ unsigned long long wkey[16];
    __shared__ int snode[4];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int nthr = blockDim.x;
    const bool regr = D.nclass == 1;
    const int nc = D.nclass;
    const int rs = D.rs, ro = D.ro;
    uint8_t* stage = smem;
    uint8_t* wbase = smem + (size_t)stage_rows * rs + (size_t)wib * warp_bytes;
    // per-warp scratch
    uint32_t* mask = reinterpret_cast<uint32_t*>(wbase);                // [8]
    uint8_t* bl = wbase + 32;                                           // [256]
    float* sy = reinterpret_cast<float*>(wbase + 288);                  // [256] / class hist
    float* sy2 = sy + kBins;
    int* cn = reinterpret_cast<int*>(sy2 + kBins);
    float* r1 = reinterpret_cast<float*>(cn + kBins);
    float* r2 = r1 + kBins;
    int* h = reinterpret_cast<int*>(wbase + 288);                       // [256][nc] + tc[32]
    int* tc = h + kBins * nc;
    // scratch starts zeroed
    for (int k = lane; k < warp_bytes / 4; k += 32) reinterpret_cast<uint32_t*>(wbase)[k] = 0u;
    __syncwarp();
    const int total = B.counters[1];
    const uint32_t lt = (1u << lane) - 1u;
    for (int si = blockIdx.x; si < total; si += gridDim.x) {
        if (threadIdx.x == 0) {
            const int t = tree_of(B.srch_off, B.T, si);
            snode[0] = t;
            snode[1] = B.srch[(size_t)t * B.M + (si - B.srch_off[t])];
        }
        __syncthreads();
        const int t = snode[0], node = snode[1];
        const size_t m = (size_t)t * B.M + node;
        const int start = B.nd_start[m], c = B.nd_cnt[m];
        const int* seg = B.seg[cur] + (size_t)t * D.N + start;
        const uint16_t* featp = B.feat + (size_t)t * B.M * B.mtry + (size_t)node * B.mtry;
        unsigned long long best_key = kNoKey;
        for (int r0 = 0; r0 < B.mtry; r0 += nwarp_blk) {
            const int mv = r0 + wib;
            const bool active = mv < B.mtry;
            const int f = active ? featp[mv] : 0;
            // ---- histogram over the node's rows, staged chunk by chunk
            for (int c0 = 0; c0 < c; c0 += stage_rows) {
                const int ch = min(stage_rows, c - c0);
                const int pieces = rs >> 4;
                for (int k = threadIdx.x; k < ch * pieces; k += nthr) {
                    const int rr = k / pieces, pc = k - rr * pieces;
                    const uint4* src = reinterpret_cast<const uint4*>(D.rows + (size_t)seg[c0 + rr] * rs) + pc;
                    reinterpret_cast<uint4*>(stage + (size_t)rr * rs)[pc] = __ldg(src);
                }
                __syncthreads();
                if (active) {
                    for (int s0 = 0; s0 < ch; s0 += 32) {
                        const int i = s0 + lane;
                        const bool valid = i < ch;
                        const uint8_t* row = stage + (size_t)i * rs;
                        const int b = valid ? row[f] : kBins;
                        const uint32_t peers = __match_any_sync(kFull, b);
                        const int rank = __popc(peers & lt);
                        if (valid && rank == 0) atomicOr(&mask[b >> 5], 1u << (b & 31));
                        if (regr) {
                            float v = 0.0f, v2 = 0.0f;
                            if (valid) {
                                const float2 yy = *reinterpret_cast<const float2*>(row + ro);
                                v = yy.x;
                                v2 = yy.y;
                            }
                            const int maxr = __reduce_max_sync(kFull, valid ? __popc(peers) - 1 : 0);
                            for (int q = 0; q <= maxr; ++q) {
                                if (valid && rank == q) {
                                    sy[b] += v * 1.0f;
                                    sy2[b] += v2 * 1.0f;
                                    cn[b] += 1;
                                }
                                __syncwarp();
                            }
                        } else if (valid) {
                            atomicAdd(&h[b * nc + *reinterpret_cast<const int*>(row + ro)], 1);
                        }
                    }
                }
                __syncthreads();
            }
            // ---- scan of the non-empty bins
            unsigned long long key = kNoKey;
            if (active) {
                __syncwarp();
                int nm;
                warp_compact_bins(mask, bl, lane, nm);
                const int nbf = D.nb[f];
                (void)nbf;
                float bestv = 1e20f;
                int bestj = 0x7fffffff;
                if (regr) {
                    if (lane == 0) {
                        float tot = 0.0f;
                        for (int j = 0; j < nm; ++j) tot += sy[bl[j]];
                        float l = 0.0f, r = tot;
                        for (int j = 0; j < nm; ++j) {
                            const float s = sy[bl[j]];
                            l += s;
                            r -= s;
                            sy[j] = l;
                            r1[j] = r;
                        }
                    } else if (lane == 1) {
                        float tot = 0.0f;
                        for (int j = 0; j < nm; ++j) tot += sy2[bl[j]];
                        float l = 0.0f, r = tot;
                        for (int j = 0; j < nm; ++j) {
                            const float s = sy2[bl[j]];
                            l += s;
                            r -= s;
                            sy2[j] = l;
                            r2[j] = r;
                        }
                    } else if (lane == 2) {
                        int l = 0;
                        for (int j = 0; j < nm; ++j) {
                            l += cn[bl[j]];
                            cn[j] = l;
                        }
                    }
                    __syncwarp();
                    for (int j = lane; j < nm - 1; j += 32) {
                        const float cl = (float)cn[j], cr = (float)(c - cn[j]);
                        const float sl = sy[j], sr = r1[j], s2l = sy2[j], s2r = r2[j];
                        const float ml = sl / cl, mr = sr / cr;
                        const float vl = s2l / cl - ml * ml, vr = s2r / cr - mr * mr;
                        const float tot = cl + cr;
                        const float mse = (cl * vl + cr * vr) / tot;
                        if (mse < bestv) { bestv = mse; bestj = j; }
                    }
                } else {
                    if (lane < nc) {
                        int l = 0;
                        for (int j = 0; j < nm; ++j) {
                            l += h[bl[j] * nc + lane];
                            h[j * nc + lane] = l;
                        }
                        tc[lane] = l;
                    }
                    __syncwarp();
                    for (int j = lane; j < nm - 1; j += 32) {
                        int tl = 0;
                        for (int k = 0; k < nc; ++k) tl += h[j * nc + k];
                        const float tlf = (float)tl, trf = (float)(c - tl);
                        float gl = 1.0f, gr = 1.0f;
                        for (int k = 0; k < nc; ++k) {
                            const int lk = h[j * nc + k];
                            const float pl = (float)lk / tlf;
                            const float pr = (float)(tc[k] - lk) / trf;
                            gl -= pl * pl;
                            gr -= pr * pr;
                        }
                        const float tot = tlf + trf;
                        const float g = (tlf * gl + trf * gr) / tot;
                        if (g < bestv) { bestv = g; bestj = j; }
                    }
                }
                // first minimum across lanes
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(kFull, bestv, o);
                    const int oj = __shfl_xor_sync(kFull, bestj, o);
                    if (ov < bestv || (ov == bestv && oj < bestj)) { bestv = ov; bestj = oj; }
                }
                if (bestj != 0x7fffffff) {
                    const float crit = regr ? bestv : -(2.0f - bestv);
                    key = ((unsigned long long)ord_of(crit) << 32) |
                          ((unsigned long long)mv << 8) | (unsigned long long)bl[bestj];
                }
                __syncwarp();
                // restore zeroed scratch
                if (regr) {
                    for (int j = lane; j < nm; j += 32) {
                        const int b = bl[j];
                        sy[j] = 0.0f; sy2[j] = 0.0f; cn[j] = 0;
                        sy[b] = 0.0f; sy2[b] = 0.0f; cn[b] = 0;
                    }
                } else {
                    for (int j = lane; j < nm; j += 32) {
                        const int b = bl[j];
                        for (int k = 0; k < nc; ++k) { h[j * nc + k] = 0; h[b * nc + k] = 0; }
                    }
                }
                __syncwarp();
            }
            if (lane == 0) wkey[wib] = key;
            __syncthreads();
            if (threadIdx.x == 0)
                for (int w = 0; w < nwarp_blk; ++w) best_key = min(best_key, wkey[w]);
            __syncthreads();
        }
        if (threadIdx.x == 0) B.nd_key[m] = best_key;
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

}  // namespace rfx
