// Histogram split search: histogram_find_best_split_classification / _regression
// (src/rf_growtree.cpp:22-184) and the per-node comparison across the mtry draws
// (src/rf_growtree.cpp:820-836, :929-955), for every searched node of a level at once.
//
// Two kernels share the work by node size:
//   k_hist        nodes above small_node_limit rows (64, regression 128): one block per (node, group of up to
//                 8 draws), one warp per drawn feature, the node's rows streamed through
//                 shared memory in chunks;
//   k_hist_small  nodes up to that limit (the great majority at deep levels):
//                 one warp per node does all mtry draws from rows staged once.
//
// Each warp builds its feature's histogram: classification as integer class counts (the
// reference's float counts are small integers, so exact); regression as float sums that
// equal the reference's row-order serial sums bin by bin -- rows that hit the same bin
// within a 32-row step are added one rank at a time, in row order.
//
// Only non-empty bins can win (an empty bin repeats the previous bin's criterion and the
// reference keeps the first of equal values), so the scan runs over the ascending list of
// non-empty bins.  The scan's running left/right sums are serial float chains in the
// reference and are computed in bin order; the criterion of every candidate bin is then
// evaluated in parallel and the first minimum wins.
//
// Winner key = (order-preserving bits of the criterion, draw index, bin); the smallest key
// over all draws of the node is the reference's choice (regression: lowest MSE, first draw
// wins ties; classification: highest 2 - gini, i.e. lowest -(2 - gini), first draw wins).
#include "rfx_device.cuh"
#include "rfx_kernels.h"

namespace rfx {

// bl[0..m) = ascending list of the non-empty bins (cnt[b] > 0).
__device__ __forceinline__ int warp_nonempty_bins(const int* cnt, uint8_t* bl, int lane) {
    int k = 0;
    uint32_t bits = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q)
        if (cnt[lane * 8 + q] > 0) { bits |= 1u << q; ++k; }
    int x = k;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    int off = x - k;
    while (bits) {
        const int q = __ffs(bits) - 1;
        bits &= bits - 1;
        bl[off++] = (uint8_t)(lane * 8 + q);
    }
    const int m = __shfl_sync(kFull, x, 31);
    __syncwarp();
    return m;
}

// Byte q of each of four words -> one word (row r in byte r).
__device__ __forceinline__ uint32_t gather_byte(uint32_t a, uint32_t b, uint32_t c, uint32_t d, int q) {
    const uint32_t lo = __byte_perm(a, b, (uint32_t)(q | ((q + 4) << 4)));
    const uint32_t hi = __byte_perm(c, d, (uint32_t)(q | ((q + 4) << 4)));
    return __byte_perm(lo, hi, 0x5410);
}

// Gini criterion of every candidate bin j < nm - 1 from the inclusive class prefixes
// h[j * nc + k] and the class totals h[256 * nc + k] (node rows c): the lane's first minimum.
__device__ __forceinline__ void class_best(int nc, int c, int nm, int lane, const int* h,
                                           float& bestv, int& bestj) {
    const int* tc = h + 256 * nc;
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
        const float tt = tlf + trf;
        const float g = (tlf * gl + trf * gr) / tt;
        if (g < bestv) { bestv = g; bestj = j; }
    }
}

// Key of the warp's best (first minimum over the lanes' candidates) for draw mv.
__device__ __forceinline__ unsigned long long best_key(bool regr, float bestv, int bestj, int mv,
                                                       const uint8_t* bl) {
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bestv, o);
        const int oj = __shfl_xor_sync(kFull, bestj, o);
        if (ov < bestv || (ov == bestv && oj < bestj)) { bestv = ov; bestj = oj; }
    }
    if (bestj == 0x7fffffff) return kNoKey;
    const float crit = regr ? bestv : -(2.0f - bestv);
    return ((unsigned long long)ord_of(crit) << 32) | ((unsigned long long)mv << 8) |
           (unsigned long long)bl[bestj];
}

// Fold one draw's histogram (sy/sy2/cn or h/cn) into its best key; restores the zeroed
// scratch.  `c` = node rows, `mv` = draw index.  All lanes call it.
__device__ __forceinline__ unsigned long long scan_bins(bool regr, int nc, int c, int mv, int lane,
                                                        uint8_t* bl, float* sy, float* sy2,
                                                        int* cn, int* h) {
    const int nm = warp_nonempty_bins(cn, bl, lane);
    float bestv = 1e20f;
    int bestj = 0x7fffffff;
    if (regr) {
        // bins in 32-wide slices; the serial chains run redundantly on every lane from
        // shuffled per-bin totals (one add per non-empty bin, no shared-memory round trips)
        float tot = 0.0f, tot2 = 0.0f;
        for (int s0 = 0; s0 < nm; s0 += 32) {
            const int j = s0 + lane;
            const int b = j < nm ? bl[j] : 0;
            const float sa = j < nm ? sy[b] : 0.0f, qa = j < nm ? sy2[b] : 0.0f;
            const int kmax = min(32, nm - s0);
            for (int k = 0; k < kmax; ++k) {
                tot += __shfl_sync(kFull, sa, k);
                tot2 += __shfl_sync(kFull, qa, k);
            }
        }
        float L = 0.0f, R = tot, L2 = 0.0f, R2 = tot2;
        int kc = 0;
        for (int s0 = 0; s0 < nm; s0 += 32) {
            const int j = s0 + lane;
            const int b = j < nm ? bl[j] : 0;
            const float sa = j < nm ? sy[b] : 0.0f, qa = j < nm ? sy2[b] : 0.0f;
            const int ka = j < nm ? cn[b] : 0;
            float mL = 0.0f, mR = 0.0f, mL2 = 0.0f, mR2 = 0.0f;
            int mC = 0;
            const int kmax = min(32, nm - s0);
            for (int k = 0; k < kmax; ++k) {
                const float a = __shfl_sync(kFull, sa, k);
                const float a2 = __shfl_sync(kFull, qa, k);
                kc += __shfl_sync(kFull, ka, k);
                L += a;
                R -= a;
                L2 += a2;
                R2 -= a2;
                if (k == lane) { mL = L; mR = R; mL2 = L2; mR2 = R2; mC = kc; }
            }
            if (j < nm - 1) {
                const float cl = (float)mC, cr = (float)(c - mC);
                const float ml = mL / cl, mr = mR / cr;
                const float vl = mL2 / cl - ml * ml, vr = mR2 / cr - mr * mr;
                const float tt = cl + cr;
                const float mse = (cl * vl + cr * vr) / tt;
                if (mse < bestv) { bestv = mse; bestj = j; }
            }
        }
    } else {
        // integer class prefix over the non-empty bins (exact in any order): per class a
        // warp scan over 32 bins at a time, compacted in place (entry j <= bin bl[j])
        __syncwarp();
        for (int k = 0; k < nc; ++k) {
            int carry = 0;
            for (int s0 = 0; s0 < nm; s0 += 32) {
                const int j = s0 + lane;
                int v = j < nm ? h[bl[j] * nc + k] : 0;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(kFull, v, o);
                    if (lane >= o) v += y;
                }
                __syncwarp();
                if (j < nm) h[j * nc + k] = carry + v;
                carry += __shfl_sync(kFull, v, 31);
                __syncwarp();
            }
            if (lane == 0) h[256 * nc + k] = carry;  // class totals
        }
        __syncwarp();
        class_best(nc, c, nm, lane, h, bestv, bestj);
    }
    const unsigned long long key = best_key(regr, bestv, bestj, mv, bl);
    __syncwarp();
    for (int j = lane; j < nm; j += 32) {
        const int b = bl[j];
        if (regr) {
            sy[b] = 0.0f;
            sy2[b] = 0.0f;
        } else {
            for (int k = 0; k < nc; ++k) { h[j * nc + k] = 0; h[b * nc + k] = 0; }
        }
        cn[b] = 0;
    }
    __syncwarp();
    return key;
}

// ---------------------------------------------------------------------------------------
// Regression scan over compacted bin lists.  A draw's non-empty bins (ascending) are a list
// of (sum, sum of squares, count); the scan's serial float chains -- the totals, then the
// running left/right sums -- run lane-serially, one draw per lane, so that one warp
// instruction advances several draws' chains at once; the criterion of every candidate bin
// is then evaluated in parallel over all lists.
// ---------------------------------------------------------------------------------------
constexpr uint32_t kLastEntry = 1u << 31;  // list entry flag: a draw's last bin (no split)

// In place over one list of `len` entries: A/A2/K (bin sum, square sum, count) become the
// running left sums and count; R/R2 receive the running right sums.
__device__ __forceinline__ void regr_chains(float* A, float* A2, int* K, float* R, float* R2,
                                            int len) {
    float tot = 0.0f, tot2 = 0.0f;
    int j = 0;
    for (; j + 8 <= len; j += 8) {
        float a[8], b[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) { a[u] = A[j + u]; b[u] = A2[j + u]; }
#pragma unroll
        for (int u = 0; u < 8; ++u) { tot += a[u]; tot2 += b[u]; }
    }
    for (; j < len; ++j) { tot += A[j]; tot2 += A2[j]; }
    float L = 0.0f, Rv = tot, L2 = 0.0f, Rv2 = tot2;
    int kc = 0;
    j = 0;
    for (; j + 8 <= len; j += 8) {
        float a[8], b[8];
        int k[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) { a[u] = A[j + u]; b[u] = A2[j + u]; k[u] = K[j + u]; }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            kc += k[u];
            L += a[u];
            Rv -= a[u];
            L2 += b[u];
            Rv2 -= b[u];
            A[j + u] = L;
            A2[j + u] = L2;
            K[j + u] = kc;
            R[j + u] = Rv;
            R2[j + u] = Rv2;
        }
    }
    for (; j < len; ++j) {
        kc += K[j];
        L += A[j];
        Rv -= A[j];
        L2 += A2[j];
        Rv2 -= A2[j];
        A[j] = L;
        A2[j] = L2;
        K[j] = kc;
        R[j] = Rv;
        R2[j] = Rv2;
    }
}

// Key of one candidate split (left sums mL/mL2 over mC rows, right sums mR/mR2, node rows c):
// the reference's MSE criterion; candidates whose criterion is not below 1e20 (or NaN) never
// win.  `mvbin` = (draw << 8) | bin.
__device__ __forceinline__ unsigned long long regr_key(float mL, float mR, float mL2, float mR2,
                                                       int mC, int c, uint32_t mvbin) {
    const float cl = (float)mC, cr = (float)(c - mC);
    const float ml = mL / cl, mr = mR / cr;
    const float vl = mL2 / cl - ml * ml, vr = mR2 / cr - mr * mr;
    const float tt = cl + cr;
    const float mse = (cl * vl + cr * vr) / tt;
    return mse < 1e20f ? ((unsigned long long)ord_of(mse) << 32) | mvbin : kNoKey;
}

__device__ __forceinline__ unsigned long long warp_min_key(unsigned long long k) {
    for (int o = 16; o > 0; o >>= 1) k = min(k, __shfl_xor_sync(kFull, k, o));
    return k;
}

// Per-warp scratch layout shared by both kernels (after any staging area):
//   bl[256] uint8 | sy[256] f32 | sy2[256] f32 | cn[256] i32 | h[(256+1) * nclass] i32
// (regression: k_hist uses h as the right sums R[256] | R2[256]; k_hist_small keeps its
// list area at kHistScratch)
__device__ __forceinline__ void warp_scratch(uint8_t* w, uint8_t*& bl, float*& sy, float*& sy2,
                                             int*& cn, int*& h) {
    bl = w;
    sy = reinterpret_cast<float*>(w + 256);
    sy2 = sy + kBins;
    cn = reinterpret_cast<int*>(sy2 + kBins);
    h = cn + kBins;
}

// Histogram of one feature over the 32-row step starting at row s0 (bins `b`, targets v/v2
// or label), rows in order.  All lanes call it.
__device__ __forceinline__ void hist_step(bool regr, int nc, bool valid, int b, float v, float v2,
                                          int label, int lane, float* sy, float* sy2, int* cn,
                                          int* h) {
    const uint32_t peers = __match_any_sync(kFull, b);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (regr) {
        const int maxr = __reduce_max_sync(kFull, valid ? __popc(peers) - 1 : 0);
        for (int qq = 0; qq <= maxr; ++qq) {
            if (valid && rank == qq) {
                sy[b] += v * 1.0f;
                sy2[b] += v2 * 1.0f;
                cn[b] += 1;
            }
            __syncwarp();
        }
    } else {
        if (valid) {
            atomicAdd(&h[b * nc + label], 1);
            if (rank == 0) atomicAdd(&cn[b], __popc(peers));
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------
// Large nodes.  The block streams the node's packed rows (uint8 bins of every feature +
// the target) from L2 through shared memory: each thread loads 4 consecutive rows x 16
// bytes into registers, the next chunk's loads in flight while the warps work on the
// current one, and stores them transposed (feature-major, padded stride) so that the 32
// lanes of a warp read 32 consecutive bytes of their feature without bank conflicts.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512, 2) k_hist(Data D, Batch B, int cur, HistArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int snode[2];
    __shared__ int slen[32];  // regression: list length of each warp's draw
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int nthr = blockDim.x;
    const bool regr = D.nclass == 1;
    const int nc = D.nclass;
    const int rs = D.rs, ro = D.ro;
    const int pieces = rs >> 4;
    const int CH = a.stage_rows;
    const int CS = a.cstride;
    uint8_t* col = smem;                                                    // [rs][CS]
    uint32_t* ytgt = reinterpret_cast<uint32_t*>(smem + (size_t)rs * CS);   // [CH][2]
    uint8_t* wbase = smem + (size_t)rs * CS + (size_t)CH * 8 + (size_t)wib * a.warp_bytes;
    uint8_t* bl;
    float *sy, *sy2;
    int *cn, *h;
    warp_scratch(wbase, bl, sy, sy2, cn, h);
    for (int k = lane; k < a.warp_bytes / 4; k += 32) reinterpret_cast<uint32_t*>(wbase)[k] = 0u;
    __syncwarp();
    const int total = B.counters[4] * a.groups;
    const int units = (CH >> 2) * pieces;
    for (int task = blockIdx.x; task < total; task += gridDim.x) {
        const int si = task / a.groups, grp = task - si * a.groups;
        if (threadIdx.x == 0) {
            const int t = tree_of(B.srch_big_off, B.T, si);
            snode[0] = t;
            snode[1] = B.srch_big[(size_t)t * B.M + (si - B.srch_big_off[t])];
        }
        __syncthreads();
        const int t = snode[0], node = snode[1];
        const size_t m = (size_t)t * B.M + node;
        const int start = B.nd_start[m], c = B.nd_cnt[m];
        const int* seg = B.seg[cur] + (size_t)t * D.N + start;
        const uint16_t* featp = B.feat + (size_t)t * B.M * B.mtry + (size_t)node * B.mtry;
        if (threadIdx.x == 0 && grp == 0 && B.hist_bytes)
            atomicAdd(B.hist_bytes, (unsigned long long)c * (unsigned long long)(B.mtry + (regr ? 4 : 1)));
        const int mv = grp * a.warps + wib;
        const bool active = mv < B.mtry;
        const int f = active ? featp[mv] : 0;
        uint4 reg[2][4];
        auto load_chunk = [&](int c0) {
            const int ch = min(CH, c - c0);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int unit = threadIdx.x + u * nthr;
                if (unit < units) {
                    const int rg = unit / pieces, pc = unit - rg * pieces;
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int i = rg * 4 + r;
                        reg[u][r] = i < ch ? __ldg(reinterpret_cast<const uint4*>(D.rows + (size_t)seg[c0 + i] * rs) + pc)
                                           : make_uint4(0, 0, 0, 0);
                    }
                }
            }
        };
        auto store_chunk = [&]() {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int unit = threadIdx.x + u * nthr;
                if (unit < units) {
                    const int rg = unit / pieces, pc = unit - rg * pieces;
                    const uint32_t* w0 = reinterpret_cast<const uint32_t*>(&reg[u][0]);
                    const uint32_t* w1 = reinterpret_cast<const uint32_t*>(&reg[u][1]);
                    const uint32_t* w2 = reinterpret_cast<const uint32_t*>(&reg[u][2]);
                    const uint32_t* w3 = reinterpret_cast<const uint32_t*>(&reg[u][3]);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int w = j >> 2, q = j & 3;
                        *reinterpret_cast<uint32_t*>(col + (size_t)(pc * 16 + j) * CS + rg * 4) =
                            gather_byte(w0[w], w1[w], w2[w], w3[w], q);
                    }
                    if (pc == (ro >> 4)) {
                        const bool hi = (ro & 15) != 0;  // target in words 2,3 of the piece
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const uint4 v = reg[u][r];
                            reinterpret_cast<uint2*>(ytgt)[rg * 4 + r] =
                                hi ? make_uint2(v.z, v.w) : make_uint2(v.x, v.y);
                        }
                    }
                }
            }
        };
        if (c > 0) load_chunk(0);
        for (int c0 = 0; c0 < c; c0 += CH) {
            const int ch = min(CH, c - c0);
            __syncthreads();
            store_chunk();
            __syncthreads();
            if (c0 + CH < c) load_chunk(c0 + CH);  // in flight during the histogram work
            if (active) {
                const uint8_t* fcol = col + (size_t)f * CS;
                for (int s0 = 0; s0 < ch; s0 += 32) {
                    const int i = s0 + lane;
                    const bool valid = i < ch;
                    const int b = valid ? fcol[i] : kBins;
                    const uint2 yy = reinterpret_cast<const uint2*>(ytgt)[i];
                    hist_step(regr, nc, valid, b, __uint_as_float(yy.x), __uint_as_float(yy.y),
                              (int)yy.x, lane, sy, sy2, cn, h);
                }
            }
        }
        if (!regr) {
            if (active) {
                __syncwarp();
                const unsigned long long key = scan_bins(regr, nc, c, mv, lane, bl, sy, sy2, cn, h);
                if (lane == 0 && key != kNoKey) atomicMin(&B.nd_key[m], key);
            }
            continue;
        }
        // regression: every warp compacts its histogram in place to the list of non-empty
        // bins, lanes of warp 0 run the draws' chains, every warp scores its own list
        int nm = 0;
        if (active) {
            __syncwarp();
            nm = warp_nonempty_bins(cn, bl, lane);
            for (int s0 = 0; s0 < nm; s0 += 32) {  // entry j <= bin bl[j]: forward in place
                const int j = s0 + lane;
                float x = 0.0f, x2 = 0.0f;
                int k = 0;
                if (j < nm) {
                    const int b = bl[j];
                    x = sy[b];
                    x2 = sy2[b];
                    k = cn[b];
                }
                __syncwarp();
                if (j < nm) {
                    sy[j] = x;
                    sy2[j] = x2;
                    cn[j] = k;
                }
                __syncwarp();
            }
        }
        if (lane == 0) slen[wib] = nm;
        __syncthreads();
        if (wib == 0 && lane < a.warps) {
            uint8_t* bl2;
            float *a1, *a2;
            int *k1, *h2;
            warp_scratch(smem + (size_t)rs * CS + (size_t)CH * 8 + (size_t)lane * a.warp_bytes,
                         bl2, a1, a2, k1, h2);
            float* r1 = reinterpret_cast<float*>(h2);
            regr_chains(a1, a2, k1, r1, r1 + kBins, slen[lane]);
        }
        __syncthreads();
        if (active) {
            const float* r1 = reinterpret_cast<const float*>(h);
            unsigned long long best = kNoKey;
            for (int j = lane; j < nm - 1; j += 32)
                best = min(best, regr_key(sy[j], r1[j], sy2[j], r1[kBins + j], cn[j], c,
                                          ((uint32_t)mv << 8) | bl[j]));
            best = warp_min_key(best);
            if (lane == 0 && best != kNoKey) atomicMin(&B.nd_key[m], best);
            __syncwarp();
            for (int k = lane; k < kBins; k += 32) {
                sy[k] = 0.0f;
                sy2[k] = 0.0f;
                cn[k] = 0;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// Small nodes (c <= small_node_limit rows): one warp per searched node does all mtry draws.
// Each lane holds up to four of the node's rows (address and target in registers) and
// reads the drawn feature's bin directly from the packed row; per-warp shared memory holds
// only the histogram, which keeps many warps resident to hide the latency.
// ---------------------------------------------------------------------------------------
constexpr int kSmallRows = kSmallNodeRegr / 32;  // rows per lane in k_hist_small
constexpr int kSmallListOff = 64;                 // regression list area offset per warp

__global__ void __launch_bounds__(256) k_hist_small(Data D, Batch B, int cur, int warp_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const bool regr = D.nclass == 1;
    const int nc = D.nclass;
    const int rs = D.rs, ro = D.ro;
    uint8_t* wbase = smem + (size_t)wib * warp_bytes;
    uint8_t* bl;
    float *sy, *sy2;
    int *cn, *h;
    warp_scratch(wbase, bl, sy, sy2, cn, h);
    // regression: the bin set's words and their rank offsets (8 + 8 words), then the list
    // area: sums, square sums, counts, right sums, right square sums, (draw, bin, last)
    // words -- kListCap entries each (no 256-bin histogram)
    uint32_t* SW = reinterpret_cast<uint32_t*>(wbase);
    int* SP = reinterpret_cast<int*>(SW + 8);
    float* LA = reinterpret_cast<float*>(wbase + kSmallListOff);
    float* LA2 = LA + kListCap;
    int* LK = reinterpret_cast<int*>(LA2 + kListCap);
    float* LR = reinterpret_cast<float*>(LK + kListCap);
    float* LR2 = LR + kListCap;
    uint32_t* LDB = reinterpret_cast<uint32_t*>(LR2 + kListCap);
    for (int k = lane; k < warp_bytes / 4; k += 32)
        reinterpret_cast<uint32_t*>(bl)[k] = 0u;
    __syncwarp();
    const int total = B.counters[1];
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    for (int si = blockIdx.x * (blockDim.x >> 5) + wib; si < total; si += nwarps) {
        const int t = tree_of(B.srch_off, B.T, si);
        const int node = B.srch[(size_t)t * B.M + (si - B.srch_off[t])];
        const size_t m = (size_t)t * B.M + node;
        const int c = B.nd_cnt[m];
        if (c > small_node_limit(nc)) continue;  // k_hist
        if (lane == 0 && B.hist_bytes)
            atomicAdd(B.hist_bytes, (unsigned long long)c * (unsigned long long)(B.mtry + (regr ? 4 : 1)));
        const int* seg = B.seg[cur] + (size_t)t * D.N + B.nd_start[m];
        const uint16_t* featp = B.feat + (size_t)t * B.M * B.mtry + (size_t)node * B.mtry;
        // each lane keeps its rows' address and target in registers; the bins are read
        // straight from the packed rows (L1-resident after the first draw)
        const uint8_t* rowp[kSmallRows];
        float v[kSmallRows], v2[kSmallRows];
        int lab[kSmallRows];
#pragma unroll
        for (int hh = 0; hh < kSmallRows; ++hh) {
            const int i = hh * 32 + lane;
            rowp[hh] = D.rows;
            v[hh] = v2[hh] = 0.0f;
            lab[hh] = 0;
            if (i < c) {
                rowp[hh] = D.rows + (size_t)seg[i] * rs;
                const uint2 tg = __ldg(reinterpret_cast<const uint2*>(rowp[hh] + ro));
                v[hh] = __uint_as_float(tg.x);
                v2[hh] = __uint_as_float(tg.y);
                lab[hh] = (int)tg.x;
            }
        }
        unsigned long long best = kNoKey;
        if (!regr) {
            // classification: the draw's bins as a 256-bit set (words in the unused sums
            // area), class counts per ranked bin with integer atomics, then per-class warp
            // scans (exact in any order) and the criterion of scan_bins
            uint32_t* CW = reinterpret_cast<uint32_t*>(sy);
            int* CP = reinterpret_cast<int*>(sy) + 8;
            for (int mv = 0; mv < B.mtry; ++mv) {
                const int f = featp[mv];
                int bb[kSmallRows];
                uint32_t qmask[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) qmask[q] = 0u;
#pragma unroll
                for (int hh = 0; hh < kSmallRows; ++hh) {
                    bb[hh] = -1;
                    if (hh * 32 < c) {
                        const int i = hh * 32 + lane;
                        if (i < c) bb[hh] = (int)__ldg(rowp[hh] + f);
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            qmask[q] |= (bb[hh] >> 5) == q ? 1u << (bb[hh] & 31) : 0u;
                    }
                }
                int nm = 0;
                uint32_t myw = 0u;
                int myp = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const uint32_t wq = __reduce_or_sync(kFull, qmask[q]);
                    if (lane == q) {
                        myw = wq;
                        myp = nm;
                    }
                    nm += __popc(wq);
                }
                if (lane < 8) {
                    CW[lane] = myw;
                    CP[lane] = myp;
                }
                for (int e = lane; e < nm * nc; e += 32) h[e] = 0;
                __syncwarp();
#pragma unroll
                for (int hh = 0; hh < kSmallRows; ++hh) {
                    if (hh * 32 < c && bb[hh] >= 0) {
                        const int b = bb[hh], q = b >> 5;
                        const int e = CP[q] + __popc(CW[q] & ((1u << (b & 31)) - 1u));
                        atomicAdd(&h[e * nc + lab[hh]], 1);
                        bl[e] = (uint8_t)b;
                    }
                }
                __syncwarp();
                for (int k = 0; k < nc; ++k) {
                    int carry = 0;
                    for (int s0 = 0; s0 < nm; s0 += 32) {
                        const int j = s0 + lane;
                        int x = j < nm ? h[j * nc + k] : 0;
#pragma unroll
                        for (int o = 1; o < 32; o <<= 1) {
                            const int y = __shfl_up_sync(kFull, x, o);
                            if (lane >= o) x += y;
                        }
                        __syncwarp();
                        if (j < nm) h[j * nc + k] = carry + x;
                        carry += __shfl_sync(kFull, x, 31);
                        __syncwarp();
                    }
                    if (lane == 0) h[256 * nc + k] = carry;
                }
                __syncwarp();
                float bestv = 1e20f;
                int bestj = 0x7fffffff;
                class_best(nc, c, nm, lane, h, bestv, bestj);
                best = min(best, best_key(false, bestv, bestj, mv, bl));
                __syncwarp();
            }
        } else {
            // regression: the draws' lists of non-empty bins fill the warp's list area (as
            // many draws as fit, at most 32), then lane d runs draw d's chains and the
            // whole list is scored in parallel
            for (int mv = 0; mv < B.mtry;) {
                int used = 0, nd = 0, my_off = 0, my_len = 0;
                while (mv < B.mtry && nd < 32 && used + c <= kListCap) {
                    const int f = featp[mv];
                    // the node's bins of this draw as a 256-bit set; a row's list entry is
                    // its bin's rank in the set
                    int bb[kSmallRows];
                    uint32_t qmask[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) qmask[q] = 0u;
#pragma unroll
                    for (int hh = 0; hh < kSmallRows; ++hh) {
                        bb[hh] = -1;
                        if (hh * 32 < c) {
                            const int i = hh * 32 + lane;
                            if (i < c) bb[hh] = (int)__ldg(rowp[hh] + f);
#pragma unroll
                            for (int q = 0; q < 8; ++q)
                                qmask[q] |= (bb[hh] >> 5) == q ? 1u << (bb[hh] & 31) : 0u;
                        }
                    }
                    int nm = 0;
                    uint32_t myw = 0u;
                    int myp = 0;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const uint32_t wq = __reduce_or_sync(kFull, qmask[q]);
                        if (lane == q) {
                            myw = wq;
                            myp = nm;
                        }
                        nm += __popc(wq);
                    }
                    if (lane < 8) {
                        SW[lane] = myw;
                        SP[lane] = myp;
                    }
                    for (int e = lane; e < nm; e += 32) {
                        LA[used + e] = 0.0f;
                        LA2[used + e] = 0.0f;
                        LK[used + e] = 0;
                    }
                    __syncwarp();
                    // per 32-row step, rows of the same bin add one rank at a time (row order)
#pragma unroll
                    for (int hh = 0; hh < kSmallRows; ++hh) {
                        if (hh * 32 < c) {
                            const int b = bb[hh];
                            const bool valid = b >= 0;
                            int e = 0;
                            if (valid) {
                                const int q = b >> 5;
                                e = used + SP[q] + __popc(SW[q] & ((1u << (b & 31)) - 1u));
                                LDB[e] = ((uint32_t)mv << 8) | (uint32_t)b |
                                         (e == used + nm - 1 ? kLastEntry : 0u);
                            }
                            const uint32_t peers = __match_any_sync(kFull, b);
                            const int rank = __popc(peers & ((1u << lane) - 1u));
                            const int maxr = __reduce_max_sync(kFull, valid ? __popc(peers) - 1 : 0);
                            for (int qq = 0; qq <= maxr; ++qq) {
                                if (valid && rank == qq) {
                                    LA[e] += v[hh] * 1.0f;
                                    LA2[e] += v2[hh] * 1.0f;
                                    LK[e] += 1;
                                }
                                __syncwarp();
                            }
                        }
                    }
                    if (lane == nd) {
                        my_off = used;
                        my_len = nm;
                    }
                    used += nm;
                    ++nd;
                    ++mv;
                }
                if (lane < nd)
                    regr_chains(LA + my_off, LA2 + my_off, LK + my_off, LR + my_off,
                                LR2 + my_off, my_len);
                __syncwarp();
                for (int e = lane; e < used; e += 32) {
                    const uint32_t db = LDB[e];
                    if (!(db & kLastEntry))
                        best = min(best, regr_key(LA[e], LR[e], LA2[e], LR2[e], LK[e], c, db));
                }
                __syncwarp();
            }
            best = warp_min_key(best);
        }
        if (lane == 0) B.nd_key[m] = best;
        __syncwarp();
    }
}

}  // namespace rfx
