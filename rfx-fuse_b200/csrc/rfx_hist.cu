// Histogram split search: histogram_find_best_split_classification / _regression
// (src/rf_growtree.cpp:22-184) and the per-node comparison across the mtry draws
// (src/rf_growtree.cpp:820-836, :929-955), for every searched node of a level at once.
//
// Three kernels share the work by node size:
//   k_hist_warp   nodes above the small-node limit: one block per (node, group of up to 16
//                 draws), one warp per drawn feature streaming the node's rows 32 at a time
//                 (bins and targets gathered from the packed rows, no block barriers);
//   k_hist_lane   regression nodes up to kLaneNode rows: one LANE per (node, drawn
//                 feature), several nodes per warp, the node's rows staged in shared memory
//                 once and every lane running its feature's histogram serially;
//   k_hist_small  classification nodes up to kSmallNode rows: one warp per node.
//
// Exactness.  Classification histograms are integer class counts (the reference's float
// counts are small integers).  Regression bin sums equal the reference's row-order serial
// float sums bin by bin: in k_hist_warp the rows of a 32-row step that share a bin are
// chained through register shuffles in row order and the last of them writes the bin back;
// in k_hist_lane one lane adds its feature's rows in row order.
//
// Winner key = (order-preserving bits of the criterion, draw index, bin); the smallest key
// over all draws of the node is the reference's choice (regression: lowest MSE, first draw
// wins ties; classification: highest 2 - gini, i.e. lowest -(2 - gini), first draw wins).
//
// Approximate-then-exact criterion.  The reference evaluates its float criterion (five or
// 2*nclass+1 IEEE divisions) at every bin.  Here every candidate bin first gets a cheap
// approximation (reciprocals, warp-parallel prefix sums) with a rigorous bound E on its
// distance from the reference's float value:
//   regression      |mse_f - mse_h| <= E = 1.25 (P + 2^-19 Q) with P the propagated error of
//                   the serial left/right float chains (recursive-summation bound
//                   (2m + 64) u sum|S|, u = 2^-24, m = non-empty bins) and Q the magnitude of
//                   the formula's terms (covers the rounding of both evaluations);
//   classification  |g_f - g_h| <= E = 1.5 (2 nclass + 16) u (every term <= 1).
// With U = min(g_h + E) over the node's draws, a bin whose g_h - E exceeds U (plus the width
// of one rounding of 2 - gini for classification, whose conversion can merge two values)
// cannot be the reference's choice; only the remaining candidates (usually one to three per
// node) get the exact float criterion, from the exact serial chains.
#include "rfx_device.cuh"
#include "rfx_kernels.h"

namespace rfx {

// bl[0..m) = ascending list of the non-empty bins (cnt[b] > 0).
__device__ __forceinline__ int warp_nonempty_bins(const int* cnt, uint8_t* bl, int lane) {
    int k = 0;
    uint32_t bits = 0;
    const int4 c0 = reinterpret_cast<const int4*>(cnt)[2 * lane];
    const int4 c1 = reinterpret_cast<const int4*>(cnt)[2 * lane + 1];
    const int cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int q = 0; q < 8; ++q)
        if (cc[q] > 0) { bits |= 1u << q; ++k; }
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

// The reference's gini for the left prefix counts lk = hp[k * 256] (k < nc), class totals
// tk[k], node rows c.
__device__ __forceinline__ float class_gini_exact(const int* hp, const int* tk, int nc, int c) {
    int tl = 0;
    for (int k = 0; k < nc; ++k) tl += hp[k * 256];
    const float tlf = (float)tl, trf = (float)(c - tl);
    float gl = 1.0f, gr = 1.0f;
    for (int k = 0; k < nc; ++k) {
        const int lk = hp[k * 256];
        const float pl = (float)lk / tlf;
        const float pr = (float)(tk[k] - lk) / trf;
        gl -= pl * pl;
        gr -= pr * pr;
    }
    const float tt = tlf + trf;
    return (tlf * gl + trf * gr) / tt;
}

__device__ __forceinline__ unsigned long long warp_min_key(unsigned long long k) {
    for (int o = 16; o > 0; o >>= 1) k = min(k, __shfl_xor_sync(kFull, k, o));
    return k;
}

__device__ __forceinline__ float warp_min_f(float x) {
    for (int o = 16; o > 0; o >>= 1) x = fminf(x, __shfl_xor_sync(kFull, x, o));
    return x;
}

__device__ __forceinline__ float warp_sum_f(float x) {
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

template <class T>
__device__ __forceinline__ T warp_incl_scan(T x, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    return x;
}

// ---------------------------------------------------------------------------------------
// k_hist_warp: nodes above kSmallNode rows.
//
// Per-warp shared memory (warp_bytes):
//   regression      SS float2[256] (bin sum, sum of squares) | KC int[256] | BL u8[256]
//                   (non-empty bins, ascending) | CF u8[256] (candidate flags) | TAG u32[256]
//                   (round tags, all-ones between steps)
//   classification  H int[nclass][256] (class-major counts, then inclusive prefixes) |
//                   KC int[256] | BL u8[256] | TK int[32] (class totals)
// ---------------------------------------------------------------------------------------
constexpr int kWarpUnroll = 4;  // 32-row steps whose loads are in flight together (regression)
constexpr int kWarpUnrollClass = 8;  // classification: rows mostly come from DRAM

template <bool REGR>
__device__ __forceinline__ void hist_warp(const Data& D, const Batch& B, int cur, const HistArgs& a,
                                          uint8_t* smem, unsigned* s_umin) {
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int nc = D.nclass;
    const int rs = D.rs, ro = D.ro;
    uint8_t* wbase = smem + (size_t)wib * a.warp_bytes;
    const int hbytes = REGR ? 2048 : 1024 * nc;
    float2* SS = reinterpret_cast<float2*>(wbase);
    int* H = reinterpret_cast<int*>(wbase);
    int* KC = reinterpret_cast<int*>(wbase + hbytes);
    uint8_t* BL = wbase + hbytes + 1024;
    uint8_t* CF = BL + 256;
    int* TK = reinterpret_cast<int*>(BL + 256);
    unsigned* TAG = reinterpret_cast<unsigned*>(BL + 512);  // regression: per-bin round tags
    if (REGR)
        for (int k = lane; k < 256; k += 32) TAG[k] = 0xffffffffu;
    if (threadIdx.x < 2) s_umin[threadIdx.x] = 0xffffffffu;
    __syncthreads();
    const int total = B.counters[4] * a.groups;
    int it = 0;
    for (int task = blockIdx.x; task < total; task += gridDim.x, ++it) {
        const int si = task / a.groups, grp = task - si * a.groups;
        const int4 rec = B.big_rec[si];  // {tree, node, start, rows}
        const int t = rec.x, node = rec.y, start = rec.z, c = rec.w;
        const size_t m = (size_t)t * B.M + node;
        const int* seg = B.seg[cur] + (size_t)t * D.N + start;
        const int mv = grp * a.warps + wib;
        const bool active = mv < B.mtry;
        unsigned* umin = &s_umin[it & 1];
        if (threadIdx.x == 0 && grp == 0 && B.hist_bytes)
            atomicAdd(B.hist_bytes, (unsigned long long)c * (unsigned long long)(B.mtry + (REGR ? 4 : 1)));
        float lo[8];
        int binq[8];
        int nm = 0;
        bool dense = false;
        const int f = active ? (int)B.feat[(size_t)t * B.M * B.mtry + (size_t)node * B.mtry + mv] : 0;
        if (active) {
            // ---- zero the histogram
            uint4* z = reinterpret_cast<uint4*>(wbase);
            const int words = (hbytes + 1024) / 16;
            for (int k = lane; k < words; k += 32) z[k] = make_uint4(0, 0, 0, 0);
            __syncwarp();
        }
        if (active) {
            // ---- accumulate, 32 rows per step in row order (bins and targets gathered from
            // the packed rows; the loads of kWarpUnroll steps in flight together)
            constexpr int kU = REGR ? kWarpUnroll : kWarpUnrollClass;
            for (int s0 = 0; s0 < c; s0 += 32 * kU) {
                int bb[kU];
                uint2 tg[kU];
                int r[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int i = s0 + u * 32 + lane;
                    r[u] = i < c ? __ldg(seg + i) : -1;
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    bb[u] = -1;
                    tg[u] = make_uint2(0, 0);
                    if (r[u] >= 0) {
                        const uint8_t* row = D.rows + (size_t)r[u] * rs;
                        bb[u] = (int)__ldg(row + f);
                        tg[u] = __ldg(reinterpret_cast<const uint2*>(row + ro));
                    }
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    if (s0 + u * 32 >= c) break;
                    const int b = bb[u];
                    const bool valid = b >= 0;
                    if (REGR) {
                        // rounds: in each, the lowest pending lane of every bin (the earliest
                        // row) adds its target; the bin's next row goes in the next round
                        const float v = __uint_as_float(tg[u].x), v2 = __uint_as_float(tg[u].y);
                        if (valid) atomicAdd(&KC[b], 1);
                        bool pend = valid;
                        int rounds = 0;
                        while (__any_sync(kFull, pend)) {
                            ++rounds;
                            if (pend) atomicMin(&TAG[b], (unsigned)lane);
                            __syncwarp();
                            const bool first = pend && TAG[b] == (unsigned)lane;
                            if (first) {
                                float2 h = SS[b];
                                h.x += v;
                                h.y += v2;
                                SS[b] = h;
                                TAG[b] = 0xffffffffu;
                            }
                            pend = pend && !first;
                            __syncwarp();
                        }
                        if (B.diag && lane == 0) {
                            atomicAdd(&B.diag[1], (unsigned long long)rounds);
                            atomicAdd(&B.diag[2], 1ull);
                        }
                    } else if (valid) {
                        atomicAdd(&H[(int)tg[u].x * 256 + b], 1);
                        atomicAdd(&KC[b], 1);
                    }
                }
            }
            __syncwarp();
            __syncwarp();
            nm = warp_nonempty_bins(KC, BL, lane);
            // ---- approximate criterion over the lane's entries: dense (bins 8*lane..+7)
            // or, for few non-empty bins, the lane's share of the compacted list
            dense = nm > 96;
            const int E = dense ? 8 : (nm + 31) >> 5;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                lo[q] = __int_as_float(0x7f800000);
                binq[q] = -1;
                if (q < E) {
                    if (dense) binq[q] = lane * 8 + q;
                    else if (lane * E + q < nm) binq[q] = BL[lane * E + q];
                }
            }
            float hmin = __int_as_float(0x7f800000);
            const float rtt = __frcp_rn((float)c);
            if (REGR) {
                float S[8], S2[8];
                int K[8];
                float ps = 0.0f, ps2 = 0.0f, sa = 0.0f;
                int pk = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    S[q] = S2[q] = 0.0f;
                    K[q] = 0;
                    if (binq[q] >= 0) {
                        const float2 h = SS[binq[q]];
                        S[q] = h.x;
                        S2[q] = h.y;
                        K[q] = KC[binq[q]];
                    }
                    sa += fabsf(S[q]);
                    ps += S[q];
                    ps2 += S2[q];
                    pk += K[q];
                    S[q] = ps;    // inclusive local prefixes from here on
                    S2[q] = ps2;
                    K[q] = K[q] > 0 ? pk : -1;  // -1: empty bin (never a candidate)
                }
                const float is = warp_incl_scan(ps, lane), is2 = warp_incl_scan(ps2, lane);
                const int ik = warp_incl_scan(pk, lane);
                const float es = is - ps, es2 = is2 - ps2;  // approximate exclusive prefixes
                const int ek = ik - pk;
                const float tot = __shfl_sync(kFull, is, 31), tot2 = __shfl_sync(kFull, is2, 31);
                const float A = warp_sum_f(sa);
                const float d = (float)(2 * nm + 64) * 0x1p-24f;
                const float dA = d * A, dA2 = d * fabsf(tot2) * 1.001f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (K[q] < 0) continue;
                    const int kc = ek + K[q];
                    if (kc >= c) continue;
                    const float Lh = es + S[q], L2h = es2 + S2[q];
                    const float Rh = tot - Lh, R2h = tot2 - L2h;
                    const float rcl = __frcp_rn((float)kc), rcr = __frcp_rn((float)(c - kc));
                    const float t1 = Lh * Lh * rcl, t2 = Rh * Rh * rcr, P = L2h + R2h;
                    const float mse = (P - t1 - t2) * rtt;
                    const float pert = (2.0f * dA2 + (2.0f * fabsf(Lh) + 3.0f * dA) * dA * rcl +
                                        (2.0f * fabsf(Rh) + 3.0f * dA) * dA * rcr) * rtt;
                    const float Q = (fabsf(P) + t1 + t2) * rtt + pert;
                    const float Eb = 1.25f * (pert + 0x1p-19f * Q) + 1e-30f;
                    lo[q] = mse - Eb;
                    hmin = fminf(hmin, mse + Eb);
                }
            } else {
                float SL[8], SR[8];
                int kc[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) { SL[q] = SR[q] = 0.0f; kc[q] = 0; }
                for (int k = 0; k < nc; ++k) {
                    int hv[8];
                    int pk = 0;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        hv[q] = binq[q] >= 0 ? H[k * 256 + binq[q]] : 0;
                        pk += hv[q];
                        hv[q] = pk;
                    }
                    const int ik = warp_incl_scan(pk, lane);
                    const int ek = ik - pk;
                    const int tk = __shfl_sync(kFull, ik, 31);
                    if (lane == 0) TK[k] = tk;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int lk = ek + hv[q];
                        const float fl = (float)lk, fr = (float)(tk - lk);
                        SL[q] += fl * fl;
                        SR[q] += fr * fr;
                        kc[q] += lk;
                        if (binq[q] >= 0) H[k * 256 + binq[q]] = lk;  // left prefix, in place
                    }
                }
                const float Ec = 1.5f * (float)(2 * nc + 16) * 0x1p-24f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (binq[q] < 0 || KC[binq[q]] == 0 || kc[q] >= c) continue;
                    const float rcl = __frcp_rn((float)kc[q]), rcr = __frcp_rn((float)(c - kc[q]));
                    const float g = 1.0f - (SL[q] * rcl + SR[q] * rcr) * rtt;
                    lo[q] = g - Ec;
                    hmin = fminf(hmin, g + Ec);
                }
            }
            hmin = warp_min_f(hmin);
            if (lane == 0 && hmin < __int_as_float(0x7f800000)) atomicMin(umin, ord_of(hmin));
        }
        __syncthreads();
        if (threadIdx.x == 0) s_umin[(it + 1) & 1] = 0xffffffffu;
        if (!active) continue;
        const unsigned uo = *umin;
        if (uo == 0xffffffffu) continue;
        const float thr = REGR ? float_of(uo) : float_of(uo) + 0x1p-21f;
        // ---- exact criterion for the candidates
        bool any = false;
        int bmax = -1;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const bool cq = binq[q] >= 0 && lo[q] <= thr;
            if (REGR && binq[q] >= 0) CF[binq[q]] = cq ? 1 : 0;
            if (cq) { any = true; bmax = max(bmax, binq[q]); }
        }
        if (!__any_sync(kFull, any)) continue;
        if (REGR) {
            bmax = __reduce_max_sync(kFull, (unsigned)(bmax + 1)) - 1;
            __syncwarp();
            if (lane == 0) {
                // the reference's serial chains over the non-empty bins (empty bins add +0)
                float tot = 0.0f, tot2 = 0.0f;
                int j = 0;
                for (; j + 8 <= nm; j += 8) {
                    float2 h[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) h[u] = SS[BL[j + u]];
#pragma unroll
                    for (int u = 0; u < 8; ++u) { tot += h[u].x; tot2 += h[u].y; }
                }
                for (; j < nm; ++j) {
                    const float2 h = SS[BL[j]];
                    tot += h.x;
                    tot2 += h.y;
                }
                float L = 0.0f, R = tot, L2 = 0.0f, R2 = tot2;
                int kc = 0;
                unsigned long long best = kNoKey;
                for (j = 0; j < nm; ++j) {
                    const int b = BL[j];
                    if (b > bmax) break;
                    const float2 h = SS[b];
                    kc += KC[b];
                    L += h.x;
                    R -= h.x;
                    L2 += h.y;
                    R2 -= h.y;
                    if (CF[b]) {
                        best = min(best, regr_key(L, R, L2, R2, kc, c, ((uint32_t)mv << 8) | (uint32_t)b));
                        if (B.diag) atomicAdd(&B.diag[0], 1ull);
                    }
                }
                if (best != kNoKey) atomicMin(&B.nd_key[m], best);
            }
            __syncwarp();
        } else {
            unsigned long long kb = kNoKey;  // (gini bits, bin): the draw's first minimum
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (binq[q] >= 0 && lo[q] <= thr) {
                    const float g = class_gini_exact(H + binq[q], TK, nc, c);
                    kb = min(kb, ((unsigned long long)ord_of(g) << 32) | (unsigned long long)binq[q]);
                }
            }
            kb = warp_min_key(kb);
            if (lane == 0 && kb != kNoKey) {
                const float g = float_of((uint32_t)(kb >> 32));
                const unsigned long long key = ((unsigned long long)ord_of(-(2.0f - g)) << 32) |
                                               ((unsigned long long)mv << 8) | (kb & 0xffull);
                atomicMin(&B.nd_key[m], key);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// k_hist_pipe: regression nodes above kLaneNode rows, warp-specialised.  A block takes one
// searched node and up to `warps` of its draws.  Warp 0 (producer) streams the node's packed
// rows into a ring of kPipeBufs chunks of `ch` rows in shared memory (16-byte cp.async; row
// stride rs + 16 bytes, the 16-byte multiple that spreads 32 consecutive rows over the most
// banks: a lane reading one byte of its row meets at most 3 others in its bank); warps
// 1..warps (consumers) each build one drawn feature's
// histogram from the staged rows, 32 rows per step, in the conflict rounds of k_hist_warp.
// Chunks are handed over with mbarriers (full: the producer's copies have landed; empty:
// every consumer is done with the buffer), so the producer runs up to kPipeBufs - 1 chunks
// ahead and no block-wide barrier sits in the row loop.  One histogram entry per bin,
// HE[bin] = {sum, sum of squares, count, round tag}: a round's read and write are one 16-byte
// access each.  Every wait is bounded (about one second); on expiry the block records
// counters[3] and returns after its own copies have landed.
//
// Shared memory: mbarriers full[kPipeBufs], empty[kPipeBufs] | umin[kPipeBounds] | ring
// [kPipeBufs][ch][rs + 16] | per consumer HE float4[256] | BL u8[256] | CF u8[256].
// ---------------------------------------------------------------------------------------
// Slots of the per-node bound (the consumers of one block are at most kPipeBufs chunks, so
// at most kPipeBufs tasks, apart).
constexpr int kPipeBounds = 16;
static_assert(kPipeBounds / 2 >= kPipeBufs, "bound slots must cover the consumers' skew");
static_assert(16 * kPipeBufs + 4 * kPipeBounds <= kPipeHead, "k_hist_pipe header");
constexpr int kPipeDraw = 256 * 16 + 512;  // shared memory per consumer warp
constexpr unsigned long long kPipeWaitNs = 1000000000ull;

__device__ __forceinline__ unsigned pipe_smem(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long pipe_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void pipe_init(uint64_t* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(pipe_smem(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool pipe_wait(uint64_t* b, unsigned parity) {
    const unsigned a = pipe_smem(b);
    const unsigned long long t0 = pipe_now();
    for (unsigned spin = 1;; ++spin) {
        unsigned ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((spin & 63u) == 0 && pipe_now() - t0 > kPipeWaitNs) return false;
    }
}
__device__ __forceinline__ void pipe_arrive(uint64_t* b) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(pipe_smem(b))
                 : "memory");
}
__device__ __forceinline__ void pipe_copy16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(pipe_smem(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void pipe_arrive_on_copies(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(pipe_smem(b)) : "memory");
}
__device__ __forceinline__ void pipe_wait_copies() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(544, 2) k_hist_pipe(Data D, Batch B, int cur, PipeArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kPipeBufs;
    unsigned* s_umin = reinterpret_cast<unsigned*>(smem + 16 * kPipeBufs);  // [kPipeBounds]
    uint8_t* ring = smem + kPipeHead;
    const int ch = a.ch, RS = a.rstride, W = a.warps;
    uint8_t* dbase = ring + (size_t)kPipeBufs * ch * RS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rs = D.rs, ro = D.ro, pieces = rs >> 4;
    if (threadIdx.x == 0) {
        for (int b = 0; b < kPipeBufs; ++b) {
            pipe_init(&full[b], 32);
            pipe_init(&empty[b], W);
        }
        for (int k = 0; k < kPipeBounds; ++k) s_umin[k] = 0xffffffffu;
    }
    __syncthreads();
    const int total = B.counters[4] * a.groups;
    long long g = 0;  // chunk counter, identical sequence in every warp
    if (warp == 0) {
        // ---- producer: lane l copies rows l and l + 32 of each chunk (16-byte pieces), in
        // one flat sequence of chunks over the block's tasks.  The row ids of the chunk three
        // ahead load while this chunk's copies issue (and the record of the task after the
        // furthest one is loaded a task ahead), so the copies never wait on an id load.
        auto rec_of = [&](int task) {
            return task < total ? B.big_rec[task / a.groups] : make_int4(0, 0, 0, 0);
        };
        auto ids = [&](const int4& r, int c0, int& q0, int& q1) {
            const int n = min(ch, r.w - c0);
            const int* seg = B.seg[cur] + (size_t)r.x * D.N + r.z + c0;
            q0 = lane < n ? __ldg(seg + lane) : -1;
            q1 = lane + 32 < n ? __ldg(seg + 32 + lane) : -1;
        };
        // chunk positions: (task, first row, record); `after` = record of the task that
        // follows the furthest position's task
        int t0 = blockIdx.x, c00 = 0;
        int4 rc0 = rec_of(t0);
        int4 after = rec_of(t0 + (int)gridDim.x);
        auto advance = [&](int& t, int& c, int4& r) {
            c += ch;
            if (c >= r.w) {
                t += gridDim.x;
                c = 0;
                r = after;
                after = rec_of(t + (int)gridDim.x);
            }
        };
        int t1 = t0, c1 = c00, t2, c2;
        int4 rc1 = rc0, rc2;
        int r0 = -1, r1 = -1, q0 = -1, q1 = -1, s0 = -1, s1 = -1;
        if (t0 < total) ids(rc0, 0, r0, r1);
        advance(t1, c1, rc1);
        if (t1 < total) ids(rc1, c1, q0, q1);
        t2 = t1; c2 = c1; rc2 = rc1;
        advance(t2, c2, rc2);
        if (t2 < total) ids(rc2, c2, s0, s1);
        while (t0 < total) {
            int t3 = t2, c3 = c2;
            int4 rc3 = rc2;
            advance(t3, c3, rc3);
            int u0 = -1, u1 = -1;
            if (t3 < total) ids(rc3, c3, u0, u1);
            const int b = (int)(g % kPipeBufs);
            const long long u = g / kPipeBufs;
            if (u > 0 && !pipe_wait(&empty[b], (unsigned)((u - 1) & 1))) {
                atomicExch(&B.counters[3], 1);
                pipe_wait_copies();
                return;
            }
            uint8_t* dst = ring + (size_t)b * ch * RS + (size_t)lane * RS;
            if (r0 >= 0) {
                const uint8_t* src = D.rows + (size_t)r0 * rs;
                for (int pc = 0; pc < pieces; ++pc) pipe_copy16(dst + 16 * pc, src + 16 * pc);
            }
            if (r1 >= 0) {
                const uint8_t* src = D.rows + (size_t)r1 * rs;
                for (int pc = 0; pc < pieces; ++pc)
                    pipe_copy16(dst + (size_t)32 * RS + 16 * pc, src + 16 * pc);
            }
            pipe_arrive_on_copies(&full[b]);
            ++g;
            t0 = t1; t1 = t2; t2 = t3;
            c1 = c2; c2 = c3;
            rc1 = rc2; rc2 = rc3;
            r0 = q0; r1 = q1;
            q0 = s0; q1 = s1;
            s0 = u0; s1 = u1;
        }
        pipe_wait_copies();
        return;
    }
    // ---- consumers
    const int cw = warp - 1;
    float4* HE = reinterpret_cast<float4*>(dbase + (size_t)cw * kPipeDraw);
    uint8_t* BL = dbase + (size_t)cw * kPipeDraw + 4096;
    uint8_t* CF = BL + 256;
    const float tag0 = __uint_as_float(0xffffffffu);
    int it = 0;
    // the drawn feature of a task (-1: this warp has no draw in it)
    auto feat_of = [&](int task, const int4& r) {
        const int mv_ = (task - (task / a.groups) * a.groups) * W + cw;
        return (task < total && mv_ < B.mtry)
                   ? (int)B.feat[(size_t)r.x * B.M * B.mtry + (size_t)r.y * B.mtry + mv_] : -1;
    };
    int4 nrec = blockIdx.x < total ? B.big_rec[blockIdx.x / a.groups] : make_int4(0, 0, 0, 0);
    int nf = feat_of(blockIdx.x, nrec);
    for (int task = blockIdx.x; task < total; task += gridDim.x, ++it) {
        const int4 rec = nrec;  // {tree, node, start, rows}; the next task's is prefetched
        const int fcur = nf;
        if (task + (int)gridDim.x < total) {
            nrec = B.big_rec[(task + gridDim.x) / a.groups];
            nf = feat_of(task + gridDim.x, nrec);
        }
        const int t = rec.x, node = rec.y, c = rec.w;
        const int grp = task - (task / a.groups) * a.groups;
        const size_t m = (size_t)t * B.M + node;
        const int mv = grp * W + cw;
        const bool active = mv < B.mtry;
        const int f = active ? fcur : 0;
        unsigned* umin = &s_umin[it % kPipeBounds];
        // the slot of task it + kPipeBounds / 2 starts empty: no consumer is that far ahead
        // of consumer 0, nor still on the task that used it before
        if (cw == 0 && lane == 0) s_umin[(it + kPipeBounds / 2) % kPipeBounds] = 0xffffffffu;
        if (cw == 0 && lane == 0 && grp == 0 && B.hist_bytes)
            atomicAdd(B.hist_bytes, (unsigned long long)c * (unsigned long long)(B.mtry + 4));
        for (int k = lane; k < 256; k += 32) HE[k] = make_float4(0.0f, 0.0f, 0.0f, tag0);
        __syncwarp();
        for (int c0 = 0; c0 < c; c0 += ch, ++g) {
            const int b = (int)(g % kPipeBufs);
            if (!pipe_wait(&full[b], (unsigned)((g / kPipeBufs) & 1))) {
                atomicExch(&B.counters[3], 1);
                return;
            }
            if (active) {
                const int n = min(ch, c - c0);
                const uint8_t* buf = ring + (size_t)b * ch * RS;
                for (int s0 = 0; s0 < n; s0 += 32) {
                    const int i = s0 + lane;
                    const bool valid = i < n;
                    const uint8_t* row = buf + (size_t)(valid ? i : 0) * RS;
                    const int bn = valid ? (int)row[f] : 0;
                    const float2 vv = valid ? *reinterpret_cast<const float2*>(row + ro)
                                            : make_float2(0.0f, 0.0f);
                    const float v = vv.x, v2 = vv.y;
                    // rounds: the lowest pending lane of every bin (the earliest row) adds
                    bool pend = valid;
                    while (__any_sync(kFull, pend)) {
                        if (pend) atomicMin(reinterpret_cast<unsigned*>(&HE[bn].w), (unsigned)lane);
                        __syncwarp();
                        bool first = false;
                        float4 h;
                        if (pend) {
                            h = HE[bn];
                            first = __float_as_uint(h.w) == (unsigned)lane;
                        }
                        if (first) {
                            h.x += v;
                            h.y += v2;
                            h.z += 1.0f;
                            h.w = tag0;
                            HE[bn] = h;
                        }
                        pend = pend && !first;
                        __syncwarp();
                    }
                }
            }
            __syncwarp();
            if (lane == 0) pipe_arrive(&empty[b]);
        }
        // ---- approximate criterion (k_hist_warp's, over HE)
        float lo[8];
        int binq[8];
        int nm = 0;
        unsigned own = 0xffffffffu;
        if (active) {
            {
                int k = 0;
                uint32_t bits = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    if (HE[lane * 8 + q].z > 0.0f) { bits |= 1u << q; ++k; }
                const int x = warp_incl_scan(k, lane);
                int off = x - k;
                while (bits) {
                    const int q = __ffs(bits) - 1;
                    bits &= bits - 1;
                    BL[off++] = (uint8_t)(lane * 8 + q);
                }
                nm = __shfl_sync(kFull, x, 31);
                __syncwarp();
            }
            const bool dense = nm > 96;
            const int E = dense ? 8 : (nm + 31) >> 5;
            float S[8], S2[8];
            int K[8];
            float ps = 0.0f, ps2 = 0.0f, sa = 0.0f;
            int pk = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                lo[q] = __int_as_float(0x7f800000);
                binq[q] = -1;
                if (q < E) {
                    if (dense) binq[q] = lane * 8 + q;
                    else if (lane * E + q < nm) binq[q] = BL[lane * E + q];
                }
                S[q] = S2[q] = 0.0f;
                K[q] = 0;
                if (binq[q] >= 0) {
                    const float4 h = HE[binq[q]];
                    S[q] = h.x;
                    S2[q] = h.y;
                    K[q] = (int)h.z;
                }
                sa += fabsf(S[q]);
                ps += S[q];
                ps2 += S2[q];
                pk += K[q];
                S[q] = ps;
                S2[q] = ps2;
                K[q] = K[q] > 0 ? pk : -1;
            }
            const float is = warp_incl_scan(ps, lane), is2 = warp_incl_scan(ps2, lane);
            const int ik = warp_incl_scan(pk, lane);
            const float es = is - ps, es2 = is2 - ps2;
            const int ek = ik - pk;
            const float tot = __shfl_sync(kFull, is, 31), tot2 = __shfl_sync(kFull, is2, 31);
            const float A = warp_sum_f(sa);
            const float d = (float)(2 * nm + 64) * 0x1p-24f;
            const float dA = d * A, dA2 = d * fabsf(tot2) * 1.001f;
            const float rtt = __frcp_rn((float)c);
            float hmin = __int_as_float(0x7f800000);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (K[q] < 0) continue;
                const int kc = ek + K[q];
                if (kc >= c) continue;
                const float Lh = es + S[q], L2h = es2 + S2[q];
                const float Rh = tot - Lh, R2h = tot2 - L2h;
                const float rcl = __frcp_rn((float)kc), rcr = __frcp_rn((float)(c - kc));
                const float t1 = Lh * Lh * rcl, t2 = Rh * Rh * rcr, P = L2h + R2h;
                const float mse = (P - t1 - t2) * rtt;
                const float pert = (2.0f * dA2 + (2.0f * fabsf(Lh) + 3.0f * dA) * dA * rcl +
                                    (2.0f * fabsf(Rh) + 3.0f * dA) * dA * rcr) * rtt;
                const float Q = (fabsf(P) + t1 + t2) * rtt + pert;
                const float Eb = 1.25f * (pert + 0x1p-19f * Q) + 1e-30f;
                lo[q] = mse - Eb;
                hmin = fminf(hmin, mse + Eb);
            }
            hmin = warp_min_f(hmin);
            if (lane == 0 && hmin < __int_as_float(0x7f800000)) atomicMin(umin, ord_of(hmin));
            own = hmin < __int_as_float(0x7f800000) ? ord_of(hmin) : 0xffffffffu;
        }
        // The threshold: this draw's bound and the smallest bound the node's other draws have
        // posted so far (each is an upper bound of the node's best criterion, so the best
        // split stays a candidate of its own draw whatever the others have posted).  No
        // consumer waits for the others.
        __syncwarp();
        if (!active) continue;
        const unsigned uo = min(own, __shfl_sync(kFull, *reinterpret_cast<volatile unsigned*>(umin), 0));
        if (uo == 0xffffffffu) continue;
        const float thr = float_of(uo);
        bool any = false;
        int bmax = -1;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const bool cq = binq[q] >= 0 && lo[q] <= thr;
            if (binq[q] >= 0) CF[binq[q]] = cq ? 1 : 0;
            if (cq) { any = true; bmax = max(bmax, binq[q]); }
        }
        if (!__any_sync(kFull, any)) continue;
        bmax = __reduce_max_sync(kFull, (unsigned)(bmax + 1)) - 1;
        __syncwarp();
        if (lane == 0) {
            // the reference's serial chains over the non-empty bins (empty bins add +0); the
            // entries of 4 bins are loaded ahead of their additions (the order of the float
            // additions is unchanged)
            float tot = 0.0f, tot2 = 0.0f;
            for (int j0 = 0; j0 < nm; j0 += 4) {
                float hx[4], hy[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 h = j0 + u < nm ? HE[BL[j0 + u]] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    hx[u] = h.x;
                    hy[u] = h.y;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (j0 + u < nm) {
                        tot += hx[u];
                        tot2 += hy[u];
                    }
                }
            }
            float L = 0.0f, R = tot, L2 = 0.0f, R2 = tot2;
            int kc = 0;
            unsigned long long best = kNoKey;
            const int jend = nm;  // entries past bmax are skipped below
            for (int j0 = 0; j0 < jend; j0 += 4) {
                int bq[4];
                float hx[4], hy[4], hz[4];
                bool cf[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    bq[u] = j0 + u < nm ? (int)BL[j0 + u] : 256;
                    const bool in = bq[u] <= bmax;
                    const float4 h = in ? HE[bq[u]] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    hx[u] = h.x;
                    hy[u] = h.y;
                    hz[u] = h.z;
                    cf[u] = in && CF[bq[u]];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (bq[u] <= bmax) {
                        kc += (int)hz[u];
                        L += hx[u];
                        R -= hx[u];
                        L2 += hy[u];
                        R2 -= hy[u];
                        if (cf[u]) {
                            best = min(best, regr_key(L, R, L2, R2, kc, c, ((uint32_t)mv << 8) | (uint32_t)bq[u]));
                            if (B.diag) atomicAdd(&B.diag[0], 1ull);
                        }
                    }
                }
                if (bq[3] >= bmax) break;  // bins ascend: nothing after bmax
            }
            if (best != kNoKey) atomicMin(&B.nd_key[m], best);
        }
        __syncwarp();
    }
}

__global__ void __launch_bounds__(512, 2) k_hist_warp_regr(Data D, Batch B, int cur, HistArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ unsigned s_umin[2];
    hist_warp<true>(D, B, cur, a, smem, s_umin);
}

__global__ void __launch_bounds__(512, 1) k_hist_warp_class(Data D, Batch B, int cur, HistArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ unsigned s_umin[2];
    hist_warp<false>(D, B, cur, a, smem, s_umin);
}

// ---------------------------------------------------------------------------------------
// k_hist_lane: regression nodes of at most kLaneNode rows.  A warp takes `slots` nodes of
// the level's small list; lane = slot * mtry + draw.  The nodes' rows (drawn bins and
// targets) are staged in shared memory by the whole warp, then every lane builds its draw's
// histogram as a list of the non-empty bins (a 256-bit set gives each bin its list index),
// adding its rows in row order, and runs the reference's serial chains over the list.
//
// Filter.  With the exact chain values L, R (left/right sums), the reference's MSE times
// the node size is P - G + d, where P = L2 + R2 is within 2m u T2 of T2 = sum of the node's
// squared targets (m <= kLaneNode list entries), G = L^2/cl + R^2/cr, and |d| <= 16.1 u T2
// (rounding of the float formula; G <= P).  The approximation G_h (hardware reciprocals) is
// within 5.1 u T2 of G.  So the reference's choice has G_h >= max G_h - 2 (2 kLaneNode + 22) u T2
// over all draws of the node; only those entries get the exact criterion (kLaneWin is that
// bound times 1.25, rounded up).
//
// Per-warp shared memory (lane_bytes(slots)):
//   LS float2[kLaneNode][32] (bin sum, sum of squares) | LK u8[kLaneNode][32] (counts) |
//   BM u32[8][32] (bin sets) | BS u32[8][32] (list index of each set word) |
//   TL u8[32][kLaneTile] (bins, lane-major) | TG float2[slots][kLaneNode] (targets) |
//   UM u32[kLaneSlots] (ordered max G_h per node)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// NODE: the largest node of the instantiation; part 0 takes sml_rec [0, counters[20]) (nodes
// of at most kLaneTiny rows), part 1 sml2_rec [0, counters[22]) (up to kLaneSmall rows),
// part 2 the last counters[21] records of sml_rec (up to kLaneNode rows).
template <int NODE>
__device__ __forceinline__ void hist_lane(const Data& D, const Batch& B, int cur, int slots, int part) {
    constexpr int kLaneTile = lane_tile(NODE);
    constexpr int kLaneH = NODE / 32;  // rows per lane when staging a node
    constexpr float kLaneWin = (float)((5 * (2 * NODE + 22) + 1) / 2 + 8) * 0x1p-24f;
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x;
    float2* LS = reinterpret_cast<float2*>(smem);
    uint8_t* LK = smem + NODE * 32 * 8;
    uint32_t* BM = reinterpret_cast<uint32_t*>(LK + NODE * 32);
    uint32_t* BS = BM + 256;
    uint8_t* TL = reinterpret_cast<uint8_t*>(BS + 256);
    float2* TG = reinterpret_cast<float2*>(TL + 32 * kLaneTile);
    unsigned* UM = reinterpret_cast<unsigned*>(TG + slots * NODE);
    const int mtry = B.mtry, rs = D.rs, ro = D.ro;
    const int4* recs = part == 1 ? B.sml2_rec : B.sml_rec;
    const int first = part == 2 ? B.counters[6] - B.counters[21] : 0;
    const int total = part == 0 ? B.counters[20] : part == 1 ? B.counters[22] : B.counters[6];
    const int slot = lane / mtry, d = lane - slot * mtry;
    const bool lane_on = slot < slots;
    const uint8_t* tl = TL + lane * kLaneTile;
    for (int g0 = first + blockIdx.x * slots; g0 < total; g0 += gridDim.x * slots) {
        int my_t = 0, my_node = 0, my_c = 0, my_start = 0;
        if (lane < slots && g0 + lane < total) {
            const int4 rec = recs[g0 + lane];  // {tree, node, start, rows}
            my_t = rec.x;
            my_node = rec.y;
            my_start = rec.z;
            my_c = rec.w;
        }
        if (lane < slots) UM[lane] = 0u;
        // ---- stage: lanes take rows, every drawn feature's bin and the target (row ids of
        // all slots first, so that their loads are in flight together)
        int rid[kLaneH * kLaneSlots];
#pragma unroll
        for (int s = 0; s < kLaneSlots; ++s) {
#pragma unroll
            for (int h = 0; h < kLaneH; ++h) rid[kLaneH * s + h] = -1;
            if (s < slots) {
                const int c = __shfl_sync(kFull, my_c, s);
                const int t = __shfl_sync(kFull, my_t, s);
                const int start = __shfl_sync(kFull, my_start, s);
                const int* seg = B.seg[cur] + (size_t)t * D.N + start;
#pragma unroll
                for (int h = 0; h < kLaneH; ++h)
                    if (lane + 32 * h < c) rid[kLaneH * s + h] = __ldg(seg + lane + 32 * h);
            }
        }
#pragma unroll
        for (int s = 0; s < kLaneSlots; ++s) {
            if (s >= slots) break;
            const int c = __shfl_sync(kFull, my_c, s);
            if (c == 0) continue;
            const int t = __shfl_sync(kFull, my_t, s), node = __shfl_sync(kFull, my_node, s);
            const uint16_t* featp = B.feat + (size_t)t * B.M * mtry + (size_t)node * mtry;
            const int fl = lane < mtry ? (int)featp[lane] : 0;
            if (lane == 0 && B.hist_bytes)
                atomicAdd(B.hist_bytes, (unsigned long long)c * (unsigned long long)(mtry + 4));
#pragma unroll
            for (int h = 0; h < kLaneH; ++h) {
                if (h * 32 >= c) break;
                const int i = h * 32 + lane;
                const bool ok = rid[kLaneH * s + h] >= 0;
                const uint8_t* row = D.rows + (ok ? (size_t)rid[kLaneH * s + h] * rs : 0);
                if (ok) TG[s * NODE + i] = __ldg(reinterpret_cast<const float2*>(row + ro));
                uint8_t* dst = TL + (s * mtry) * kLaneTile + i;
                for (int dd = 0; dd < mtry; ++dd) {
                    const int fd = __shfl_sync(kFull, fl, dd);
                    if (ok) dst[dd * kLaneTile] = __ldg(row + fd);
                }
            }
        }
        __syncwarp();
        const int sl = lane_on ? slot : 0;
        const int cs = __shfl_sync(kFull, my_c, sl);
        const int c = lane_on ? cs : 0;
        const int t = __shfl_sync(kFull, my_t, sl);
        const int node = __shfl_sync(kFull, my_node, sl);
        const float2* tg = TG + sl * NODE;
        // ---- bin set and list indices
#pragma unroll
        for (int q = 0; q < 8; ++q) BM[q * 32 + lane] = 0u;
        for (int i = 0; i < c; ++i) {
            const int b = tl[i];
            BM[(b >> 5) * 32 + lane] |= 1u << (b & 31);
        }
        int nm = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            BS[q * 32 + lane] = (uint32_t)nm;
            nm += __popc(BM[q * 32 + lane]);
        }
        for (int j = 0; j < nm; ++j) {
            LS[j * 32 + lane] = make_float2(0.0f, 0.0f);
            LK[j * 32 + lane] = 0;
        }
        auto entry = [&](int b) -> int {
            const int q = b >> 5;
            return (int)BS[q * 32 + lane] + __popc(BM[q * 32 + lane] & ((1u << (b & 31)) - 1u));
        };
        // ---- histogram in row order, four rows at a time (equal entries forwarded)
        int i = 0;
        for (; i + 4 <= c; i += 4) {
            const uint32_t bw = *reinterpret_cast<const uint32_t*>(tl + i);
            const int e0 = entry(bw & 0xff), e1 = entry((bw >> 8) & 0xff);
            const int e2 = entry((bw >> 16) & 0xff), e3 = entry(bw >> 24);
            const float2 y0 = tg[i], y1 = tg[i + 1], y2 = tg[i + 2], y3 = tg[i + 3];
            const float2 a0 = LS[e0 * 32 + lane], a1 = LS[e1 * 32 + lane];
            const float2 a2 = LS[e2 * 32 + lane], a3 = LS[e3 * 32 + lane];
            const int k0 = LK[e0 * 32 + lane], k1 = LK[e1 * 32 + lane];
            const int k2 = LK[e2 * 32 + lane], k3 = LK[e3 * 32 + lane];
            const float2 n0 = make_float2(a0.x + y0.x, a0.y + y0.y);
            const int m0 = k0 + 1;
            const bool f10 = e1 == e0;
            const float2 b1 = f10 ? n0 : a1;
            const float2 n1 = make_float2(b1.x + y1.x, b1.y + y1.y);
            const int m1 = (f10 ? m0 : k1) + 1;
            const bool f21 = e2 == e1, f20 = e2 == e0;
            const float2 b2 = f21 ? n1 : (f20 ? n0 : a2);
            const float2 n2 = make_float2(b2.x + y2.x, b2.y + y2.y);
            const int m2 = (f21 ? m1 : (f20 ? m0 : k2)) + 1;
            const bool f32 = e3 == e2, f31 = e3 == e1, f30 = e3 == e0;
            const float2 b3 = f32 ? n2 : (f31 ? n1 : (f30 ? n0 : a3));
            const float2 n3 = make_float2(b3.x + y3.x, b3.y + y3.y);
            const int m3 = (f32 ? m2 : (f31 ? m1 : (f30 ? m0 : k3))) + 1;
            LS[e0 * 32 + lane] = n0;
            LK[e0 * 32 + lane] = (uint8_t)m0;
            LS[e1 * 32 + lane] = n1;
            LK[e1 * 32 + lane] = (uint8_t)m1;
            LS[e2 * 32 + lane] = n2;
            LK[e2 * 32 + lane] = (uint8_t)m2;
            LS[e3 * 32 + lane] = n3;
            LK[e3 * 32 + lane] = (uint8_t)m3;
        }
        for (; i < c; ++i) {
            const int e = entry(tl[i]);
            const float2 a = LS[e * 32 + lane];
            const float2 y = tg[i];
            LS[e * 32 + lane] = make_float2(a.x + y.x, a.y + y.y);
            LK[e * 32 + lane] = (uint8_t)(LK[e * 32 + lane] + 1);
        }
        // ---- the reference's chains: totals, then left/right sums with G_h
        float tot = 0.0f, tot2 = 0.0f;
        for (int j = 0; j < nm; ++j) {
            const float2 e = LS[j * 32 + lane];
            tot += e.x;
            tot2 += e.y;
        }
        float gmax = -1.0f;
        {
            float L = 0.0f, R = tot;
            int kc = 0;
            for (int j = 0; j < nm - 1; ++j) {
                const float S = LS[j * 32 + lane].x;
                kc += LK[j * 32 + lane];
                L += S;
                R -= S;
                const float G = L * L * rcp_approx((float)kc) + R * R * rcp_approx((float)(c - kc));
                gmax = fmaxf(gmax, G);
            }
        }
        if (lane_on && gmax >= 0.0f) atomicMax(&UM[slot], ord_of(gmax));
        __syncwarp();
        const unsigned um = lane_on ? UM[slot] : 0u;
        const float thr = um ? float_of(um) - kLaneWin * tot2 : 0.0f;
        if (um != 0u && gmax >= thr) {
            float L = 0.0f, R = tot, L2 = 0.0f, R2 = tot2;
            int kc = 0;
            unsigned long long best = kNoKey;
            for (int j = 0; j < nm - 1; ++j) {
                const float2 e = LS[j * 32 + lane];
                kc += LK[j * 32 + lane];
                L += e.x;
                R -= e.x;
                L2 += e.y;
                R2 -= e.y;
                const float G = L * L * rcp_approx((float)kc) + R * R * rcp_approx((float)(c - kc));
                if (G >= thr) {
                    // bin of list entry j: the (j - BS[q])-th set bit of word q
                    int q = 0;
                    while (q < 7 && (int)BS[(q + 1) * 32 + lane] <= j) ++q;
                    uint32_t w = BM[q * 32 + lane];
                    for (int k = j - (int)BS[q * 32 + lane]; k > 0; --k) w &= w - 1u;
                    const int b = q * 32 + __ffs(w) - 1;
                    best = min(best, regr_key(L, R, L2, R2, kc, c, ((uint32_t)d << 8) | (uint32_t)b));
                    if (B.diag) atomicAdd(&B.diag[0], 1ull);
                }
            }
            if (best != kNoKey) atomicMin(&B.nd_key[(size_t)t * B.M + node], best);
        }
        __syncwarp();
    }
}

__global__ void __launch_bounds__(32) k_hist_lane_tiny(Data D, Batch B, int cur, int slots) {
    hist_lane<kLaneTiny>(D, B, cur, slots, 0);
}
__global__ void __launch_bounds__(32) k_hist_lane(Data D, Batch B, int cur, int slots) {
    hist_lane<kLaneSmall>(D, B, cur, slots, 1);
}
__global__ void __launch_bounds__(32) k_hist_lane_mid(Data D, Batch B, int cur, int slots) {
    hist_lane<kLaneNode>(D, B, cur, slots, 2);
}

// ---------------------------------------------------------------------------------------
// k_hist_small: classification nodes of at most kSmallNode rows, one warp per searched
// node doing all mtry draws.  Each lane holds up to two of the node's rows (address and
// label in registers) and reads the drawn feature's bin directly from the packed row; the
// draw's bins form a 256-bit set ranking each row's bin, class counts go to the ranked
// entries, and per-class warp scans give the prefixes of the criterion.
// Per-warp scratch: bl u8[256] | set words + rank offsets (16 words) | h int[(256+1) nclass]
// ---------------------------------------------------------------------------------------
constexpr int kSmallRows = kSmallNode / 32;  // rows per lane in k_hist_small

__global__ void __launch_bounds__(256) k_hist_small(Data D, Batch B, int cur, int warp_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int nc = D.nclass;
    const int rs = D.rs, ro = D.ro;
    uint8_t* wbase = smem + (size_t)wib * warp_bytes;
    uint8_t* bl = wbase;
    uint32_t* CW = reinterpret_cast<uint32_t*>(wbase + 256);
    int* CP = reinterpret_cast<int*>(CW + 8);
    int* h = reinterpret_cast<int*>(CW + 16);
    for (int k = lane; k < warp_bytes / 4; k += 32) reinterpret_cast<uint32_t*>(wbase)[k] = 0u;
    __syncwarp();
    const int total = B.counters[1];
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    for (int si = blockIdx.x * (blockDim.x >> 5) + wib; si < total; si += nwarps) {
        const int t = tree_of(B.srch_off, B.T, si);
        const int node = B.srch[(size_t)t * B.M + (si - B.srch_off[t])];
        const size_t m = (size_t)t * B.M + node;
        const int c = B.nd_cnt[m];
        if (c > kSmallNode) continue;  // k_hist_warp
        if (lane == 0 && B.hist_bytes)
            atomicAdd(B.hist_bytes, (unsigned long long)c * (unsigned long long)(B.mtry + 1));
        const int* seg = B.seg[cur] + (size_t)t * D.N + B.nd_start[m];
        const uint16_t* featp = B.feat + (size_t)t * B.M * B.mtry + (size_t)node * B.mtry;
        const uint8_t* rowp[kSmallRows];
        int lab[kSmallRows];
#pragma unroll
        for (int hh = 0; hh < kSmallRows; ++hh) {
            const int i = hh * 32 + lane;
            rowp[hh] = D.rows;
            lab[hh] = 0;
            if (i < c) {
                rowp[hh] = D.rows + (size_t)seg[i] * rs;
                lab[hh] = __ldg(reinterpret_cast<const int*>(rowp[hh] + ro));
            }
        }
        unsigned long long best = kNoKey;
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
                    x = warp_incl_scan(x, lane);
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
        if (lane == 0) B.nd_key[m] = best;
        __syncwarp();
    }
}

}  // namespace rfx
