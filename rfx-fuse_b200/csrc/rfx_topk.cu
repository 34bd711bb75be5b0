// Quantised low-rank proximity product P = diag(s) Q Q^T diag(s) on the tcgen05 tensor
// cores with the per-row top-k selection fused into the accumulator read-out.
//
// Q holds int8 values (|q| <= 127) stored as bf16, which represents them exactly; products
// accumulate in fp32, exactly as integers (64 * 127^2 < 2^24), so the bf16 MMA equals the
// int8 dot product.  P_ij = (acc_ij * s_i) * s_j in fp32.
//
// CTA = 128 rows (the MMA's M), sweeping all column tiles of 256 (N) in ascending order:
//   warp 0      one thread issues TMA loads: the CTA's 128x64 row tile once, then the
//               256x64 column tiles through a 3-stage ring (128-byte swizzle, K-major);
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and one thread
//               issues 4 x tcgen05.mma (K = 16 each) per tile, committing to the ring's
//               "empty" barrier and to the accumulator's "full" barrier;
//   warps 2-5   read the accumulator (tcgen05.ld 32x32b, thread = row), release it, and
//               keep each row's best k under (value desc, column asc): a chunk of 32 columns
//               is skipped when an upper bound of its values (chunk max * s_i * max s_j) does
//               not beat the row's current k-th value; survivors go to the row's candidate
//               slots in shared memory (slot-major, conflict-free), compacted by quickselect
//               when full.
// Columns arrive in ascending order, so a new candidate with a value equal to the k-th
// never displaces it, and the result is the exact top-k under the total order.
//
// Every wait is bounded (about one second); on expiry the CTA records the failure in
// a.err, drains its own copies in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "rfx_lowrank.h"

namespace rfx {

namespace {

constexpr unsigned long long kWaitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase of `parity` to complete; false on timeout or when another role of the
// CTA has aborted (abort may be null: wait regardless).
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    const unsigned long long t0 = now_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try(bar, parity)) return true;
        if ((spin & 63u) == 0) {
            if (abort && *abort) return false;
            if (now_ns() - t0 > kWaitNs) return false;
        }
    }
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// 2-D tiled TMA load (box 64 x 128 of bf16) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap* tm, int x, int y,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((unsigned long long)tm), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address
    d |= (uint64_t)1 << 16;                           // leading offset (unused when swizzled)
    d |= (uint64_t)(1024 >> 4) << 32;                 // stride offset
    d |= (uint64_t)1 << 46;                           // descriptor version
    d |= (uint64_t)2 << 61;                           // 128-byte swizzle
    return d;
}

// Instruction descriptor of kind::f16: bf16 x bf16 -> fp32, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4)            // D fp32
                            | (1u << 7)          // A bf16
                            | (1u << 10)         // B bf16
                            | ((256u >> 3) << 17)  // N
                            | ((128u >> 4) << 24); // M

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
}

// Candidate slots of one row: slot s of the row at v[s * kTkRows], j[s * kTkRows].
__device__ __forceinline__ bool better(float va, int ja, float vb, int jb) {
    return va > vb || (va == vb && ja < jb);
}

__device__ __forceinline__ void swap_slots(float* v, int* j, int a, int b) {
    const float tv = v[a * kTkRows];
    const int tj = j[a * kTkRows];
    v[a * kTkRows] = v[b * kTkRows];
    j[a * kTkRows] = j[b * kTkRows];
    v[b * kTkRows] = tv;
    j[b * kTkRows] = tj;
}

// Reorder slots [0, n) so that [0, k) hold the k best (Hoare quickselect on slot k-1).
__device__ void select_best(float* v, int* j, int n, int k) {
    int lo = 0, hi = n - 1;
    const int kth = k - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const float pv = v[mid * kTkRows];
        const int pj = j[mid * kTkRows];
        int a = lo, b = hi;
        while (a <= b) {
            while (better(v[a * kTkRows], j[a * kTkRows], pv, pj)) ++a;
            while (better(pv, pj, v[b * kTkRows], j[b * kTkRows])) --b;
            if (a <= b) {
                swap_slots(v, j, a, b);
                ++a;
                --b;
            }
        }
        if (kth <= b) hi = b;
        else if (kth >= a) lo = a;
        else break;
    }
}

struct PushResult {
    int cnt;
    float theta;
};

// Append a candidate; when the slots are full keep the best k and return the new bar
// (the k-th value).
__device__ __noinline__ PushResult push_candidate(float* v, int* j, int cnt, int k, float val,
                                                  int col, float theta) {
    v[cnt * kTkRows] = val;
    j[cnt * kTkRows] = col;
    ++cnt;
    if (cnt == kTkSlots) {
        select_best(v, j, cnt, k);
        cnt = k;
        float worst = v[0];
        for (int s = 1; s < k; ++s) worst = fminf(worst, v[s * kTkRows]);
        theta = worst;
    }
    return {cnt, theta};
}

}  // namespace

__global__ void __launch_bounds__(kTkThreads, 1)
k_topk_tc(const __grid_constant__ CUtensorMap tm, TopkArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = sm;
    uint8_t* sB = sm + 16384;
    float* cand_v = (float*)(sm + 16384 + kTkStages * 32768);
    int* cand_j = (int*)(sm + 16384 + kTkStages * 32768 + kTkSlots * kTkRows * 4);
    uint64_t* bars = (uint64_t*)(sm + 16384 + kTkStages * 32768 + kTkSlots * kTkRows * 8);
    // bars: full[0..2], empty[3..5], acc_full[6..7], acc_empty[8..9], a_full[10]
    uint32_t* tmem_slot = (uint32_t*)(bars + 11);
    volatile int* abort = (volatile int*)(tmem_slot + 1);
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (3 + s); };
    auto accf = [&](int b) { return bar0 + 8u * (6 + b); };
    auto acce = [&](int b) { return bar0 + 8u * (8 + b); };
    const uint32_t afull = bar0 + 80u;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_base = a.r0 + blockIdx.x * kTkRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTkStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accf(b), 1);
            mbar_init(acce(b), 128);
        }
        mbar_init(afull, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = a.ntiles;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int issued = 0;
            mbar_expect_tx(afull, 16384);
            tma_load(smem_u32(sA), &tm, 0, row_base, afull);
            for (int it = 0; it < ntiles; ++it) {
                const int s = it % kTkStages;
                const uint32_t ph = (uint32_t)(it / kTkStages) & 1u;
                if (!mbar_wait(empty(s), ph ^ 1u, abort)) {
                    if (!*abort) atomicExch(a.err, 1);
                    *abort = 1;
                    break;
                }
                const uint32_t dst = smem_u32(sB + s * 32768);
                mbar_expect_tx(full(s), 32768);
                tma_load(dst, &tm, 0, it * kTkCols, full(s));
                tma_load(dst + 16384, &tm, 0, it * kTkCols + 128, full(s));
                issued = it + 1;
            }
            // drain this thread's copies still in flight
            mbar_wait(afull, 0, nullptr);
            for (int it = issued > kTkStages ? issued - kTkStages : 0; it < issued; ++it)
                mbar_wait(full(it % kTkStages), (uint32_t)(it / kTkStages) & 1u, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            bool ok = mbar_wait(afull, 0, abort);
            int last = -1;
            const uint64_t da = sw128_desc(smem_u32(sA));
            for (int it = 0; ok && it < ntiles; ++it) {
                const int s = it % kTkStages, b = it & 1;
                const uint32_t ph = (uint32_t)(it / kTkStages) & 1u;
                const uint32_t bph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(acce(b), bph ^ 1u, abort) || !mbar_wait(full(s), ph, abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t db = sw128_desc(smem_u32(sB + s * 32768));
                const uint32_t d = tmem + (uint32_t)(b * kTkCols);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)  // K = 16 per MMA: +32 bytes in the swizzled row
                    mma_bf16(d, da + 2 * kk, db + 2 * kk, kk > 0 ? 1u : 0u);
                mma_commit(empty(s));
                mma_commit(accf(b));
                last = it;
            }
            if (!ok) {
                if (!*abort) atomicExch(a.err, 2);
                *abort = 1;
            }
            // the last MMAs must finish before the accumulators are freed
            if (last >= 0) mbar_wait(accf(last & 1), (uint32_t)(last >> 1) & 1u, nullptr);
        }
        __syncwarp();
    } else {
        // ---------------- read-out and selection ----------------
        const int rl = 32 * (warp & 3) + lane;  // TMEM lane = row of the tile
        const int row = row_base + rl;
        const bool valid = row < a.r1;
        const float si = valid ? __ldg(a.scale + row) : 0.0f;
        const int k = a.k;
        float* cv = cand_v + rl;
        int* cj = cand_j + rl;
        int cnt = 0;
        float theta = -__int_as_float(0x7f800000);
        const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
        bool ok = true;
        for (int it = 0; it < ntiles; ++it) {
            const int b = it & 1;
            if (!mbar_wait(accf(b), (uint32_t)(it >> 1) & 1u, abort)) {
                ok = false;
                break;
            }
            __syncwarp();
            tc_fence_after();
            const int jt = it * kTkCols;
#pragma unroll 1
            for (int c = 0; c < kTkCols / 32; ++c) {
                float v[32];
                __syncwarp();
                tmem_ld32(tmem + lane_addr + (uint32_t)(b * kTkCols + 32 * c), v);
                if (c == kTkCols / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(acce(b));
                }
                const int j0 = jt + 32 * c;
                if (k == 0) {
                    if (valid) {
                        float* o = a.dense + (size_t)(row - a.r0) * a.dense_ld + j0;
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (j0 + e < a.R) o[e] = (v[e] * si) * __ldg(a.scale + j0 + e);
                    }
                    continue;
                }
                float mx = v[0];
#pragma unroll
                for (int e = 1; e < 32; ++e) mx = fmaxf(mx, v[e]);
                const float bound = mx >= 0.0f ? (mx * si) * __ldg(a.smax + (j0 >> 5)) : 0.0f;
                if (!(valid && bound > theta)) continue;
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int col = j0 + e;
                    const float val = (v[e] * si) * __ldg(a.scale + col);
                    if (val > theta && col != row && col < a.R) {
                        const PushResult pr = push_candidate(cv, cj, cnt, k, val, col, theta);
                        cnt = pr.cnt;
                        theta = pr.theta;
                    }
                }
            }
        }
        if (!ok) {
            if (!*abort) atomicExch(a.err, 3);
            *abort = 1;
        } else if (valid && k > 0) {
            if (cnt > k) {
                select_best(cv, cj, cnt, k);
                cnt = k;
            }
            for (int s = 1; s < cnt; ++s) {  // insertion sort of the kept slots
                const float tv = cv[s * kTkRows];
                const int tj = cj[s * kTkRows];
                int u = s - 1;
                while (u >= 0 && better(tv, tj, cv[u * kTkRows], cj[u * kTkRows])) {
                    cv[(u + 1) * kTkRows] = cv[u * kTkRows];
                    cj[(u + 1) * kTkRows] = cj[u * kTkRows];
                    --u;
                }
                cv[(u + 1) * kTkRows] = tv;
                cj[(u + 1) * kTkRows] = tj;
            }
            int* oi = a.out_idx + (size_t)(row - a.r0) * k;
            float* ov = a.out_val + (size_t)(row - a.r0) * k;
            for (int s = 0; s < k; ++s) {
                oi[s] = s < cnt ? cj[s * kTkRows] : -1;
                ov[s] = s < cnt ? cv[s * kTkRows] : -__int_as_float(0x7f800000);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                     : "memory");
    }
}

}  // namespace rfx
