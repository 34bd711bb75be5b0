// Quantised low-rank proximity product P = diag(s) Q Q^T diag(s) on the tcgen05 tensor
// cores with the per-row top-k selection fused into the accumulator read-out.
//
// Q holds int8 values (|q| <= 127) stored as bf16, which represents them exactly; products
// accumulate in fp32, exactly as integers (64 * 127^2 < 2^24), so the bf16 MMA equals the
// int8 dot product.  P_ij = (acc_ij * s_i) * s_j in fp32.
//
// The factor rows are stored by descending n_j = s_j |q_j| (Cauchy-Schwarz: P_ij <= n_i n_j),
// so the strongest candidates come first and each row's k-th value rises at once.
// CTA = 128 rows (the MMA's M), sweeping the column tiles of 256 (N) in stored order:
//   warp 0      one thread issues TMA loads: the CTA's 128x64 row tile once, then the
//               256x64 column tiles through a 2-stage ring (128-byte swizzle, K-major);
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and one thread
//               issues 4 x tcgen05.mma (K = 16 each) per tile, committing to the ring's
//               "empty" barrier and to the accumulator's "full" barrier;
//   warps 2-5   read the accumulator (tcgen05.ld 32x32b, thread = row, 128 columns per
//               wait), release it, and keep each row's best k under (value desc, original
//               column asc).  The tile's 256 column scales and ids are staged in shared
//               memory (each thread loads two for the next tile while it works on this one).
//               A chunk of 32 columns is scanned only when max_j(acc_ij * s_j) * s_i reaches
//               the row's current k-th value less a 1e-6 relative margin (the exact value
//               rounds the same three factors in another order).  Scanned values that beat
//               the bar are appended to the row's candidate buffer; the warp moves its 32
//               buffers into the rows' heaps of the best k together, so most lanes work in
//               each heap step (a stream in no particular order replaces the k-th entry about
//               k ln(N / k) times, and single-lane pushes cost a whole warp each).  Every
//               fourth tile, after such a flush, a row is final once n_i * n_(next tile's
//               first column) is below its k-th value; when all 128 rows are final the CTA
//               lowers its stop limit and the three roles end their sweeps.
// The single-thread producer and MMA roles sleep inside mbarrier.try_wait (suspend-time
// hint), so their waits do not take issue slots from the read-out warps.
// The bar carries the k-th entry's column id, so ties are broken by the original index
// whatever the sweep order, and the result is the exact top-k under the total order.
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
// A sleeping waiter stays in try_wait until the phase completes or this many nanoseconds pass.
constexpr uint32_t kSuspendNs = 2000;
#ifndef RFX_TK_CHECK
#define RFX_TK_CHECK 4
#endif
constexpr int kTkCheck = RFX_TK_CHECK;  // tiles between flush + finality checks

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

template <bool kSleep>
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    if (kSleep) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity), "r"(kSuspendNs)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
    }
    return ok != 0;
}

// Wait for the phase of `parity` to complete.  Returns kWaitOk, or kWaitFail on timeout or
// when another role of the CTA has aborted (abort may be null: wait regardless), or
// kWaitStop once step `it` is at or beyond the CTA's stop limit (limit may be null).
constexpr int kWaitFail = 0, kWaitOk = 1, kWaitStop = 2;

template <bool kSleep = true>
__device__ int mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                         unsigned long long* polls = nullptr, volatile int* limit = nullptr,
                         int it = 0) {
    const unsigned long long t0 = now_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (polls) ++*polls;
        if (mbar_try<kSleep>(bar, parity)) return kWaitOk;
        if (limit && it >= *limit) return kWaitStop;
        if (abort && *abort) return kWaitFail;
        if ((spin & 15u) == 0 && now_ns() - t0 > kWaitNs) return kWaitFail;
    }
}

// mbar_wait that also adds the cycles it spent to *cyc.
template <bool kSleep = true>
__device__ __forceinline__ int mbar_wait_t(uint32_t bar, uint32_t parity, volatile int* abort,
                                           unsigned long long* polls, unsigned long long* cyc,
                                           volatile int* limit = nullptr, int it = 0) {
    const long long t0 = clock64();
    const int r = mbar_wait<kSleep>(bar, parity, abort, polls, limit, it);
    *cyc += (unsigned long long)(clock64() - t0);
    return r;
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

// Issue a load of 32 consecutive fp32 accumulator columns of this thread's TMEM lane; the
// registers are valid after tmem_wait().
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t* r) {
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
}

__device__ __forceinline__ void tmem_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Ties 32 loaded registers to a point after tmem_wait() so no use moves above the wait.
__device__ __forceinline__ void tmem_pin32(uint32_t* r) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31]));
}

// The best k of one row are kept as a 4-ary heap in shared memory whose root is the
// worst kept entry (the bar a new column must beat).  Entry s of the row sits at
// v[s * kTkRows], j[s * kTkRows] (slot-major: lanes never share a bank).  Sift-up and
// sift-down run a fixed number of predicated steps, so lanes of a warp stay converged.
__device__ __forceinline__ bool better(float va, int ja, float vb, int jb) {
    return va > vb || (va == vb && ja < jb);
}

constexpr int kHeapDepth = 3;  // levels below the root of a 4-ary heap of <= 64 entries
                               // (1 + 4 + 16 + 64 slots); a node's 4 children load together

// Insert (val, col) into a heap of n < k entries.
__device__ __forceinline__ void heap_insert(float* v, int* j, int n, float val, int col) {
    int i = n;
#pragma unroll
    for (int l = 0; l < kHeapDepth; ++l) {
        const int p = (i - 1) >> 2;
        if (i > 0 && better(v[p * kTkRows], j[p * kTkRows], val, col)) {  // parent is better:
            v[i * kTkRows] = v[p * kTkRows];                               // the new entry rises
            j[i * kTkRows] = j[p * kTkRows];
            i = p;
        }
    }
    v[i * kTkRows] = val;
    j[i * kTkRows] = col;
}

// Replace the root (worst) of a full heap of n entries by (val, col) and restore the order.
__device__ __forceinline__ void heap_replace_root(float* v, int* j, int n, float val, int col) {
    int i = 0;
#pragma unroll
    for (int l = 0; l < kHeapDepth; ++l) {
        const int c0 = 4 * i + 1;
        float cv[4];
        int cj[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool in = c0 + u < n;
            cv[u] = in ? v[(c0 + u) * kTkRows] : __int_as_float(0x7f800000);
            cj[u] = in ? j[(c0 + u) * kTkRows] : 0x7fffffff;
        }
        // the worst child (absent children rank as +inf, never the worst)
        int w = 0;
#pragma unroll
        for (int u = 1; u < 4; ++u)
            if (better(cv[w], cj[w], cv[u], cj[u])) w = u;
        if (c0 < n && better(val, col, cv[w], cj[w])) {  // the worst child rises
            v[i * kTkRows] = cv[w];
            j[i * kTkRows] = cj[w];
            i = c0 + w;
        }
    }
    v[i * kTkRows] = val;
    j[i * kTkRows] = col;
}

// Largest of three floats (the three-input max.f32 of sm_100).
__device__ __forceinline__ float fmax3(float x, float y, float z) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(x), "f"(y), "f"(z));
    return d;
}

// Two fp32 products in one packed instruction (mul.rn.f32x2 of sm_100; each lane of the pair
// rounds like a scalar multiply).
__device__ __forceinline__ float2 fmul2(float x0, float x1, float y0, float y1) {
    float2 d;
    asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 c, a, b;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}\n"
        : "=f"(d.x), "=f"(d.y)
        : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
    return d;
}

}  // namespace

__global__ void __launch_bounds__(kTkThreads, 1)
k_topk_tc(const __grid_constant__ CUtensorMap tm, TopkArgs a) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, indexed from the shared array so accesses stay shared-space
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int k = a.k;
    const TkLayout lay = tk_layout(k);
    uint8_t* sA = sm;
    uint8_t* sB = sm + 16384;
    float* heap_v = (float*)(sm + lay.heap);                  // [k][128]
    int* heap_j = (int*)(sm + lay.heap + k * kTkRows * 4);    // [k][128]
    float* buf_v = (float*)(sm + lay.buf);                    // [kTkBuf][128]
    int* buf_j = (int*)(sm + lay.buf + kTkBuf * kTkRows * 4); // [kTkBuf][128]
    float* scr_all = (float*)(sm + lay.scr);                 // [4 warps][32][33]
    uint64_t* bars = (uint64_t*)(sm + lay.misc);
    // bars: full[0..1], empty[2..3], acc_full[4..5], acc_empty[6..7], a_full[8],
    // sready[9..10] (the tile's column scales and ids are in sc[b] / sid[b])
    uint32_t* tmem_slot = (uint32_t*)(bars + 11);
    volatile int* abort = (volatile int*)(tmem_slot + 1);
    volatile int* limit = (volatile int*)(tmem_slot + 2);  // column tiles the CTA still needs
    int* ndone = (int*)(tmem_slot + 3);                     // read-out warps whose rows are final
    float* sc = (float*)((uint8_t*)bars + 256);             // [2][256] column scales of a tile
    int* sid = (int*)((uint8_t*)bars + 256 + 2048);         // [2][256] original ids of its columns
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (kTkStages + s); };
    auto accf = [&](int b) { return bar0 + 8u * (4 + b); };
    auto acce = [&](int b) { return bar0 + 8u * (6 + b); };
    const uint32_t afull = bar0 + 64u;
    auto sready = [&](int b) { return bar0 + 8u * (9 + b); };
    const float kNegInf = -__int_as_float(0x7f800000);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // first position (row of the stored factor order) of this CTA's 128 rows
    const int pos_base = a.blocks ? a.blocks[blockIdx.x] * kTkRows : a.r0 + blockIdx.x * kTkRows;
    const int ntiles = a.ntiles;

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
        mbar_init(sready(0), 128);
        mbar_init(sready(1), 128);
        *abort = 0;
        *limit = ntiles;
        *ndone = 0;
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

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int issued = 0;
            unsigned long long polls = 0, cyc_empty = 0;
            mbar_expect_tx(afull, 16384);
            tma_load(smem_u32(sA), &tm, 0, pos_base, afull);
            for (int it = 0; it < ntiles && it < *limit; ++it) {
                const int s = it % kTkStages;
                const uint32_t ph = (uint32_t)(it / kTkStages) & 1u;
                const int w = mbar_wait_t(empty(s), ph ^ 1u, abort, &polls, &cyc_empty, limit, it);
                if (w == kWaitStop) break;
                if (w == kWaitFail) {
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
            if (a.prof) {
                atomicAdd(a.prof + 6, polls);
                atomicAdd(a.prof + 11, cyc_empty);
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
            bool ok = mbar_wait(afull, 0, abort) == kWaitOk;
            int last = -1;
            unsigned long long polls = 0, cyc_acce = 0, cyc_full = 0;
            const uint64_t da = sw128_desc(smem_u32(sA));
            for (int it = 0; ok && it < ntiles && it < *limit; ++it) {
                const int s = it % kTkStages, b = it & 1;
                const uint32_t ph = (uint32_t)(it / kTkStages) & 1u;
                const uint32_t bph = (uint32_t)(it >> 1) & 1u;
                int w = mbar_wait_t(acce(b), bph ^ 1u, abort, &polls, &cyc_acce, limit, it);
                if (w == kWaitOk) w = mbar_wait_t(full(s), ph, abort, &polls, &cyc_full, limit, it);
                if (w == kWaitStop) break;
                if (w == kWaitFail) {
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
            atomicAdd(a.err + 1, last + 1);  // column tiles multiplied by this CTA
            if (a.prof) {
                atomicAdd(a.prof + 5, polls);
                atomicAdd(a.prof + 9, cyc_acce);
                atomicAdd(a.prof + 10, cyc_full);
            }
            // the last MMAs must finish before the accumulators are freed
            if (last >= 0) mbar_wait(accf(last & 1), (uint32_t)(last >> 1) & 1u, nullptr);
        }
        __syncwarp();
    } else {
        // ---------------- read-out and selection ----------------
        const int rl = 32 * (warp & 3) + lane;  // TMEM lane = row of the tile
        const int pos = pos_base + rl;
        const int row = pos < a.R ? (a.perm ? __ldg(a.perm + pos) : pos) : -1;  // original id
        const bool valid = row >= a.r0 && row < a.r1;
        const float si = pos < a.R ? __ldg(a.scale + pos) : 0.0f;
        // Cauchy-Schwarz bound of the row against later columns: P_ij <= n_i n_j, with the
        // columns stored by n_j descending; 1e-5 covers the roundings of P and of n
        const float ni = a.norm && pos < a.R ? __ldg(a.norm + pos) * 1.00001f : 0.0f;
        bool warp_final = false;
        float* cv = heap_v + rl;
        int* cj = heap_j + rl;
        float* bv = buf_v + rl;
        int* bj = buf_j + rl;
        float* scr = scr_all + (warp & 3) * (32 * 33);
        const unsigned lt = (1u << lane) - 1u;
        int cnt = 0;                  // heap entries
        int nb = 0;                   // buffered candidates
        float theta = kNegInf;        // bar: the root once the heap is full
        int theta_j = 0x7fffffff;
        const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
        bool ok = true;
        unsigned long long n_test = 0, n_scan = 0, n_push = 0, polls = 0, n_flush = 0;
        unsigned long long cyc_wait = 0, cyc_tm = 0, cyc_f = 0, cyc_s = 0, cyc_fin = 0, cyc_stage = 0;
        const bool timing = a.prof != nullptr;  // per-warp cycle split when counters are on
        const long long cyc0 = clock64();
        // Candidates that beat the bar are appended to the row's buffer; the warp moves its 32
        // buffers into the heaps together (most lanes busy at once, rather than one lane per
        // push), when a buffer may not hold another chunk and before each finality check.
        auto flush = [&]() {
            const int nmax = __reduce_max_sync(0xffffffffu, nb);
            ++n_flush;
            for (int s = 0; s < nmax; ++s) {
                if (s < nb) {
                    const float val = bv[s * kTkRows];
                    const int col = bj[s * kTkRows];
                    if (better(val, col, theta, theta_j)) {  // the bar may have risen since
                        ++n_push;
                        if (cnt < k) {
                            heap_insert(cv, cj, cnt, val, col);
                            ++cnt;
                        } else {
                            heap_replace_root(cv, cj, cnt, val, col);
                        }
                        if (cnt == k) {
                            theta = cv[0];
                            theta_j = cj[0];
                        }
                    }
                }
            }
            nb = 0;
            __syncwarp();
        };
        // column scales and ids of a tile: each thread stages two of the 256 (loaded one tile
        // ahead, stored once the tile's reads of the other buffer are done)
        auto fetch = [&](int it, float2& s2, int2& i2) {
            const int p0 = it * kTkCols + 2 * rl;
            s2 = __ldg(reinterpret_cast<const float2*>(a.scale + p0));
            i2 = a.perm ? __ldg(reinterpret_cast<const int2*>(a.perm + p0)) : make_int2(p0, p0 + 1);
        };
        auto stage = [&](int b, float2 s2, int2 i2) {
            reinterpret_cast<float2*>(sc + b * kTkCols)[rl] = s2;
            reinterpret_cast<int2*>(sid + b * kTkCols)[rl] = i2;
            mbar_arrive(sready(b));
        };
        float2 nxt_s;
        int2 nxt_i;
        fetch(0, nxt_s, nxt_i);
        stage(0, nxt_s, nxt_i);
        for (int it = 0; it < ntiles; ++it) {
            const int b = it & 1;
            if (it + 1 < ntiles) fetch(it + 1, nxt_s, nxt_i);
            int w = mbar_wait_t<false>(sready(b), (uint32_t)(it >> 1) & 1u, abort, &polls, &cyc_wait, limit, it);
            // one decision per warp (the TMEM loads below are warp-collective)
            if (__any_sync(0xffffffffu, w == kWaitFail)) {
                ok = false;
                break;
            }
            if (__any_sync(0xffffffffu, w == kWaitStop)) break;
            if (__any_sync(0xffffffffu, *(volatile int*)ndone == 4)) {  // every row is final
                atomicMin((int*)limit, it);
                break;
            }
            w = mbar_wait_t<false>(accf(b), (uint32_t)(it >> 1) & 1u, abort, &polls, &cyc_wait, limit, it);
            if (__any_sync(0xffffffffu, w == kWaitFail)) {
                ok = false;
                break;
            }
            if (__any_sync(0xffffffffu, w == kWaitStop)) break;
            tc_fence_after();
            const float* scb = sc + b * kTkCols;
            const int* idb = sid + b * kTkCols;
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {  // 128 columns per TMEM wait
                long long t0 = timing ? clock64() : 0;
                uint32_t r[4][32];
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    tmem_ld32_issue(tmem + lane_addr + (uint32_t)(b * kTkCols + 128 * h + 32 * c), r[c]);
                tmem_wait();
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_pin32(r[c]);
                if (h == 1) {
                    tc_fence_before();
                    mbar_arrive(acce(b));
                }
                if (timing) {
                    const long long t1 = clock64();
                    cyc_tm += t1 - t0;
                    t0 = t1;
                }
                if (k == 0) {
                    if (valid) {
                        float* o = a.dense + (size_t)(row - a.r0) * a.dense_ld;
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                const int j = idb[128 * h + 32 * c + e];
                                if (j < a.R)
                                    o[j] = (__uint_as_float(r[c][e]) * si) * scb[128 * h + 32 * c + e];
                            }
                        }
                    }
                    continue;
                }
                // max_j acc_j s_j of each 32-column chunk (four independent chains), then
                // times s_i: the exact value rounds the same three factors in another order,
                // so the test keeps a 1e-6 relative margin
                float m[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) m[c] = kNegInf;
#pragma unroll
                for (int e4 = 0; e4 < 8; ++e4) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float4 sj = reinterpret_cast<const float4*>(scb + 128 * h + 32 * c)[e4];
                        const float2 p01 = fmul2(__uint_as_float(r[c][4 * e4]),
                                                 __uint_as_float(r[c][4 * e4 + 1]), sj.x, sj.y);
                        const float2 p23 = fmul2(__uint_as_float(r[c][4 * e4 + 2]),
                                                 __uint_as_float(r[c][4 * e4 + 3]), sj.z, sj.w);
                        m[c] = fmax3(m[c], p01.x, p01.y);
                        m[c] = fmax3(m[c], p23.x, p23.y);
                    }
                }
                n_test += 4;
                const float bar_lo = theta - fabsf(theta) * 1e-6f;
                uint32_t passes = 0;
#pragma unroll
                for (int c = 0; c < 4; ++c) passes |= (valid && m[c] * si >= bar_lo ? 1u : 0u) << c;
                if (timing) {
                    const long long t1 = clock64();
                    cyc_f += t1 - t0;
                    t0 = t1;
                }
                if (!__any_sync(0xffffffffu, passes != 0)) continue;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const bool pass = (passes >> c) & 1u;
                    if (!__any_sync(0xffffffffu, pass)) continue;
                    if (__any_sync(0xffffffffu, nb > kTkBuf - 32)) flush();  // room for a chunk
                    // the passing rows' 32 accumulators go through the warp's transpose, and
                    // the whole warp tests one row's 32 columns at a time (lane = column)
                    if (pass) {
                        ++n_scan;
#pragma unroll
                        for (int e = 0; e < 32; ++e) scr[lane * 33 + e] = __uint_as_float(r[c][e]);
                    }
                    __syncwarp();
                    const float sj = scb[128 * h + 32 * c + lane];
                    const int jj = idb[128 * h + 32 * c + lane];
                    uint32_t todo = __ballot_sync(0xffffffffu, pass);
                    while (todo) {
                        const int L = __ffs(todo) - 1;
                        todo &= todo - 1;
                        const float sL = __shfl_sync(0xffffffffu, si, L);
                        const float thL = __shfl_sync(0xffffffffu, theta, L);
                        const int thjL = __shfl_sync(0xffffffffu, theta_j, L);
                        const int rowL = __shfl_sync(0xffffffffu, row, L);
                        const int nbL = __shfl_sync(0xffffffffu, nb, L);
                        const float val = (scr[L * 33 + lane] * sL) * sj;
                        const bool take = better(val, jj, thL, thjL) && jj != rowL && jj < a.R;
                        const unsigned bal = __ballot_sync(0xffffffffu, take);
                        if (take) {
                            const int slot = (nbL + __popc(bal & lt)) * kTkRows + (rl - lane + L);
                            buf_v[slot] = val;
                            buf_j[slot] = jj;
                        }
                        if (lane == L) nb += __popc(bal);
                    }
                    __syncwarp();
                }
                if (timing) cyc_s += clock64() - t0;
            }
            // a row is final once no later column can beat its k-th value (checked every
            // kTkCheck-th tile, after the buffers are moved into the heaps)
            long long tf = timing ? clock64() : 0;
            if (k > 0 && a.norm && !warp_final && it + 1 < ntiles && (it % kTkCheck) == kTkCheck - 1) {
                flush();
                const float nb1 = __ldg(a.norm + (it + 1) * kTkCols);
                const bool fin = !valid || ni * nb1 < theta;
                if (__all_sync(0xffffffffu, fin)) {
                    warp_final = true;
                    if (lane == 0) atomicAdd(ndone, 1);
                }
            }
            if (timing) {
                const long long t1 = clock64();
                cyc_fin += t1 - tf;
                tf = t1;
            }
            if (it + 1 < ntiles) stage(b ^ 1, nxt_s, nxt_i);
            if (timing) cyc_stage += clock64() - tf;
        }
        if (k > 0) flush();
        if (a.prof) {
            atomicAdd(a.prof + 0, n_test);
            atomicAdd(a.prof + 1, n_scan);
            atomicAdd(a.prof + 2, n_push);
            atomicAdd(a.prof + 4, polls);
            atomicAdd(a.prof + 7, cyc_wait);
            atomicAdd(a.prof + 8, (unsigned long long)(clock64() - cyc0));
            atomicAdd(a.prof + 12, cyc_tm);
            atomicAdd(a.prof + 13, cyc_f);
            atomicAdd(a.prof + 14, cyc_s);
            atomicAdd(a.prof + 3, cyc_fin);   // (replaces the flush count)
            atomicAdd(a.prof + 15, cyc_stage);
        }
        if (!ok) {
            if (!*abort) atomicExch(a.err, 3);
            *abort = 1;
        } else if (valid && k > 0) {
            // heap sort: the worst entry goes to the back, best first at the end
            for (int n = cnt; n > 1; --n) {
                const float wv = cv[0];
                const int wj = cj[0];
                heap_replace_root(cv, cj, n - 1, cv[(n - 1) * kTkRows], cj[(n - 1) * kTkRows]);
                cv[(n - 1) * kTkRows] = wv;
                cj[(n - 1) * kTkRows] = wj;
            }
            const size_t orow = a.out_pos0 >= 0 ? (size_t)(pos - a.out_pos0) : (size_t)(row - a.r0);
            int* oi = a.out_idx + orow * k;
            float* ov = a.out_val + orow * k;
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
