// Device-side building blocks shared by the rfx_b200 kernels.
//
// Everything here is compiled with -fmad=false and IEEE division/square root so that each
// float expression rounds exactly like the reference's scalar CPU code.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rfx {

constexpr int kMaxClass = 32;     // classes supported by the device histograms
constexpr int kBins = 256;        // histogram bins (uint8 codes)
constexpr uint32_t kFull = 0xffffffffu;
constexpr unsigned long long kNoKey = ~0ull;
constexpr int kBigSegment = 2048;  // segments above this are partitioned by a whole block
constexpr int kSmallNode = 64;     // classification nodes up to this size go to k_hist_small
// k_hist_lane (regression nodes of at most kLaneNode rows, one lane per drawn feature), in
// three instantiations by node size (at most kLaneTiny, kLaneSmall, kLaneNode rows): the
// smaller the nodes, the smaller the shared memory of a warp and the more warps per SM.
constexpr int kLaneNode = 128;
constexpr int kLaneSmall = 64;
constexpr int kLaneTiny = 32;
constexpr int kLaneSlots = 8;      // nodes per warp at most
// k_hist_pipe: chunks in the shared-memory ring; bytes before the ring (mbarriers, bounds)
constexpr int kPipeBufs = 6;
constexpr int kPipeHead = 256;
// staged bins per lane for nodes of `node` rows (an odd number of words: lanes in distinct banks)
__host__ __device__ constexpr int lane_tile(int node) { return node + 4; }
// shared memory of one k_hist_lane warp taking `slots` nodes of at most `node` rows
__host__ __device__ constexpr int lane_bytes(int node, int slots) {
    return node * 32 * 9 + 2 * 1024 + 32 * lane_tile(node) + slots * node * 8 + kLaneSlots * 4;
}
// Rows of the largest node the small kernels search (the rest go to the block-per-node
// kernels); 0 when regression draws more than 32 features (k_hist_lane needs a lane per draw).
__host__ __device__ __forceinline__ int small_node_limit(int nclass, int mtry) {
    return nclass == 1 ? (mtry > 32 ? 0 : kLaneNode) : kSmallNode;
}

// ------------------------------------------------------------------------------------
// MT19937, the generator of include/rf_utils.hpp:74-141: init_genrand seeding, standard
// twist and tempering, and randomu() = float(double(y) / (2^32 - 1)).
// The 624-word state lives in shared memory and one thread block advances it: the twist
// is split into the four dependency phases of the recurrence (words [0,227) read only old
// words; [227,454) read words of the first phase; [454,623) read words of the second;
// word 623 reads the new word 0), so every word is produced by its own thread.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

__device__ __forceinline__ float mt_uniform(uint32_t tempered) {
    return (float)((double)tempered / 4294967295.0);
}

__device__ __forceinline__ uint32_t mt_mix(uint32_t a, uint32_t b, uint32_t c) {
    const uint32_t y = (a & 0x80000000u) | (b & 0x7fffffffu);
    return c ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
}

// Requires blockDim.x >= 227.  All threads of the block must call it.
__device__ __forceinline__ void mt_twist_block(uint32_t* s) {
    const int t = threadIdx.x;
    uint32_t v = 0;
    if (t < 227) v = mt_mix(s[t], s[t + 1], s[t + 397]);
    __syncthreads();
    if (t < 227) s[t] = v;
    __syncthreads();
    if (t < 227) v = mt_mix(s[227 + t], s[228 + t], s[t]);
    __syncthreads();
    if (t < 227) s[227 + t] = v;
    __syncthreads();
    if (t < 169) v = mt_mix(s[454 + t], s[455 + t], s[227 + t]);
    __syncthreads();
    if (t < 169) s[454 + t] = v;
    __syncthreads();
    if (t == 0) s[623] = mt_mix(s[623], s[0], s[396]);
    __syncthreads();
}

// Sequential init_genrand (one thread); returns the read position (624 = twist first).
__device__ __forceinline__ void mt_seed_serial(uint32_t* s, uint32_t seed) {
    s[0] = seed;
    for (int k = 1; k < 624; ++k) s[k] = 1812433253u * (s[k - 1] ^ (s[k - 1] >> 30)) + (uint32_t)k;
}

// Consume `count` outputs of the stream held in shared state `s` whose next unread word is
// at `pos` (uniform across the block); f(index, tempered) is called once per output by
// some thread.  Returns the new read position.  All threads must call it.
template <class F>
__device__ __forceinline__ int mt_generate(uint32_t* s, int pos, long long count, F&& f) {
    long long done = 0;
    while (done < count) {
        if (pos >= 624) {
            mt_twist_block(s);
            pos = 0;
        }
        const int take = (int)min((long long)(624 - pos), count - done);
        for (int j = threadIdx.x; j < take; j += blockDim.x) f(done + j, mt_temper(s[pos + j]));
        done += take;
        pos += take;
        __syncthreads();
    }
    return pos;
}

// ------------------------------------------------------------------------------------
// Order-preserving float <-> uint32 maps (total order on non-NaN floats; -0 < +0).
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ord_of(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float float_of(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// ------------------------------------------------------------------------------------
// Dataset resident in HBM (one per loaded fit).
// ------------------------------------------------------------------------------------
struct Data {
    int N;            // grown rows (2n for unsupervised)
    int p;            // features
    int nclass;       // 1 for regression
    int task;
    int rs;           // bytes per packed row
    int ro;           // byte offset of the target inside a packed row
    int maxcat;       // category bound of the importance walks (the estimator's maxcat)
    int has_cat;      // any feature with cat > 1
    const float* xc;       // [p][N] raw values, column-major
    const uint8_t* rows;   // [N][rs]: uint8 bin of every feature, then the target
                           //   (float val, float val*val for regression; int label otherwise)
    const float* edges;    // [p][257]
    const int* nb;         // [p] bins per feature
    const int* kind;       // [p] 0 continuous, 1 binary, 2 categorical
    const int* cat;        // [p]
    const int* lab;        // [N] 0-based class, or (int)(y*1000) for regression
    const float* yreg;     // [N] regression targets
    const float* yv;       // [N] regression (float)lab/1000
    const int* perm;       // [N] importance permutation
    const float* cumw;     // [N] cumulative bootstrap weights or nullptr
    float totw;            // total bootstrap weight
};

// ------------------------------------------------------------------------------------
// Trees grown concurrently (one batch).  Row arrays have stride N, node arrays stride M.
// ------------------------------------------------------------------------------------
struct Batch {
    int T;            // trees in this batch
    int M;            // maxnode
    int mtry;
    int minsplit;     // rows needed to search a node
    int lane_split;   // 1: the small list's task records are split by size for k_hist_lane
    int tree0;        // global id of tree 0 of the batch
    int iseed, boot_seed;
    int* nin;         // [T][N]
    int* seg[2];      // [T][N] row ids, node segments (ping-pong by level parity)
    int* ninbag;      // [T]
    int* oob;         // [T][N] ascending OOB rows
    int* noob;        // [T]
    uint32_t* mt;     // [T][624] grower MT state
    int* mt_pos;      // [T]
    // tree arrays (reference layout)
    int* status; int* bestvar; float* xbest; int* treemap; int* nodeclass;
    float* nodepred; float* tnodewt;
    int4* imp_node;   // [T][M] regression importance: a node in one 16-byte record
                      //   {status << 24 | split feature, threshold (terminal: prediction), left,
                      //   right}, or nullptr
    // node work arrays
    int* nd_start; int* nd_cnt; uint8_t* nd_buf; uint8_t* nd_flag;
    float* nd_crit0; int* nd_maj; float* nd_sum;
    unsigned long long* nd_key;   // best (criterion, draw, bin) of the node
    uint16_t* feat;               // [T][M*mtry] drawn features
    // level bookkeeping
    int* lvl_lo; int* lvl_hi; int* nxt_lo; int* nxt_hi; int* nnode;
    int* lvl_off;     // [T+1] prefix of level widths
    int* srch;        // [T][M] searched nodes of the level, in node order
    int* srch_cnt;    // [T]
    int* srch_off;    // [T+1]
    int* counters;    // [32]: 0 level total, 1 searched total, 2 next-level total, 3 pipeline
                      //      timeouts, 4 big searched, 5 big partitions, 6 small searched,
                      //      7 levels with nodes, 8-9 hist_bytes, 10-11 prox_pairs, 12-19 diag,
                      //      20 / 21 / 22 small-list records of at most kLaneTiny / above
                      //      kLaneSmall / in between rows
    unsigned long long* hist_bytes;  // algorithmic bytes read by k_hist (sum of c_v*(mtry+L))
    unsigned long long* prox_pairs;  // proximity pair updates counted by k_prox
    unsigned long long* diag;        // [4] optional histogram diagnostics (nullptr: off): exact
                                     // criterion evaluations, conflict rounds, 32-row steps
    int* srch_big;    // [T][M] searched nodes above small_node_limit rows, in node order
    int* srch_big_cnt;  // [T]
    int* srch_big_off;  // [T+1]
    int4* big_rec;    // flat over the level's big searched nodes: {tree, node, start, rows}
    int4* sml_rec;    // the same for the small searched nodes
    int4* sml2_rec;   // regression: the small searched nodes of kLaneTiny+1..kLaneSmall rows
    int* srch_sml;    // [T][M] searched nodes of at most small_node_limit rows; total in counters[6]
                      // (regression task records: nodes of at most kLaneTiny rows first,
                      // counters[20] of them, nodes above kLaneSmall rows last, counters[21])
    int* srch_sml_cnt;  // [T]
    int* srch_sml_off;  // [T+1]
    long long* part_big;  // split nodes (t*M + node) with segments above kBigSegment; count in counters[5]
    // post-growth
    int* oob_leaf;    // [T][N] terminal node of OOB rows (-1 in-bag)
    uint8_t* used;    // [T][p]
    int* right;       // [T] correct OOB votes (classification importance)
    int* rightimp;    // [T][p]
    float* d2;        // [T][p][N] regression importance squared errors per OOB rank
    float* d0;        // [T][N]
    float* rr;        // [T][p]
    float* rsum;      // [T][p + 1] regression importance: row-order error sums
    float* tree_oob;  // [T][N] per-tree OOB predictions (NaN in-bag), optional
};

// Launch shape of k_hist_warp (rfx_hist.cu).
struct HistArgs {
    int warps;       // warps per block = drawn features per work unit
    int groups;      // work units per searched node = ceil(mtry / warps)
    int warp_bytes;  // per-warp shared memory
};

// Launch shape of k_hist_pipe (rfx_hist.cu).
struct PipeArgs {
    int warps;    // consumer warps (one drawn feature each); the block adds a producer warp
    int groups;   // work units per searched node = ceil(mtry / warps)
    int ch;       // rows per staged chunk (<= 64)
    int rstride;  // bytes per staged row (rs + 16)
};

// Locate the tree of a flattened task index given an exclusive prefix `off` of length T+1.
__device__ __forceinline__ int tree_of(const int* off, int T, int idx) {
    int lo = 0, hi = T;  // off[lo] <= idx < off[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (off[mid] <= idx) lo = mid; else hi = mid;
    }
    return lo;
}

}  // namespace rfx
