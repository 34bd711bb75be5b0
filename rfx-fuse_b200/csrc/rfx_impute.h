// Imputation kernel (rfx_impute.cu).
#pragma once
#include <cstdint>

namespace rfx {

// leaves[] slot that carries the leaf count from lane 0 to the warp (leaves start after it)
constexpr int kImpLeafCountSlot = -1;

struct ImputeArgs {
    const float* S;          // finished proximity rows [r0, r0 + rows) x n, row stride ldS
    long long ldS;
    int r0;
    int n, p;
    const float* xc;         // [p][n] current values (column-major)
    const uint8_t* miss;     // [p][n] 1 = missing in the input
    const uint8_t* is_cat;   // [p]
    const int* cells;        // [ncells][2] (row, column), sorted by row
    const int* rows;         // [nrows] rows with missing cells, in [r0, r0 + rows of S)
    const int* row_cells;    // [nrows + 1] cells of rows[r]: [row_cells[r], row_cells[r + 1])
    int nrows;
    float* out;              // [ncells] new value, NaN = unchanged
    float* scratch;          // per warp: 7 n floats, then leaves and leaf sums
    long long scratch_stride;
    int max_leaves;
    int top_k;               // >= 0: only the top_k neighbours by proximity (0: all, reordered);
                             // -1: all in row order
    int median;              // 1: median / most frequent value, 0: proximity-weighted mean / mode
    unsigned long long* prof;  // optional counters (RFX_IMPUTE_PROF), null = off
};

// floats of one n-long scratch buffer (a multiple of 8, so the next one starts on 32 bytes)
__host__ __device__ inline int impute_row_floats(int n) { return (n + 7) / 8 * 8; }

// floats of scratch one warp needs for n rows: seven n-long buffers, the leaf list (int2, one
// extra slot for the count) and the leaf sums
inline long long impute_scratch_floats(int n, int max_leaves) {
    long long f = 7LL * impute_row_floats(n) + 2LL * (max_leaves + 2) + max_leaves + 2;
    return (f + 7) / 8 * 8;
}

__global__ void k_impute(ImputeArgs a);

}  // namespace rfx
