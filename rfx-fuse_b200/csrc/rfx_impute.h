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
    const int* cells;        // [ncells][2] (row, column), rows in [r0, r0 + rows)
    int ncells;
    float* out;              // [ncells] new value, NaN = unchanged
    float* scratch;          // per warp: 3 n floats, then leaves and leaf sums
    long long scratch_stride;
    int max_leaves;
};

// floats of scratch one warp needs for n rows
inline long long impute_scratch_floats(int n, int max_leaves) {
    long long f = 3LL * n + 2LL * (max_leaves + 2) + max_leaves + 2;
    return (f + 3) / 4 * 4;
}

__global__ void k_impute(ImputeArgs a);

}  // namespace rfx
