// Prediction kernels (rfx_predict.cu).
#pragma once
#include <cstdint>

#include "rfx_device.cuh"

namespace rfx {

constexpr int kPredMaxClass = 32;

// One node of a stored tree: a split on `feat` at `val` going to `left` / `right`, or a
// terminal node (feat == -1) whose `val` holds the value (regression) or the class bits.
struct __align__(16) PNode {
    int feat;
    float val;
    int left;
    int right;
};

__global__ void k_pack_forest(Batch B, int task, PNode* forest, float* root_value);
__global__ void k_predict_walk(const PNode* forest, const float* root_value, int M, int T,
                               const float* xc, int n, int p, const int* cat, int task,
                               int nclass, uint8_t* vote, float* value);
__global__ void k_predict_reduce(const uint8_t* vote, const float* value, int n, int T, int task,
                                 int nclass, const float* classwt, int* cls, float* proba,
                                 float* pred);

}  // namespace rfx
