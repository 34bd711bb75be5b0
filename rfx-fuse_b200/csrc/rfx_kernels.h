// Kernel entry points of rfx_b200 (definitions in rfx_prep.cu, rfx_grow.cu, rfx_post.cu).
#pragma once
#include "rfx_device.cuh"

namespace rfx {

// rfx_prep.cu
__global__ void k_transpose(const float* X, int N, int p, float* xc);
__global__ void k_sort_columns(const float* xc, int N, const int* cat, uint32_t* ka, uint32_t* kb);
__global__ void k_edges(const uint32_t* sorted, int N, const int* cat, int nbins, float* uniq,
                        float* edges, int* nb, int* kind);
__global__ void k_pack_rows(Data D);
__global__ void k_regr_targets(const float* y, int N, int* lab, float* yv);
__global__ void k_cumw(const float* w, int N, float* cum, float* total);
__global__ void k_permutation(int N, uint32_t seed, int* ks, int* perm);
__global__ void k_bootstrap(Data D, Batch B);
__global__ void k_compact(Data D, Batch B);

// rfx_grow.cu
__global__ void k_level_begin(Batch B, int level);
__global__ void k_node_eval(Data D, Batch B, int cur);
__global__ void k_draw(Data D, Batch B);
__global__ void k_srch_scan(Batch B);
__global__ void k_task_records(Batch B);
__global__ void k_commit(Data D, Batch B);
__global__ void k_partition(Data D, Batch B, int cur);
__global__ void k_partition_big(Data D, Batch B, int cur);

// rfx_hist.cu
__global__ void k_hist_warp_regr(Data D, Batch B, int cur, HistArgs a);
__global__ void k_hist_warp_class(Data D, Batch B, int cur, HistArgs a);
__global__ void k_hist_pipe(Data D, Batch B, int cur, PipeArgs a);
__global__ void k_hist_lane(Data D, Batch B, int cur, int slots);
__global__ void k_hist_lane_mid(Data D, Batch B, int cur, int slots);
__global__ void k_hist_lane_tiny(Data D, Batch B, int cur, int slots);
__global__ void k_hist_small(Data D, Batch B, int cur, int warp_bytes);

// rfx_post.cu
__global__ void k_oob_drop(Data D, Batch B);
__global__ void k_votes(Data D, Batch B, int* nout, int* votes, float* oob_sum, float* tree_oob,
                        int tree_oob_stride);
__global__ void k_imp_used(Data D, Batch B);
__global__ void k_imp_class(Data D, Batch B);
__global__ void k_imp_class_rr(Data D, Batch B);
__global__ void k_imp_regr(Data D, Batch B);
__global__ void k_imp_pack(Batch B);
__global__ void k_imp_regr_sum(Data D, Batch B);
__global__ void k_imp_regr_rr(Data D, Batch B);
__global__ void k_imp_fold(Data D, Batch B, float* avimp, float* sqsd);
__global__ void k_prox(Data D, Batch B, int R, int* C);
__global__ void k_prox_codes(Batch B, int N, int R, uint16_t* code, int* ocnt,
                             unsigned long long* pairs);
__global__ void k_prox_pull(const uint16_t* code, int Tp, int R, int nb, int* C);
__global__ void k_prox_finish(const int* C, const int* nout, int R, int r0, int r1, float* out);
// k_prox_finish over rows [r0, r1) with its tile grid.
cudaError_t launch_prox_finish(const int* C, const int* nout, int R, int r0, int r1, float* out,
                               cudaStream_t st);
// The whole R x R finished matrix (tile pairs; inv: R doubles of scratch for 1 / nout).
cudaError_t launch_prox_finish_full(const int* C, const int* nout, int R, double* inv, float* out,
                                    cudaStream_t st);
// k_prox_finish_packed (with the 1 / nout scales) over the packed elements [e0, e0 + len).
cudaError_t launch_prox_finish_packed(const int* C, long long e0, long long len, const int* nout,
                                      int R, double* inv, float* out, cudaStream_t st);
__global__ void k_votes_to_q(const int* votes, const float* w, int N, int nclass, float* q);
__global__ void k_oob_fold(const float* tree_oob, int ntrees, int N, float* vec);

}  // namespace rfx
