// Kernels of the low-rank proximity path (rfx_lowrank.cu, rfx_topk.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "rfx_device.cuh"

namespace rfx {

constexpr uint16_t kNoGroup = 0xFFFF;  // row outside the proximity rows
constexpr int kLrMaxR = 96;            // sketch columns (rank + oversampling) at most
constexpr int kLrK = 64;               // stored factor width (rank <= 64, zero padded)

// product / top-k kernel geometry
constexpr int kTkRows = 128;    // rows of a CTA (MMA M)
constexpr int kTkCols = 256;    // columns of a tile (MMA N)
constexpr int kTkStages = 2;    // column-tile ring
constexpr int kTkSlots = 64;    // heap entries per row (k <= 64)
constexpr int kTkBuf = 48;      // candidate buffer entries per row
constexpr int kTkThreads = 192; // warp 0 loads, warp 1 issues MMAs, warps 2-5 read out
constexpr int kTkScr = 4 * 32 * 33 * 4;  // per read-out warp: a 32 x 32 chunk, rows padded to 33

// Shared-memory layout of the product kernel for k neighbours: row tile, column-tile ring,
// heaps [k][128], candidate buffers [kTkBuf][128] (values, then original ids), the read-out
// warps' chunk transposes, then barriers and the staged column scales and ids of two tiles.
struct TkLayout {
    int heap, buf, scr, misc, bytes;
};
__host__ __device__ constexpr TkLayout tk_layout(int k) {
    return TkLayout{16384 + kTkStages * 32768,
                    16384 + kTkStages * 32768 + k * kTkRows * 8,
                    16384 + kTkStages * 32768 + k * kTkRows * 8 + kTkBuf * kTkRows * 8,
                    16384 + kTkStages * 32768 + k * kTkRows * 8 + kTkBuf * kTkRows * 8 + kTkScr,
                    16384 + kTkStages * 32768 + k * kTkRows * 8 + kTkBuf * kTkRows * 8 + kTkScr +
                        4352 + 1024};
}

struct TopkArgs {
    int R;              // valid rows (= valid columns)
    int r0, r1;         // original rows whose results are written
    const int* blocks;  // [grid] 128-row blocks (of the stored order) of the CTAs, or null:
                        // CTA b takes positions r0 + 128 b (identity order)
    const int* perm;    // [Rpad] original id of every stored position (>= R for padding),
                        // or null (identity order)
    int ntiles;         // column tiles (Rpad / 256)
    int k;              // neighbours kept; 0 = write the product densely
    const float* scale; // [Rpad] by stored position
    const float* norm;  // [Rpad] s_j * |q_j| by stored position, descending (with perm), or
                        // null: no early stop
    int out_pos0;       // >= 0: results of stored position p at row p - out_pos0 of the
                        // outputs; -1: at row (original id - r0)
    int* out_idx;       // [rows][k]
    float* out_val;     // [r1 - r0][k]
    float* dense;       // [r1 - r0][dense_ld] by original column, when k == 0
    long long dense_ld;
    int* err;           // [0]: nonzero after a wait timed out; [1] += column tiles multiplied
    unsigned long long* prof;  // optional counters (null: off): chunks tested, chunks
                               // scanned, candidates pushed, -, read-out wait
                               // polls, MMA wait polls, load wait polls
};

__global__ void k_lr_count(Batch B, int N, int R, int G, int* goff, int* ngroups, int* lidx_all,
                           int* oprefix_all, int* noob_r);
__global__ void k_lr_inbag(Batch B, int N, int R, int G, int T, const int* lidx_all,
                           const int* goff, uint16_t* code, int* order);
__global__ void k_lr_oob_keys(Batch B, int N, int R, const int* lidx_all, uint16_t* code,
                              unsigned long long* keys, int* nkeys);
__global__ void k_lr_oob_place(const unsigned long long* keys, int nkeys, int N, int M, int G,
                               const int* obase, const int* oprefix_all, const int* goff,
                               int* order);
// k_lr_leafsum / k_lr_scatter for a sketch width of 32 * nq columns (1 <= nq <= 8);
// false for another width.
bool lr_launch_leafsum(int nq, dim3 grid, cudaStream_t st, const int* order, const int* goff,
                       const int* ngroups, int N, int G, int T, const float* Z, float* LS);
bool lr_launch_scatter(int nq, int grid, cudaStream_t st, const uint16_t* code, int N, int R, int T,
                       int G, const float* LS, float* Y);
__global__ void k_lr_prep(const float* X, int R, int r, const int* nout, int W, float* Z);
__global__ void k_lr_combine(const float* CZ, int W, const float* X, int R, int r, const int* nout,
                             float* Y);
__global__ void k_lr_omega(float* X, int R, int r, unsigned long long seed);
__global__ void k_lr_gram(const float* A, int ra, const float* Bm, int rb, int R, int rows_per_block,
                          double* part);
__global__ void k_lr_gram_reduce(const double* part, int nblk, int ra, int rb, int sym, double* G);
__global__ void k_lr_symmetrize(double* G, int r);
__global__ void k_lr_chol_inv(const double* Gm, int r, double* Uinv);
__global__ void k_lr_rowmat(const float* Y, int R, int rin, const double* Mat, int rout, float* Out);
__global__ void k_lr_eig_select(const double* Tm, int r, int k, double* Mk, double* lam_out);
__global__ void k_lr_quantize(const float* A, int R, int k, int Rpad, int8_t* q, uint16_t* qb,
                              float* scale);
__global__ void k_lr_load_factors(const int8_t* qin, const float* sin, int R, int rank, int Rpad,
                                  int8_t* q, uint16_t* qb, float* scale);
__global__ void k_lr_norms(const int8_t* q, const float* scale, int R, float* norm, int* ids);
__global__ void k_lr_permute(const uint16_t* qb, const float* scale, const float* norm,
                             const int* order, int R, int Rpad, uint16_t* qbp, float* sp,
                             float* np, int* perm);
__global__ void k_topk_tc(const __grid_constant__ CUtensorMap tm, TopkArgs a);

}  // namespace rfx
