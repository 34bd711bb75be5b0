// rfx_prox_dense_static: the dense proximity export of rfx_prox_dense without any device
// allocation, for callers that may not call cudaMalloc -- code running inside a host
// application that owns the device memory budget (a memory pool or a serving process that
// forbids allocations after start-up), or code driven from a context where allocating would
// synchronise the device.  Row blocks are staged in one fixed device array declared here.
#include <algorithm>
#include <mutex>
#include <string>

#include "../../include/rfx_b200.h"
#include "rfx_device.cuh"
#include "rfx_kernels.h"

namespace {

// Staging area for finished proximity rows: RFX_STATIC_SCRATCH_FLOATS floats (16 MiB),
// resident on every GPU that loads the library until the process exits.
static __device__ __align__(256) float g_prox_scratch[RFX_STATIC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

}  // namespace

// Records the message returned by rfx_last_error() (rfx_host.cu).
void rfx_record_error(const std::string& msg);

namespace {
int fail(int code, const std::string& msg) {
    rfx_record_error(msg);
    return code;
}
}  // namespace

extern "C" int rfx_prox_dense_static(const int* upper_dev, const int* nout_dev, int R,
                                     int row_begin, int row_end, float* out_host, void* stream) {
    if (!upper_dev || !nout_dev || !out_host) return fail(RFX_ERR_ARG, "null pointer");
    if (R < 1 || row_begin < 0 || row_begin > row_end || row_end > R)
        return fail(RFX_ERR_ARG, "bad row range");
    if ((long long)R > (long long)RFX_STATIC_SCRATCH_FLOATS)
        return fail(RFX_ERR_ARG, "R = " + std::to_string(R) + " exceeds the static scratch: one row " +
                                 "must fit in " + std::to_string(RFX_STATIC_SCRATCH_FLOATS) + " floats");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(RFX_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(RFX_ERR_ARG, "device index out of range");
    float* scratch = nullptr;
    {
        // Once per device, with that device current: the host-side symbol is only a stand-in,
        // the kernel must be given the device address.
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            e = cudaGetSymbolAddress(reinterpret_cast<void**>(&g_scratch_addr[dev]), g_prox_scratch);
            if (e != cudaSuccess) {
                g_scratch_addr[dev] = nullptr;
                return fail(RFX_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            }
        }
        scratch = g_scratch_addr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int rows_per = (int)std::max<long long>(1, (long long)RFX_STATIC_SCRATCH_FLOATS / R);
    for (int r0 = row_begin; r0 < row_end; r0 += rows_per) {
        const int r1 = std::min(row_end, r0 + rows_per);
        const long long total = (long long)(r1 - r0) * R;
        e = rfx::launch_prox_finish(upper_dev, nout_dev, R, r0, r1, scratch, st);
        if (e != cudaSuccess) return fail(RFX_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
        e = cudaMemcpyAsync(out_host + (size_t)(r0 - row_begin) * R, scratch, (size_t)total * 4,
                            cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return fail(RFX_ERR_CUDA, cudaGetErrorString(e));
    }
    return RFX_OK;
}
