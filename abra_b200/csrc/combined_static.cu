// combined_static.cu -- the combined pipeline (fp32 -> Q8_1 -> Q4_K MMVQ)
// with its Q8_1 scratch in a file-scope device array, so a call allocates
// nothing.
//
// Who needs it: a caller that may not allocate device memory where it
// multiplies.  Examples are an operator hook inside a host runtime that has
// already reserved the whole device for its own pool (a cudaMalloc there
// fails or steals from the pool), and latency-critical decode loops that
// must not hit cudaMalloc's implicit device synchronisation or its failure
// path.  Such a caller cannot hand abra_q4k_mmvq_combined a scratch buffer of
// its own either, because the runtime owns every buffer it could pass.
//
// Limits and rules:
//   * K * ncols <= kMaxValues (131,072 fp32 values, i.e. 147,456 bytes of
//     Q8_1 blocks); larger requests are refused with ABRA_E_UNSUPPORTED.
//   * Nothing in the scratch has to start at zero: every call's quantize
//     kernel writes each Q8_1 byte that the following MMVQ launch reads.
//   * One scratch per device.  Calls on one stream are ordered and safe;
//     calls that can overlap on the same device (different streams, or
//     different host threads on different streams) race on the scratch.
//   * The first call on each device sets up the scratch address for that
//     device (cudaGetSymbolAddress, with that device current); make that
//     first call before any stream capture.
//   * That address is kept for the life of the process.  cudaDeviceReset (or
//     anything else that destroys the device's primary context) reloads the
//     array elsewhere, so after it this entry point must not be called again
//     on that device in the same process.
//   * A refused call (bad sizes or candidate id) launches nothing and leaves
//     the scratch as it was.
#include <cstdint>
#include <mutex>

#include "../../include/abra_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr int64_t kMaxValues = 131072;                                   // K * ncols
constexpr size_t kScratchBytes = static_cast<size_t>(kMaxValues / 32) * 36;  // Q8_1 blocks
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_q8_scratch[kScratchBytes];

std::mutex g_setup_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// Address of this device's scratch; resolved once per device.
int scratch_for_current_device(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return abra::record_failure(ABRA_E_CUDA, "cudaGetDevice failed");
    if (dev < 0 || dev >= kMaxDevices)
        return abra::record_failure(ABRA_E_UNSUPPORTED, "device ordinal outside 0..63");
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_q8_scratch);
        if (e != cudaSuccess || !p)
            return abra::record_failure(ABRA_E_CUDA, "cudaGetSymbolAddress of the static Q8_1 scratch failed");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return ABRA_OK;
}

}  // namespace

extern "C" int abra_q4k_mmvq_combined_static(int32_t candidate, const void *w, const float *x,
                                             float *y, int64_t N, int64_t K, int32_t ncols,
                                             void *stream) {
    if (K > 0 && ncols > 0 && K * static_cast<int64_t>(ncols) > kMaxValues)
        return abra::record_failure(ABRA_E_UNSUPPORTED,
                                    "abra_q4k_mmvq_combined_static: K*ncols exceeds the static "
                                    "Q8_1 scratch (131072 values, 147456 bytes)");
    void *xq = nullptr;
    const int rc = scratch_for_current_device(&xq);
    if (rc != ABRA_OK) return rc;
    return abra_q4k_mmvq_combined(candidate, w, x, xq, y, N, K, ncols, stream);
}
