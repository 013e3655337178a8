// failure_probe.cu -- failure detection without a GPU fault.  One CTA waits
// on a device counter that nothing increments, with the bounded cross-rank
// wait of the tensor-parallel kernels (wait_count: WAIT_LIMIT_NS, then
// ERR_FLAG_TIMEOUT and return).  The host reads the error word; the context
// stays usable.  This is the path a rank that left mid-run takes on its peers.
#include "../../include/abra_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace abra {

__global__ void flag_wait_probe_kernel(const unsigned long long *cnt, unsigned long long target,
                                       unsigned long long *waited_ns) {
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer_ns();
        wait_count(cnt, target);
        *waited_ns = globaltimer_ns() - t0;
    }
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_failure_probe)

extern "C" int abra_test_flag_timeout(uint32_t *error_bits, uint64_t *waited_ns) {
    unsigned long long *d = nullptr;  // [0] the counter nothing increments, [1] the wait's duration
    cudaError_t e = cudaMalloc(&d, 2 * sizeof(unsigned long long));
    if (e != cudaSuccess) return abra::record_failure(ABRA_E_CUDA, "probe allocation");
    unsigned long long h[2] = {0, 0};
    e = cudaMemset(d, 0, sizeof h);
    if (e == cudaSuccess) {
        abra::flag_wait_probe_kernel<<<1, 32>>>(d, 1ull, d + 1);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(h, d, sizeof h, cudaMemcpyDeviceToHost);
    unsigned bits = 0;
    if (e == cudaSuccess) e = abra::read_error_words(&bits, true);
    cudaFree(d);
    if (e != cudaSuccess) return abra::record_failure(ABRA_E_CUDA, cudaGetErrorString(e));
    if (error_bits) *error_bits = bits;
    if (waited_ns) *waited_ns = h[1];
    return ABRA_OK;
}
