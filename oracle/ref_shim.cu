// ref_shim.cu -- glue that lets the reference's own Q4_K kernel family be
// compiled here, unmodified, into oracle/_ref/libq4k_ref.so.
//
// TEST INFRASTRUCTURE ONLY: the reference's kernels run as a reference result and as a
// timing comparison, never as part of libabra_b200.
//
// The reference's kernels/q4k/q4k_q8_mmvq.cu and q4k_family.cu are compiled
// from the reference tree as they are (see oracle/Makefile).  They reference
// the upstream ggml adapter (kernels/q4k/upstream_adapter.cuh:12-26), whose
// definition needs llama.cpp/ggml sources that are not available; the two
// symbols are defined here to record the call and do nothing, so that only
// the reference's own kernels (candidates 101..2082 and
// launch_custom_reference_q8_1_quantizer) are exercised.  A flat extern "C"
// surface is added for ctypes.
#include <cstdint>
#include <exception>

#include "kernels/q4k/q4k_family.cuh"
#include "kernels/q4k/q4k_q8_mmvq.cuh"
#include "kernels/q4k/upstream_adapter.cuh"

static int g_upstream_calls = 0;

extern "C" void launch_pinned_upstream_mmvq(const void *, const void *, float *, int64_t, int64_t,
                                            cudaStream_t) {
    ++g_upstream_calls;
}
extern "C" void launch_pinned_upstream_q8_1_quantize(const float *, void *, int64_t,
                                                     cudaStream_t) {
    ++g_upstream_calls;
}
extern "C" void quantize_row_q4_K_upstream_cpu(const float *, block_q4_K *, int64_t) {
    ++g_upstream_calls;
}
extern "C" void dequantize_row_q4_K_upstream_cpu(const block_q4_K *, float *, int64_t) {
    ++g_upstream_calls;
}

extern "C" {

int ref_upstream_calls(void) { return g_upstream_calls; }

// Candidate ids of the reference family, excluding the upstream one (0).
int ref_candidate_ids(int *out, int cap) {
    int n = 0;
    for (Q4KCandidateID id : get_all_candidate_ids()) {
        if (id == CANDIDATE_UPSTREAM_MMVQ) continue;
        if (n < cap) out[n] = static_cast<int>(id);
        ++n;
    }
    return n;
}

// 0 on success, -1 if the reference threw (invalid shape or id).
int ref_launch_candidate(int id, const void *w, const void *x, float *y, int N, int K,
                         void *stream) {
    try {
        launch_q4k_candidate(static_cast<Q4KCandidateID>(id),
                             static_cast<const block_q4_K *>(w),
                             static_cast<const block_q8_1 *>(x), y, N, K,
                             static_cast<cudaStream_t>(stream));
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}

int ref_launch_variant(int variant, const void *w, const void *x, float *y, int N, int K,
                       void *stream) {
    try {
        launch_q4k_q8_mmvq(static_cast<Q4KVariant>(variant), static_cast<const block_q4_K *>(w),
                           static_cast<const block_q8_1 *>(x), y, N, K,
                           static_cast<cudaStream_t>(stream));
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}

int ref_quantize_q8_1(const float *x, void *y, int K, void *stream) {
    try {
        launch_custom_reference_q8_1_quantizer(x, static_cast<block_q8_1 *>(y), K,
                                               static_cast<cudaStream_t>(stream));
    } catch (const std::exception &) {
        return -1;
    }
    return 0;
}

int ref_autotuned_candidate(int N, int K, int arch) {
    return static_cast<int>(get_autotuned_candidate_for_shape(N, K, arch));
}

}  // extern "C"
