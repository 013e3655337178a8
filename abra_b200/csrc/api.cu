// api.cu -- the extern "C" surface of libabra_b200.so (declared in
// include/abra_b200.h).  Argument checking, error strings, the tuning table.
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "../../include/abra_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(ABRA_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

std::mutex g_tune_mu;
std::map<std::tuple<int64_t, int64_t, int, int>, int> g_tune;
std::map<std::tuple<int64_t, int64_t, int>, int> g_tune_q6;

// Default when the table has no entry: more k-parts for few rows or long K.
int default_candidate(int64_t N, int64_t K, int ncols, int nmat) {
    (void)nmat;
    const int64_t rg = (N + 7) / 8;
    const int64_t nsb = K / 256;
    (void)ncols;
    if (rg < 148) return nsb >= 16 ? 3082 : 3042;
    if (rg < 4 * 148) return nsb >= 16 ? 3042 : 3022;
    return nsb >= 24 ? 3022 : 3012;
}

int check_mmvq_args(const void *w, const void *x, const float *y, int64_t N, int64_t K,
                    int32_t ncols, int64_t ldy) {
    if (!w || !x || !y) return fail(ABRA_E_INVALID, "null pointer");
    if (N <= 0 || K <= 0) return fail(ABRA_E_INVALID, "N and K must be positive (N=%lld K=%lld)", (long long)N, (long long)K);
    if (K % 256 != 0) return fail(ABRA_E_INVALID, "K must be a multiple of QK_K=256 (K=%lld)", (long long)K);
    if (K > 65536) return fail(ABRA_E_UNSUPPORTED, "K=%lld too large (max 65536)", (long long)K);
    if (N > (int64_t)0x7fffffff - 8) return fail(ABRA_E_UNSUPPORTED, "N=%lld too large", (long long)N);
    if (ncols < 1 || ncols > 8) return fail(ABRA_E_UNSUPPORTED, "ncols must be in 1..8 (got %d)", ncols);
    if (ldy < N) return fail(ABRA_E_INVALID, "ldy (%lld) < N (%lld)", (long long)ldy, (long long)N);
    if (!aligned16(w) || !aligned16(x)) return fail(ABRA_E_INVALID, "weights and activations must be 16-byte aligned");
    return ABRA_OK;
}

// A K-shard: canonical slices [sl_base, sl_base + sl_cnt) of rows K_full wide,
// whose width must be K.  Fills the slicing options on success.
int check_kshard(int64_t K, int64_t K_full, int32_t sl_base, int32_t sl_cnt, abra::MmvqOpts &tp) {
    if (K_full <= 0 || K_full % 256 != 0 || K_full > 65536 || sl_base < 0 ||
        !(sl_cnt == 1 || sl_cnt == 2 || sl_cnt == 4 || sl_cnt == 8) || sl_base + sl_cnt > 8)
        return fail(ABRA_E_INVALID, "bad K-shard (K_full=%lld sl_base=%d sl_cnt=%d)",
                    (long long)K_full, sl_base, sl_cnt);
    const int nsb_g = static_cast<int>(K_full / 256);
    if ((abra::slice_start(nsb_g, sl_base + sl_cnt) - abra::slice_start(nsb_g, sl_base)) * 256 != K)
        return fail(ABRA_E_INVALID, "K=%lld is not the width of canonical slices [%d, %d) of K_full=%lld",
                    (long long)K, sl_base, sl_base + sl_cnt, (long long)K_full);
    tp.sl_nsb = nsb_g;
    tp.sl_base = sl_base;
    tp.sl_cnt = sl_cnt;
    return ABRA_OK;
}

}  // namespace

int abra::record_failure(int code, const char *msg) { return fail(code, "%s", msg); }

namespace abra {
static std::vector<ErrorWordFn> &error_words() {
    static std::vector<ErrorWordFn> v;
    return v;
}
int register_error_word(ErrorWordFn fn) {
    error_words().push_back(fn);
    return 1;
}
cudaError_t read_error_words(unsigned *value, bool clear) {
    for (ErrorWordFn fn : error_words()) {
        cudaError_t e = fn(value, clear);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
}  // namespace abra

extern "C" {

const char *abra_version(void) { return "abra_b200 0.1.0 sm_100a"; }
const char *abra_last_error(void) { return g_err; }

int abra_device_error(uint32_t *out, int32_t clear) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
    unsigned v = 0;
    e = abra::read_error_words(&v, clear != 0);
    if (e != cudaSuccess) return cuda_fail(e, "device error word");
    if (out) *out = v;
    return ABRA_OK;
}

static int mmvq_common(const void *w, const void *w2, const void *x, float *y, int64_t N,
                       int64_t K, int32_t ncols, int64_t ldy, int32_t candidate, int32_t flags,
                       void *stream) {
    int rc = check_mmvq_args(w, x, y, N, K, ncols, ldy);
    if (rc) return rc;
    if (w2 && !aligned16(w2)) return fail(ABRA_E_INVALID, "weights must be 16-byte aligned");
    int id = candidate;
    if (id == 0) id = abra_tune_get(N, K, ncols, w2 ? 2 : 1);
    const abra::MmvqConfig *cfg = abra::mmvq_candidate_by_id(id);
    if (!cfg) return fail(ABRA_E_INVALID, "unknown candidate id %d", id);
    cudaError_t e = abra::launch_mmvq_q4k(*cfg, w, w2, x, y, N, K, ncols, ldy,
                                          (flags & ABRA_MMVQ_PDL) ? abra::MMVQ_PDL : 0,
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "mmvq launch");
    return ABRA_OK;
}

int abra_q4k_mmvq_ex(const void *w, const void *x, float *y, int64_t N, int64_t K,
                     int32_t ncols, int64_t ldy, int32_t candidate, int32_t flags,
                     void *stream) {
    return mmvq_common(w, nullptr, x, y, N, K, ncols, ldy, candidate, flags, stream);
}

int abra_q4k_mmvq_swiglu(const void *w_gate, const void *w_up, const void *x, float *y,
                         int64_t N, int64_t K, int32_t ncols, int64_t ldy, int32_t candidate,
                         int32_t flags, void *stream) {
    if (!w_up) return fail(ABRA_E_INVALID, "null pointer");
    return mmvq_common(w_gate, w_up, x, y, N, K, ncols, ldy, candidate, flags, stream);
}

int abra_q4k_pack(const void *w, void *w_packed, int64_t nblocks, void *stream) {
    if (!w || !w_packed) return fail(ABRA_E_INVALID, "null pointer");
    if (nblocks <= 0) return fail(ABRA_E_INVALID, "nblocks must be positive");
    if (!aligned16(w) || !aligned16(w_packed)) return fail(ABRA_E_INVALID, "weights must be 16-byte aligned");
    cudaError_t e = abra::launch_q4k_pack(w, w_packed, nblocks, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "pack launch");
    return ABRA_OK;
}

int abra_q4k_mmvq_packed(const void *w_packed, const void *x, float *y, int64_t N, int64_t K, int32_t flags,
                         void *stream) {
    int rc = check_mmvq_args(w_packed, x, y, N, K, 1, N);
    if (rc) return rc;
    // the lane-mapped kernel, 2 CTAs per SM, the largest unit whose copies
    // stay 16-byte aligned for this width
    for (int id : {4082, 4042, 4022}) {
        const abra::MmvqConfig *cfg = abra::mmvq_candidate_by_id(id);
        int64_t pl[8];
        if (!cfg || !abra::mmvq_lane_plan(*cfg, N, static_cast<int>(K / abra::QK_K), 1, 0, pl, true)) continue;
        cudaError_t e = abra::launch_mmvq_lane(*cfg, w_packed, nullptr, x, y, N, K,
                                               (flags & ABRA_MMVQ_PDL) ? abra::MMVQ_PDL : 0,
                                               static_cast<cudaStream_t>(stream), nullptr, true);
        if (e != cudaSuccess) return cuda_fail(e, "packed mmvq launch");
        return ABRA_OK;
    }
    return fail(ABRA_E_UNSUPPORTED, "no packed plan for N=%lld K=%lld", (long long)N, (long long)K);
}

int abra_q4k_mmvq(const void *w, const void *x, float *y, int64_t N, int64_t K, int32_t ncols,
                  void *stream) {
    return abra_q4k_mmvq_ex(w, x, y, N, K, ncols, N, 0, 0, stream);
}

int abra_q4k_mmvq_kshard(const void *w, const void *x, float *y, int64_t N, int64_t K,
                         int32_t ncols, int64_t K_full, int32_t sl_base, int32_t sl_cnt,
                         int32_t candidate, int32_t flags, void *stream) {
    int rc = check_mmvq_args(w, x, y, N, K, ncols, N);
    if (rc) return rc;
    abra::MmvqOpts tp;
    rc = check_kshard(K, K_full, sl_base, sl_cnt, tp);
    if (rc) return rc;
    int id = candidate;
    if (id == 0) id = abra_tune_get(N, K, ncols, 1);
    const abra::MmvqConfig *cfg = abra::mmvq_candidate_by_id(id);
    if (!cfg) return fail(ABRA_E_INVALID, "unknown candidate id %d", id);
    cudaError_t e = abra::launch_mmvq_q4k(*cfg, w, nullptr, x, y, N, K, ncols, N,
                                          (flags & ABRA_MMVQ_PDL) ? abra::MMVQ_PDL : 0,
                                          static_cast<cudaStream_t>(stream), nullptr, &tp);
    if (e != cudaSuccess) return cuda_fail(e, "mmvq launch");
    return ABRA_OK;
}

int abra_q4k_mmvq_tc(const void *w, const void *x, float *y, int64_t N, int64_t K,
                     int32_t ncols, int64_t ldy, int32_t ks, float *workspace, int32_t flags,
                     void *stream) {
    if (ncols != 32) return fail(ABRA_E_UNSUPPORTED, "the tensor-core MMVQ takes 32 columns (got %d)", ncols);
    if (!w || !x || !y) return fail(ABRA_E_INVALID, "null pointer");
    if (N <= 0 || K <= 0 || K % 256 != 0) return fail(ABRA_E_INVALID, "K must be a positive multiple of QK_K=256 (K=%lld)", (long long)K);
    if (K > 65536 || N > (int64_t)0x7fffffff - 128) return fail(ABRA_E_UNSUPPORTED, "shape too large");
    if (ldy < N) return fail(ABRA_E_INVALID, "ldy (%lld) < N (%lld)", (long long)ldy, (long long)N);
    if (!(ks == 1 || ks == 2 || ks == 4 || ks == 8)) return fail(ABRA_E_INVALID, "ks must be 1, 2, 4 or 8");
    if (ks > 1 && !workspace) return fail(ABRA_E_INVALID, "ks > 1 needs a workspace of ks*32*N floats");
    if (!aligned16(w) || (reinterpret_cast<uintptr_t>(x) & 3u)) return fail(ABRA_E_INVALID, "weights 16-byte and activations 4-byte aligned");
    cudaError_t e = abra::launch_mmvq_tc(w, x, y, N, K, ldy, ks, workspace,
                                         (flags & ABRA_MMVQ_PDL) ? abra::MMVQ_PDL : 0,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core mmvq launch");
    return ABRA_OK;
}

int abra_q4k_mmvq_combined(int32_t candidate, const void *w, const float *x, void *xq,
                           float *y, int64_t N, int64_t K, int32_t ncols, void *stream) {
    if (!x) return fail(ABRA_E_INVALID, "null pointer");
    int rc = check_mmvq_args(w, xq, y, N, K, ncols, N);
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(x) & 3u) return fail(ABRA_E_INVALID, "x must be 4-byte aligned");
    // resolve the candidate before anything is launched: a refused call
    // leaves the Q8_1 buffer untouched
    const int id = candidate ? candidate : abra_tune_get(N, K, ncols, 1);
    if (!abra::mmvq_candidate_by_id(id)) return fail(ABRA_E_INVALID, "unknown candidate id %d", id);
    cudaError_t e = abra::launch_quantize_q8_1(x, xq, K, ncols, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    return mmvq_common(w, nullptr, xq, y, N, K, ncols, N, candidate, 0, stream);
}

int abra_q4k_mmvq_candidate(int32_t candidate, const void *w, const void *x, float *y,
                            int64_t N, int64_t K, int32_t ncols, void *stream) {
    if (candidate == 0) return fail(ABRA_E_INVALID, "candidate id 0 is the tuned dispatch; use abra_q4k_mmvq");
    return abra_q4k_mmvq_ex(w, x, y, N, K, ncols, N, candidate, 0, stream);
}

int abra_q4k_mmvq_partials(const void *w, const void *x, float *y, int32_t *P, int32_t *M,
                           int64_t N, int64_t K, int32_t ncols, int32_t ks, void *stream) {
    int rc = check_mmvq_args(w, x, y, N, K, ncols, N);
    if (rc) return rc;
    if (!P || !M) return fail(ABRA_E_INVALID, "null partials pointer");
    if (!(ncols == 1 || ncols == 2 || ncols == 4 || ncols == 8))
        return fail(ABRA_E_UNSUPPORTED, "partials: ncols must be 1, 2, 4 or 8");
    if (!(ks == 1 || ks == 2 || ks == 4)) return fail(ABRA_E_UNSUPPORTED, "partials: ks must be 1, 2 or 4");
    cudaError_t e = abra::launch_mmvq_q4k_partials(w, x, y, P, M, N, K, ncols, ks,
                                                   static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "mmvq partials launch");
    return ABRA_OK;
}

void launch_pinned_upstream_mmvq(const void *d_w_q4, const void *d_x_q8, float *d_y, int64_t N,
                                 int64_t K, void *stream) {
    abra_q4k_mmvq(d_w_q4, d_x_q8, d_y, N, K, 1, stream);
}

int abra_quantize_q8_1(const float *x, void *xq, int64_t K, int32_t ncols, void *stream) {
    if (!x || !xq) return fail(ABRA_E_INVALID, "null pointer");
    if (K <= 0 || K % 32 != 0) return fail(ABRA_E_INVALID, "K must be a positive multiple of QK8_1=32 (K=%lld)", (long long)K);
    if (ncols < 1) return fail(ABRA_E_INVALID, "ncols must be >= 1");
    if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(xq) & 3u))
        return fail(ABRA_E_INVALID, "x and x_q8_1 must be 4-byte aligned");
    cudaError_t e = abra::launch_quantize_q8_1(x, xq, K, ncols, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    return ABRA_OK;
}

void launch_pinned_upstream_q8_1_quantize(const float *d_x_f32, void *d_x_q8, int64_t K,
                                          void *stream) {
    abra_quantize_q8_1(d_x_f32, d_x_q8, K, 1, stream);
}

int abra_rmsnorm_quantize_q8_1(const float *x, const float *w, float eps, void *xq,
                               float *xn_out, int64_t K, int32_t ncols, void *stream) {
    if (!x || !w || !xq) return fail(ABRA_E_INVALID, "null pointer");
    if (K <= 0 || K % 32 != 0 || K > 16384)
        return fail(ABRA_E_INVALID, "K must be a multiple of 32 in 32..16384 (K=%lld)", (long long)K);
    if (ncols < 1) return fail(ABRA_E_INVALID, "ncols must be >= 1");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
         reinterpret_cast<uintptr_t>(xq) | reinterpret_cast<uintptr_t>(xn_out)) & 3u)
        return fail(ABRA_E_INVALID, "x, w, x_q8_1 and xn_out must be 4-byte aligned");
    cudaError_t e = abra::launch_rmsnorm_quantize_q8_1(x, w, eps, xq, xn_out, K, ncols,
                                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm_quantize launch");
    return ABRA_OK;
}

int abra_q4k_mmvq_rmsnorm(const void *w, const void *w_up, const float *x, const float *norm_w,
                          float eps, float *y, void *x_q8_out, int64_t N, int64_t K,
                          int32_t candidate, int32_t flags, void *stream) {
    if (!w || !x || !norm_w || !y) return fail(ABRA_E_INVALID, "null pointer");
    if (N <= 0 || K <= 0) return fail(ABRA_E_INVALID, "N and K must be positive (N=%lld K=%lld)", (long long)N, (long long)K);
    if (K % 256 != 0) return fail(ABRA_E_INVALID, "K must be a multiple of QK_K=256 (K=%lld)", (long long)K);
    if (K > 16384) return fail(ABRA_E_UNSUPPORTED, "K=%lld too large for the fused RMSNorm (max 16384)", (long long)K);
    if (N > (int64_t)0x7fffffff - 8) return fail(ABRA_E_UNSUPPORTED, "N=%lld too large", (long long)N);
    if (!aligned16(w) || (w_up && !aligned16(w_up)) || !aligned16(norm_w))
        return fail(ABRA_E_INVALID, "weights and norm weights must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
         reinterpret_cast<uintptr_t>(x_q8_out)) & 3u)
        return fail(ABRA_E_INVALID, "x, y and x_q8_out must be 4-byte aligned");
    const int nmat = w_up ? 2 : 1;
    int id = candidate;
    if (id == 0) id = abra_tune_get(N, K, 1, nmat);
    const abra::MmvqConfig *cfg = abra::mmvq_candidate_by_id(id);
    if (!cfg) return fail(ABRA_E_INVALID, "unknown candidate id %d", id);
    abra::MmvqXin xin = {};
    xin.h_in = x;
    xin.norm_w = norm_w;
    xin.eps = eps;
    xin.x_out = static_cast<uint8_t *>(x_q8_out);
    cudaError_t e = abra::launch_mmvq_q4k_xin(*cfg, w, w_up, xin, y, N, K,
                                              (flags & ABRA_MMVQ_PDL) ? abra::MMVQ_PDL : 0,
                                              static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidConfiguration)
        return fail(ABRA_E_UNSUPPORTED, "candidate %d has no fused-RMSNorm plan for N=%lld K=%lld", id,
                    (long long)N, (long long)K);
    if (e != cudaSuccess) return cuda_fail(e, "fused rmsnorm mmvq launch");
    return ABRA_OK;
}

int abra_gen_q4k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset, void *stream) {
    if (!dst || nblocks < 0 || block_offset < 0) return fail(ABRA_E_INVALID, "bad generator arguments");
    if (reinterpret_cast<uintptr_t>(dst) & 7u) return fail(ABRA_E_INVALID, "dst must be 8-byte aligned");
    cudaError_t e = abra::launch_gen_q4k(dst, nblocks, seed, tensor_id, block_offset,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "gen_q4k launch");
    return ABRA_OK;
}

int abra_gen_uniform_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                         int64_t offset_index, float scale, float offset, void *stream) {
    if (!dst || n < 0 || offset_index < 0) return fail(ABRA_E_INVALID, "bad generator arguments");
    if (reinterpret_cast<uintptr_t>(dst) & 3u) return fail(ABRA_E_INVALID, "dst must be 4-byte aligned");
    cudaError_t e = abra::launch_gen_uniform_f32(dst, n, seed, tensor_id, offset_index, scale,
                                                 offset, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "gen_uniform launch");
    return ABRA_OK;
}

// ------------------------------------------------------------- Q6_K ---
static int q6k_common(const void *w, const void *x, float *y, int64_t N, int64_t K,
                      int32_t ncols, int64_t ldy, int32_t candidate, int32_t flags,
                      const abra::MmvqOpts *tp, void *stream) {
    int id = candidate;
    if (id == 0) id = abra_q6k_tune_get(N, K, ncols);
    const abra::MmvqConfig *cfg = abra::q6k_candidate_by_id(id);
    if (!cfg) return fail(ABRA_E_INVALID, "unknown Q6_K candidate id %d", id);
    cudaError_t e = abra::launch_mmvq_q6k(*cfg, w, x, y, N, K, ncols, ldy,
                                          (flags & ABRA_MMVQ_PDL) ? abra::MMVQ_PDL : 0,
                                          static_cast<cudaStream_t>(stream), nullptr, tp);
    if (e == cudaErrorInvalidConfiguration)
        return fail(ABRA_E_UNSUPPORTED, "Q6_K candidate %d does not fit N=%lld K=%lld ncols=%d", id,
                    (long long)N, (long long)K, ncols);
    if (e != cudaSuccess) return cuda_fail(e, "q6k mmvq launch");
    return ABRA_OK;
}

int abra_q6k_mmvq_ex(const void *w, const void *x, float *y, int64_t N, int64_t K, int32_t ncols,
                     int64_t ldy, int32_t candidate, int32_t flags, void *stream) {
    int rc = check_mmvq_args(w, x, y, N, K, ncols, ldy);
    if (rc) return rc;
    return q6k_common(w, x, y, N, K, ncols, ldy, candidate, flags, nullptr, stream);
}

int abra_q6k_mmvq(const void *w, const void *x, float *y, int64_t N, int64_t K, int32_t ncols,
                  void *stream) {
    return abra_q6k_mmvq_ex(w, x, y, N, K, ncols, N, 0, 0, stream);
}

int abra_q6k_mmvq_kshard(const void *w, const void *x, float *y, int64_t N, int64_t K,
                         int32_t ncols, int64_t K_full, int32_t sl_base, int32_t sl_cnt,
                         int32_t candidate, int32_t flags, void *stream) {
    int rc = check_mmvq_args(w, x, y, N, K, ncols, N);
    if (rc) return rc;
    abra::MmvqOpts tp;
    rc = check_kshard(K, K_full, sl_base, sl_cnt, tp);
    if (rc) return rc;
    return q6k_common(w, x, y, N, K, ncols, N, candidate, flags, &tp, stream);
}

int abra_q6k_mmvq_partials(const void *w, const void *x, float *y, int32_t *P, int64_t N,
                           int64_t K, int32_t ncols, void *stream) {
    int rc = check_mmvq_args(w, x, y, N, K, ncols, N);
    if (rc) return rc;
    if (!P) return fail(ABRA_E_INVALID, "null partials pointer");
    cudaError_t e = abra::launch_mmvq_q6k_partials(w, x, y, P, N, K, ncols,
                                                   static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidConfiguration)
        return fail(ABRA_E_UNSUPPORTED, "Q6_K partials do not fit N=%lld K=%lld ncols=%d",
                    (long long)N, (long long)K, ncols);
    if (e != cudaSuccess) return cuda_fail(e, "q6k partials launch");
    return ABRA_OK;
}

int abra_gen_q6k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset, void *stream) {
    if (!dst || nblocks < 0 || block_offset < 0) return fail(ABRA_E_INVALID, "bad generator arguments");
    if (reinterpret_cast<uintptr_t>(dst) & 1u) return fail(ABRA_E_INVALID, "dst must be 2-byte aligned");
    cudaError_t e = abra::launch_gen_q6k(dst, nblocks, seed, tensor_id, block_offset,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "gen_q6k launch");
    return ABRA_OK;
}

int abra_q6k_candidate_count(void) {
    int n = 0;
    abra::q6k_candidates(&n);
    return n;
}

int abra_q6k_candidate_info(int32_t index, int32_t *id, int32_t *mode, int32_t *ks,
                            int32_t *ctas_per_sm, int32_t *stage_kb) {
    int n = 0;
    const abra::MmvqConfig *c = abra::q6k_candidates(&n);
    if (index < 0 || index >= n) return fail(ABRA_E_INVALID, "candidate index %d out of range", index);
    if (id) *id = c[index].id;
    if (mode) *mode = c[index].mode;
    if (ks) *ks = c[index].ks;
    if (ctas_per_sm) *ctas_per_sm = c[index].ctas_per_sm;
    if (stage_kb) *stage_kb = c[index].stage_kb;
    return ABRA_OK;
}

int abra_q6k_tune_set(int64_t N, int64_t K, int32_t ncols, int32_t candidate) {
    if (!abra::q6k_candidate_by_id(candidate)) return fail(ABRA_E_INVALID, "unknown Q6_K candidate id %d", candidate);
    std::lock_guard<std::mutex> lock(g_tune_mu);
    g_tune_q6[std::make_tuple(N, K, static_cast<int>(ncols))] = candidate;
    return ABRA_OK;
}

int abra_q6k_tune_get(int64_t N, int64_t K, int32_t ncols) {
    {
        std::lock_guard<std::mutex> lock(g_tune_mu);
        auto it = g_tune_q6.find(std::make_tuple(N, K, static_cast<int>(ncols)));
        if (it != g_tune_q6.end()) return it->second;
    }
    return abra::q6k_default_candidate(N, K, ncols);
}

int abra_mmvq_plan_info(int32_t ggml_type, int32_t candidate, int64_t N, int64_t K, int32_t ncols,
                        int32_t nmat, int32_t xin, int64_t K_full, int32_t sl_base, int32_t sl_cnt,
                        int32_t sm_count, int64_t *out) {
    if (!out) return fail(ABRA_E_INVALID, "null pointer");
    if (ggml_type != ABRA_GGML_Q4_K && ggml_type != ABRA_GGML_Q6_K)
        return fail(ABRA_E_INVALID, "ggml_type must be Q4_K (12) or Q6_K (14)");
    if (N <= 0 || K <= 0 || K % 256 != 0 || K > 65536 || N > (int64_t)0x7fffffff - 8)
        return fail(ABRA_E_INVALID, "bad shape N=%lld K=%lld", (long long)N, (long long)K);
    if (ncols < 1 || ncols > 8) return fail(ABRA_E_UNSUPPORTED, "ncols must be in 1..8 (got %d)", ncols);
    if (nmat != 1 && !(nmat == 2 && ggml_type == ABRA_GGML_Q4_K))
        return fail(ABRA_E_INVALID, "nmat must be 1 (or 2 for the Q4_K gate/up form)");
    if (xin && (ggml_type != ABRA_GGML_Q4_K || ncols != 1))
        return fail(ABRA_E_INVALID, "the fused RMSNorm prologue is Q4_K at batch 1");
    if (sm_count < 0) return fail(ABRA_E_INVALID, "sm_count must be >= 0");
    abra::MmvqOpts tp;
    const abra::MmvqOpts *ptp = nullptr;
    if (K_full > 0) {
        const int rc = check_kshard(K, K_full, sl_base, sl_cnt, tp);
        if (rc) return rc;
        ptp = &tp;
    }
    const bool q6 = ggml_type == ABRA_GGML_Q6_K;
    int id = candidate;
    if (id == 0) id = q6 ? abra_q6k_tune_get(N, K, ncols) : abra_tune_get(N, K, ncols, nmat);
    const abra::MmvqConfig *cfg = q6 ? abra::q6k_candidate_by_id(id) : abra::mmvq_candidate_by_id(id);
    if (!cfg) return fail(ABRA_E_INVALID, "unknown candidate id %d", id);
    const bool ok = q6 ? abra::q6k_plan_info(*cfg, N, K, ncols, ptp, sm_count, out)
                       : abra::mmvq_plan_info(*cfg, N, K, ncols, nmat, xin != 0, ptp, sm_count, out);
    if (!ok)
        return fail(ABRA_E_UNSUPPORTED, "candidate %d has no plan for N=%lld K=%lld ncols=%d", id,
                    (long long)N, (long long)K, ncols);
    return ABRA_OK;
}

int abra_candidate_count(void) {
    int n = 0;
    abra::mmvq_candidates(&n);
    return n;
}

int abra_candidate_info(int32_t index, int32_t *id, int32_t *mode, int32_t *ks, int32_t *ncw,
                        int32_t *ctas_per_sm, int32_t *stage_kb) {
    int n = 0;
    const abra::MmvqConfig *c = abra::mmvq_candidates(&n);
    if (index < 0 || index >= n) return fail(ABRA_E_INVALID, "candidate index %d out of range", index);
    if (id) *id = c[index].id;
    if (mode) *mode = c[index].mode;
    if (ks) *ks = c[index].ks;
    if (ncw) *ncw = 8;
    if (ctas_per_sm) *ctas_per_sm = c[index].ctas_per_sm;
    if (stage_kb) *stage_kb = c[index].stage_kb;
    return ABRA_OK;
}

int abra_tune_set(int64_t N, int64_t K, int32_t ncols, int32_t nmat, int32_t candidate) {
    if (!abra::mmvq_candidate_by_id(candidate)) return fail(ABRA_E_INVALID, "unknown candidate id %d", candidate);
    if (nmat != 1 && nmat != 2) return fail(ABRA_E_INVALID, "nmat must be 1 or 2");
    std::lock_guard<std::mutex> lock(g_tune_mu);
    g_tune[std::make_tuple(N, K, static_cast<int>(ncols), static_cast<int>(nmat))] = candidate;
    return ABRA_OK;
}

int abra_tune_get(int64_t N, int64_t K, int32_t ncols, int32_t nmat) {
    {
        std::lock_guard<std::mutex> lock(g_tune_mu);
        auto it = g_tune.find(std::make_tuple(N, K, static_cast<int>(ncols), static_cast<int>(nmat)));
        if (it != g_tune.end()) return it->second;
    }
    return default_candidate(N, K, ncols, nmat);
}

int abra_tune_clear(void) {
    std::lock_guard<std::mutex> lock(g_tune_mu);
    g_tune.clear();
    g_tune_q6.clear();
    return ABRA_OK;
}

}  // extern "C"
