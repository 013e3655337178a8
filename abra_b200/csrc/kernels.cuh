// kernels.cuh -- host-side launchers shared between the .cu files of
// libabra_b200.  Nothing here crosses the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace abra {

// ---------------------------------------------------------------- MMVQ ---
// One tuning candidate of the Q4_K x Q8_1 MMVQ family.
struct MmvqConfig {
    int id;           // stable candidate id (used in tuning tables)
    int mode;         // MmvqMode: 0 TMA per-row copies, 1 TMA whole unit, 2 direct loads, 3 lane-mapped
    int ks;           // k-parts per row group (1, 2, 4, 8): warps sharing a row group;
                      // MODE_LANE: the largest rows per unit (8, 4, 2, 1)
    int ctas_per_sm;  // grid = min(row groups, SMs * ctas_per_sm)
    int stage_kb;     // shared-memory budget for the weight ring, KiB (TMA modes)
};

const MmvqConfig *mmvq_candidates(int *count);
const MmvqConfig *mmvq_candidate_by_id(int id);

// flags for launch_mmvq_q4k
enum : int {
    MMVQ_PDL = 1,  // launch with programmatic dependent launch (weights must be immutable)
};

// Options of one MMVQ launch (all off by default): tensor-parallel slicing,
// push and wait, and an L2 prefetch of other weights.
struct MmvqOpts {
    // K-shard slicing: the shard holds global canonical slices
    // [sl_base, sl_base + sl_cnt) of rows of sl_nsb superblocks (0: unsharded)
    int sl_nsb = 0, sl_base = 0, sl_cnt = 8;
    int row_offset = 0;  // global id of local row 0 (argmax keys)
    // push: rows to peer_y[q] (when set); CTAs count themselves on cta_cnt
    // (this GPU, never reset: a multiple of the grid after each launch); the
    // last one forwards the argmax keys to peer_amax[q] (when set) and adds
    // one arrival to peer_cnt[q], for q < npeer
    int npeer = 0;
    float *peer_y[8] = {};
    unsigned long long *peer_amax[8] = {};
    unsigned long long *peer_cnt[8] = {};
    unsigned long long *cta_cnt = nullptr;
    // fused-input wait: *wait_cnt >= (*epoch + 1) * wait_per_step
    const unsigned long long *wait_cnt = nullptr;
    const unsigned long long *epoch = nullptr;
    unsigned long long wait_per_step = 0;
    // L2 prefetch of up to two regions (the next kernels' weights), split
    // evenly over the CTAs; 16-byte aligned, sizes multiples of 16
    const void *pf_ptr[2] = {};
    int64_t pf_bytes[2] = {};
};

// w2 != nullptr selects the fused gate/up form: y = (w2 x) * silu(w x).
// amax != nullptr: also atomicMax an argmax key (value, row) per column into
// amax[c] (keys must start at 0).
cudaError_t launch_mmvq_q4k(const MmvqConfig &cfg, const void *w, const void *w2,
                            const void *x_q8, float *y, int64_t N, int64_t K, int ncols,
                            int64_t ldy, int flags, cudaStream_t stream,
                            unsigned long long *amax = nullptr, const MmvqOpts *tp = nullptr);
// Grid size the launch above would use (for arrival counts).
int mmvq_grid(const MmvqConfig &cfg, int64_t N, int64_t K, int ncols, int nmat, bool xin,
              const MmvqOpts *tp = nullptr);
// Fused input of launch_mmvq_q4k_xin: x = h_in + tree(deltas) (written to
// h_out when not null), quantized as Q8_1 of RMSNorm(x) * norm_w.
struct MmvqXin {
    const float *h_in;
    float *h_out;
    DeltaSet deltas;
    const float *norm_w;
    float eps;
    // when set (4-byte aligned): CTA 0 also stores the Q8_1 activation
    // (K/32 blocks), for another MMVQ on the same normalized input
    uint8_t *x_out = nullptr;
};
// Batch-1 MMVQ whose activation is built in each CTA from the fp32 residual
// stream (residual add + RMSNorm + Q8_1 fused into the prologue).
// The lane-mapped batch-1 kernel (mmvq_lane.cu): plan out = {grid, block,
// ring slots, slot bytes, shared memory, log2 rows per unit, activation and
// ring offsets}; false when the shape does not fit the candidate.
// packed: the weights are the 148-byte prepacked form (launch_q4k_pack).
bool mmvq_lane_plan(const MmvqConfig &cfg, int64_t N, int nsb, int nmat, int sms, int64_t out[8],
                    bool packed = false);
cudaError_t prepare_mmvq_lane(const MmvqConfig &cfg, int nmat);  // kernel attributes, outside a capture
cudaError_t launch_mmvq_lane(const MmvqConfig &cfg, const void *w, const void *w2, const void *x_q8, float *y,
                             int64_t N, int64_t K, int flags, cudaStream_t stream, unsigned long long *amax,
                             bool packed = false);
// Q4_K superblocks -> the reference's 148-byte prepacked form.
cudaError_t launch_q4k_pack(const void *w, void *w_packed, int64_t nblocks, cudaStream_t stream);
// The candidate a MODE_LANE candidate stands for where the lane kernel does
// not apply (batch > 1, fused input, tensor-parallel options); others as given.
const MmvqConfig &mmvq_classic(const MmvqConfig &cfg);

cudaError_t launch_mmvq_q4k_xin(const MmvqConfig &cfg, const void *w, const void *w2,
                                const MmvqXin &xin, float *y, int64_t N, int64_t K, int flags,
                                cudaStream_t stream, unsigned long long *amax = nullptr,
                                const MmvqOpts *tp = nullptr);

// Sets the kernel attributes a later launch of this candidate needs (done
// outside stream capture).
cudaError_t prepare_mmvq(const MmvqConfig &cfg, int ncols, int nmat, bool xin = false);

// Debug: same kernel, additionally storing the exact int32 partials
// P[c][r][b][s] and M[c][b][s].
cudaError_t launch_mmvq_q4k_partials(const void *w, const void *x_q8, float *y, int32_t *P,
                                     int32_t *M, int64_t N, int64_t K, int ncols, int ks,
                                     cudaStream_t stream);

// Batch-32 MMVQ on the tensor cores (tcgen05 kind::i8): ncols = 32 Q8_1
// columns, ks k-parts (1, 2, 4, 8) over the canonical slices; ks > 1 needs
// part = ks * 32 * N floats of scratch and adds a combine launch.
// A K-shard and tensor-parallel push for one tcgen05 MMVQ launch (off by
// default).  part >= 0: the launch holds exactly k-parts [part, part +
// nparts) of a ks-way split of a K of nsb_sl superblocks (its first
// superblock is sb_base) and writes the tree over them (the shard's subtree
// of the slice tree) to y, or pushes it (npeer > 0) to every peer_y[q] and
// counts on cta_cnt; the launch's last CTA adds 1 to each peer_cnt[q] with
// release semantics at system scope.  nparts > 1 needs the part workspace.
struct TcOpts {
    int nsb_sl = 0, sb_base = 0, part = -1, nparts = 1;
    int npeer = 0;
    float *peer_y[8] = {};
    unsigned long long *peer_cnt[8] = {};
    unsigned long long *cta_cnt = nullptr;
};
cudaError_t launch_mmvq_tc(const void *w, const void *x_q8, float *y, int64_t N, int64_t K,
                           int64_t ldy, int ks, float *part, int flags, cudaStream_t stream, const TcOpts *opt = nullptr);
// Sets the tensor-core kernels' attributes (outside stream capture).
cudaError_t prepare_mmvq_tc();

// ------------------------------------------------------------ quantize ---
cudaError_t launch_quantize_q8_1(const float *x, void *y, int64_t K, int ncols,
                                 cudaStream_t stream);
cudaError_t launch_rmsnorm_quantize_q8_1(const float *x, const float *w, float eps, void *y,
                                         float *xn_out, int64_t K, int ncols,
                                         cudaStream_t stream);

// ----------------------------------------------------------- generator ---
cudaError_t launch_gen_q4k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                           int64_t block_offset, cudaStream_t stream);
cudaError_t launch_gen_uniform_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                                   int64_t offset_index, float scale, float offset,
                                   cudaStream_t stream);

int device_sm_count();

// Launch plan of a Q4_K or Q6_K MMVQ on a GPU with `sms` SMs (0: this
// device's), for host-side checks of what the kernel will address: out =
// {grid, block, nstage, pitch, stage bytes, dynamic shared memory, row
// groups, offset of the stage ring in shared memory}.  False when no plan fits.
bool mmvq_plan_info(const MmvqConfig &cfg, int64_t N, int64_t K, int ncols, int nmat, bool xin,
                    const MmvqOpts *tp, int sms, int64_t out[8]);
bool q6k_plan_info(const MmvqConfig &cfg, int64_t N, int64_t K, int ncols, const MmvqOpts *tp,
                   int sms, int64_t out[8]);

// Dynamic shared memory an MMVQ plan may use (the 227 KiB opt-in limit less
// room for static shared memory), and the attribute that allows it, set once
// per (kernel, device).
constexpr int kMmvqMaxSmem = 227 * 1024 - 1024;
cudaError_t ensure_smem_attr_ptr(const void *fn);
// K-shard slicing of a launch (unsharded unless tp names a shard); false when
// the shard's slices do not add up to nsb superblocks.
bool mmvq_shard_of(const MmvqOpts *tp, int nsb, int &sl_nsb, int &sl_base, int &sl_shift);

// --------------------------------------------------------- Q6_K MMVQ ---
// Candidates of the Q6_K x Q8_1 MMVQ (MmvqConfig with mode 0 per-row
// copies, 1 whole-unit copies, 2 direct loads).
const MmvqConfig *q6k_candidates(int *count);
const MmvqConfig *q6k_candidate_by_id(int id);
// Default candidate for a shape.
int q6k_default_candidate(int64_t N, int64_t K, int ncols);
// y = W x for N x K Q6_K rows; amax and tp (slicing, row_offset and the L2
// prefetch regions; no push or wait) as for launch_mmvq_q4k.
cudaError_t launch_mmvq_q6k(const MmvqConfig &cfg, const void *w, const void *x_q8, float *y,
                            int64_t N, int64_t K, int ncols, int64_t ldy, int flags,
                            cudaStream_t stream, unsigned long long *amax = nullptr,
                            const MmvqOpts *tp = nullptr);
// Debug: also stores the exact int32 16-weight dots P[c][r][b][16].
cudaError_t launch_mmvq_q6k_partials(const void *w, const void *x_q8, float *y, int32_t *P,
                                     int64_t N, int64_t K, int ncols, cudaStream_t stream);
cudaError_t prepare_mmvq_q6k(const MmvqConfig &cfg, int ncols);
cudaError_t launch_gen_q6k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                           int64_t block_offset, cudaStream_t stream);

// Reads (and optionally clears) every translation unit's device error word.
cudaError_t read_error_words(unsigned *value, bool clear);

// Records msg for abra_last_error and returns code (for entry points that
// live outside api.cu).
int record_failure(int code, const char *msg);

}  // namespace abra
