// mmvq.cu -- host side of the Q4_K x Q8_1 MMVQ family: candidate table,
// launch planning (grid, ring depth, shared-memory layout) and dispatch to
// the per-batch-width kernel tables (mmvq_c<N>.cu; kernel in mmvq_impl.cuh).
#include <mutex>

#include "kernels.cuh"
#include "mmvq_impl.cuh"

namespace abra {

// id = 1000*mode' + 100*h + 10*ks + ctas_per_sm (mode' = 1 TMA rows, 2 TMA
// whole, 3 direct, 4 lane-mapped with ks = its rows per unit).  h = 1: the ring is sized so that the CTAs of a launch
// fill only half of each SM (96 KiB of ring at one CTA per SM, 48 KiB at
// two), leaving room for the next launch's CTAs: with programmatic dependent
// launch they start at once and stream their weights (which do not depend on
// the previous kernel) while this launch computes.
static const MmvqConfig kCandidates[] = {
    // id, mode, ks, ctas_per_sm, stage_kb
    {1011, MODE_TMA_ROWS, 1, 1, 200},  {1012, MODE_TMA_ROWS, 1, 2, 100},
    {1021, MODE_TMA_ROWS, 2, 1, 200},  {1022, MODE_TMA_ROWS, 2, 2, 100},
    {1041, MODE_TMA_ROWS, 4, 1, 200},  {1042, MODE_TMA_ROWS, 4, 2, 100},
    {1081, MODE_TMA_ROWS, 8, 1, 200},  {1082, MODE_TMA_ROWS, 8, 2, 100},
    {2011, MODE_TMA_WHOLE, 1, 1, 200}, {2012, MODE_TMA_WHOLE, 1, 2, 100},
    {3011, MODE_DIRECT, 1, 1, 0},      {3012, MODE_DIRECT, 1, 2, 0},
    {3014, MODE_DIRECT, 1, 4, 0},      {3021, MODE_DIRECT, 2, 1, 0},
    {3022, MODE_DIRECT, 2, 2, 0},      {3024, MODE_DIRECT, 2, 4, 0},
    {3041, MODE_DIRECT, 4, 1, 0},      {3042, MODE_DIRECT, 4, 2, 0},
    {3044, MODE_DIRECT, 4, 4, 0},      {3081, MODE_DIRECT, 8, 1, 0},
    {3082, MODE_DIRECT, 8, 2, 0},      {3084, MODE_DIRECT, 8, 4, 0},
    {1111, MODE_TMA_ROWS, 1, 1, 96},   {1121, MODE_TMA_ROWS, 2, 1, 96},
    {1141, MODE_TMA_ROWS, 4, 1, 96},   {1112, MODE_TMA_ROWS, 1, 2, 48},
    {2111, MODE_TMA_WHOLE, 1, 1, 96},  {2112, MODE_TMA_WHOLE, 1, 2, 48},
    // lane-mapped batch-1 kernel (mmvq_lane.cu): ks = the largest rows per unit
    {4081, MODE_LANE, 8, 1, 200},      {4082, MODE_LANE, 8, 2, 100},
    {4041, MODE_LANE, 4, 1, 200},      {4042, MODE_LANE, 4, 2, 100},
    {4021, MODE_LANE, 2, 1, 200},      {4022, MODE_LANE, 2, 2, 100},
    {4011, MODE_LANE, 1, 1, 200},
};

const MmvqConfig *mmvq_candidates(int *count) {
    *count = static_cast<int>(sizeof(kCandidates) / sizeof(kCandidates[0]));
    return kCandidates;
}
const MmvqConfig *mmvq_candidate_by_id(int id) {
    int n = 0;
    const MmvqConfig *c = mmvq_candidates(&n);
    for (int i = 0; i < n; ++i)
        if (c[i].id == id) return &c[i];
    return nullptr;
}

// Lane candidates of four or eight rows per unit win on the wide shapes,
// where whole-unit copies do best among the template's plans; those of one
// or two rows on the narrow ones, where KS=2 row copies do.
const MmvqConfig &mmvq_classic(const MmvqConfig &cfg) {
    if (cfg.mode != MODE_LANE) return cfg;
    return *mmvq_candidate_by_id(cfg.ks >= 4 ? (cfg.ctas_per_sm >= 2 ? 2012 : 2011) : 1021);
}

int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

static const MmvqTable *table_for(int ncols) {
    switch (ncols) {
        case 1: return &mmvq_table_c1();
        case 2: return &mmvq_table_c2();
        case 3: return &mmvq_table_c3();
        case 4: return &mmvq_table_c4();
        case 5: return &mmvq_table_c5();
        case 6: return &mmvq_table_c6();
        case 7: return &mmvq_table_c7();
        case 8: return &mmvq_table_c8();
        default: return nullptr;
    }
}

static int ks_index(int ks) { return ks == 1 ? 0 : ks == 2 ? 1 : ks == 4 ? 2 : ks == 8 ? 3 : -1; }

// Dynamic shared memory a plan may use: the 227 KiB opt-in limit less room
// for the kernel's static shared memory (a few bytes of argmax keys).
constexpr int kOptinSmem = 227 * 1024;
constexpr int kMaxSmem = kMmvqMaxSmem;

cudaError_t ensure_smem_attr_ptr(const void *fn) {
    // Raise the dynamic shared-memory limit once per (kernel, device).
    static std::mutex mu;
    static const void *done[1024];
    static int done_dev[1024];
    static int ndone = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < ndone; ++i)
        if (done[i] == fn && done_dev[i] == dev) return cudaSuccess;
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, fn);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kOptinSmem - static_cast<int>(fa.sharedSizeBytes));
    if (e != cudaSuccess) return e;
    // the whole unified L1/shared array as shared memory: a CTA that needs
    // less leaves room for the next launch's CTAs on the same SM (otherwise
    // the SM may be configured with just enough for one)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    if (ndone < 1024) {
        done[ndone] = fn;
        done_dev[ndone] = dev;
        ++ndone;
    }
    return cudaSuccess;
}

static cudaError_t ensure_smem_attr(MmvqFn fn) {
    return ensure_smem_attr_ptr(reinterpret_cast<const void *>(fn));
}

struct MmvqPlan {
    int grid, block, nstage, pitch, smem, rg_total;
};

// Slicing of a launch: unsharded unless tp names a K-shard.  Returns false
// when the shard's slices do not add up to nsb superblocks.
bool mmvq_shard_of(const MmvqOpts *tp, int nsb, int &sl_nsb, int &sl_base, int &sl_shift) {
    sl_nsb = nsb;
    sl_base = 0;
    int sl_cnt = 8;
    if (tp && tp->sl_nsb > 0) {
        sl_nsb = tp->sl_nsb;
        sl_base = tp->sl_base;
        sl_cnt = tp->sl_cnt;
    }
    if (sl_base < 0 || !(sl_cnt == 1 || sl_cnt == 2 || sl_cnt == 4 || sl_cnt == 8) ||
        sl_base + sl_cnt > 8)
        return false;
    sl_shift = sl_cnt == 8 ? 0 : sl_cnt == 4 ? 1 : sl_cnt == 2 ? 2 : 3;
    return shard_slice(sl_nsb, sl_base, sl_shift, 8) == nsb;
}

// sms: the SM count to plan for (0: this device's).
static bool plan_mmvq(const MmvqConfig &cfg_in, int64_t N, int nsb, int ncols, int nmat,
                      MmvqPlan &pl, bool xin = false, const MmvqOpts *tp = nullptr, int sms = 0) {
    const MmvqConfig &cfg = mmvq_classic(cfg_in);
    const int ks = cfg.ks;
    const bool staged = cfg.mode != MODE_DIRECT;
    const int nsl = 8 / ks;
    int sl_nsb, sl_base, sl_shift;
    if (!mmvq_shard_of(tp, nsb, sl_nsb, sl_base, sl_shift)) return false;
    int max_sb = 0;
    for (int j = 0; j < ks; ++j) {
        const int w = shard_slice(sl_nsb, sl_base, sl_shift, (j + 1) * nsl) -
                      shard_slice(sl_nsb, sl_base, sl_shift, j * nsl);
        max_sb = w > max_sb ? w : max_sb;
    }
    const int max_part = max_sb * Q4K_BYTES;
    int pitch = max_part;
    if (cfg.mode == MODE_TMA_ROWS && ((pitch / 16) & 1) == 0) pitch += 16;
    pl.pitch = pitch;
    pl.rg_total = static_cast<int>((N + 7) / 8);
    if (sms <= 0) sms = device_sm_count();
    pl.grid = pl.rg_total < sms * cfg.ctas_per_sm ? pl.rg_total : sms * cfg.ctas_per_sm;
    pl.block = (ABRA_MMVQ_NCW + (staged ? 1 : 0)) * 32;
    // Ring depth.  Unit u is consumed by warp u % NCW and lands in stage
    // u % nstage; a parity wait is only sound if its waiter cannot run a phase
    // ahead of the barrier (try_wait.parity on a phase that has not begun
    // reports the previous phase, which is complete).  So either every unit of
    // a CTA gets its own stage (no reuse), or nstage is a multiple of NCW and
    // each stage always has the same consumer, which awaits its phases in order.
    constexpr int W = ABRA_MMVQ_NCW;
    int nstage = 1;
    int units = 1;
    if (staged) {
        const int rg_per_cta = (pl.rg_total + pl.grid - 1) / pl.grid;
        units = rg_per_cta * ks;
        const int stage_bytes = 8 * nmat * pitch;
        const int want = (cfg.stage_kb * 1024) / stage_bytes;
        nstage = want >= units ? units : (want / W > 0 ? want / W * W : (units < W ? units : W));
    }
    for (;;) {
        const MmvqLayout L = mmvq_layout(ncols, ks, W, nsb, nstage, pitch, nmat, staged, xin);
        if (L.bytes <= kMaxSmem) {
            pl.nstage = nstage;
            pl.smem = L.bytes;
            return true;
        }
        if (!staged) return false;
        // shrink to the next depth that keeps the rule above
        if (nstage >= units && units <= W) return false;
        const int next = (nstage - 1) / W * W;
        if (next < W) return false;
        nstage = next;
    }
}

// Copies the tensor-parallel options into the kernel parameters.
static bool apply_tp(MmvqParams &prm, const MmvqOpts *tp) {
    if (!mmvq_shard_of(tp, prm.nsb, prm.sl_nsb, prm.sl_base, prm.sl_shift)) return false;
    if (!tp) return true;
    if (tp->npeer < 0 || tp->npeer > 8) return false;
    prm.row_offset = tp->row_offset;
    prm.npeer = tp->npeer;
    for (int q = 0; q < tp->npeer; ++q) {
        if (!tp->peer_cnt[q]) return false;
        prm.peer_y[q] = tp->peer_y[q];
        prm.peer_amax[q] = tp->peer_amax[q];
        prm.peer_cnt[q] = tp->peer_cnt[q];
    }
    if (tp->npeer > 0 && !tp->cta_cnt) return false;
    prm.cta_cnt = tp->cta_cnt;
    prm.wait_cnt = tp->wait_cnt;
    prm.epoch = tp->epoch;
    prm.wait_per_step = tp->wait_per_step;
    for (int r = 0; r < 2; ++r) {
        if (tp->pf_bytes[r] <= 0) continue;
        if ((reinterpret_cast<uintptr_t>(tp->pf_ptr[r]) & 15) || (tp->pf_bytes[r] & 15)) return false;
        prm.pf_ptr[r] = static_cast<const uint8_t *>(tp->pf_ptr[r]);
        prm.pf_bytes[r] = tp->pf_bytes[r];
    }
    return !prm.wait_cnt || prm.epoch;
}

static cudaError_t launch_plan(MmvqFn fn, const MmvqPlan &pl, bool pdl, MmvqParams prm,
                               cudaStream_t stream) {
    cudaError_t e = ensure_smem_attr(fn);
    if (e != cudaSuccess) return e;
    prm.rg_total = pl.rg_total;
    prm.nstage = pl.nstage;
    prm.pitch = pl.pitch;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(pl.block);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, prm);
}

cudaError_t launch_mmvq_q4k(const MmvqConfig &cfg_in, const void *w, const void *w2,
                            const void *x_q8, float *y, int64_t N, int64_t K, int ncols,
                            int64_t ldy, int flags, cudaStream_t stream,
                            unsigned long long *amax, const MmvqOpts *tp) {
    if (cfg_in.mode == MODE_LANE && ncols == 1 && !tp)
        return launch_mmvq_lane(cfg_in, w, w2, x_q8, y, N, K, flags, stream, amax);
    const MmvqConfig &cfg = mmvq_classic(cfg_in);
    const int nsb = static_cast<int>(K / QK_K);
    const int nmat = w2 ? 2 : 1;
    const MmvqTable *t = table_for(ncols);
    const int ki = ks_index(cfg.ks);
    if (!t || ki < 0 || cfg.mode < 0 || cfg.mode > MODE_DIRECT) return cudaErrorInvalidValue;
    MmvqFn fn = t->fn[cfg.mode][ki][nmat - 1];
    if (!fn) return cudaErrorInvalidValue;
    MmvqPlan pl;
    if (!plan_mmvq(cfg, N, nsb, ncols, nmat, pl, false, tp)) return cudaErrorInvalidConfiguration;
    MmvqParams prm = {};
    prm.W[0] = static_cast<const uint8_t *>(w);
    prm.W[1] = static_cast<const uint8_t *>(w2);
    prm.X = static_cast<const uint8_t *>(x_q8);
    prm.Y = y;
    prm.N = static_cast<int>(N);
    prm.nsb = nsb;
    prm.ldy = ldy;
    prm.amax = amax;
    if (!apply_tp(prm, tp)) return cudaErrorInvalidValue;
    return launch_plan(fn, pl, (flags & MMVQ_PDL) != 0, prm, stream);
}

int mmvq_grid(const MmvqConfig &cfg, int64_t N, int64_t K, int ncols, int nmat, bool xin,
              const MmvqOpts *tp) {
    if (cfg.mode == MODE_LANE && ncols == 1 && !xin && !tp) {
        int64_t lp[8];
        return mmvq_lane_plan(cfg, N, static_cast<int>(K / QK_K), nmat, 0, lp) ? static_cast<int>(lp[0]) : -1;
    }
    MmvqPlan pl;
    if (!plan_mmvq(cfg, N, static_cast<int>(K / QK_K), ncols, nmat, pl, xin, tp)) return -1;
    return pl.grid;
}

bool mmvq_plan_info(const MmvqConfig &cfg_in, int64_t N, int64_t K, int ncols, int nmat, bool xin,
                    const MmvqOpts *tp, int sms, int64_t out[8]) {
    MmvqPlan pl;
    const int nsb = static_cast<int>(K / QK_K);
    if (cfg_in.mode == MODE_LANE && ncols == 1 && !xin && !tp) {
        // {grid, block, ring slots, row pitch, slot bytes, shared memory, units, ring offset}
        int64_t lp[8];
        if (!mmvq_lane_plan(cfg_in, N, nsb, nmat, sms, lp)) return false;
        const int64_t R = int64_t(1) << lp[5];
        const int64_t v[8] = {lp[0], lp[1], lp[2], int64_t(nsb) * Q4K_BYTES, lp[3], lp[4], (N + R - 1) / R, lp[7]};
        for (int i = 0; i < 8; ++i) out[i] = v[i];
        return true;
    }
    const MmvqConfig &cfg = mmvq_classic(cfg_in);
    if (!plan_mmvq(cfg, N, nsb, ncols, nmat, pl, xin, tp, sms)) return false;
    const bool staged = cfg.mode != MODE_DIRECT;
    const MmvqLayout L = mmvq_layout(ncols, cfg.ks, ABRA_MMVQ_NCW, nsb, pl.nstage, pl.pitch, nmat,
                                     staged, xin);
    const int64_t v[8] = {pl.grid, pl.block, pl.nstage, pl.pitch, staged ? 8 * nmat * pl.pitch : 0,
                          pl.smem, pl.rg_total, L.off_stage};
    for (int i = 0; i < 8; ++i) out[i] = v[i];
    return true;
}

cudaError_t launch_mmvq_q4k_xin(const MmvqConfig &cfg_in, const void *w, const void *w2,
                                const MmvqXin &xin, float *y, int64_t N, int64_t K, int flags,
                                cudaStream_t stream, unsigned long long *amax, const MmvqOpts *tp) {
    const MmvqConfig &cfg = mmvq_classic(cfg_in);
    const int nsb = static_cast<int>(K / QK_K);
    const int nmat = w2 ? 2 : 1;
    const int ki = ks_index(cfg.ks);
    if (ki < 0 || cfg.mode < 0 || cfg.mode > MODE_DIRECT) return cudaErrorInvalidValue;
    MmvqFn fn = mmvq_table_c1().xin[cfg.mode][ki][nmat - 1];
    if (!fn || !xin.h_in || !xin.norm_w) return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(xin.norm_w) & 15) return cudaErrorInvalidValue;  // float4 loads
    if (reinterpret_cast<uintptr_t>(xin.x_out) & 3) return cudaErrorInvalidValue;
    MmvqPlan pl;
    if (!plan_mmvq(cfg, N, nsb, 1, nmat, pl, true, tp)) return cudaErrorInvalidConfiguration;
    MmvqParams prm = {};
    prm.W[0] = static_cast<const uint8_t *>(w);
    prm.W[1] = static_cast<const uint8_t *>(w2);
    prm.Y = y;
    prm.N = static_cast<int>(N);
    prm.nsb = nsb;
    prm.ldy = N;
    prm.amax = amax;
    prm.h_in = xin.h_in;
    prm.h_out = xin.h_out;
    prm.deltas = xin.deltas;
    prm.norm_w = xin.norm_w;
    prm.eps = xin.eps;
    prm.x_out = xin.x_out;
    if (!apply_tp(prm, tp)) return cudaErrorInvalidValue;
    return launch_plan(fn, pl, (flags & MMVQ_PDL) != 0, prm, stream);
}

cudaError_t prepare_mmvq(const MmvqConfig &cfg, int ncols, int nmat, bool xin) {
    if (cfg.mode == MODE_LANE) {
        if (ncols == 1 && !xin) {
            cudaError_t e = prepare_mmvq_lane(cfg, nmat);
            if (e != cudaSuccess) return e;
        }
        return prepare_mmvq(mmvq_classic(cfg), ncols, nmat, xin);  // the plan it stands for elsewhere
    }
    if (cfg.mode < 0 || cfg.mode > MODE_DIRECT) return cudaErrorInvalidValue;
    const MmvqTable *t = table_for(ncols);
    const int ki = ks_index(cfg.ks);
    if (!t || ki < 0 || nmat < 1 || nmat > 2) return cudaErrorInvalidValue;
    MmvqFn fn = xin ? t->xin[cfg.mode][ki][nmat - 1] : t->fn[cfg.mode][ki][nmat - 1];
    return fn ? ensure_smem_attr(fn) : cudaErrorInvalidValue;
}

cudaError_t launch_mmvq_q4k_partials(const void *w, const void *x_q8, float *y, int32_t *P,
                                     int32_t *M, int64_t N, int64_t K, int ncols, int ks,
                                     cudaStream_t stream) {
    const int nsb = static_cast<int>(K / QK_K);
    const MmvqTable *t = table_for(ncols);
    const int ki = ks_index(ks);
    if (!t || ki < 0 || ki > 2 || !t->partials[ki]) return cudaErrorInvalidValue;
    const MmvqConfig cfg = {0, MODE_TMA_ROWS, ks, 1, 200};
    MmvqPlan pl;
    if (!plan_mmvq(cfg, N, nsb, ncols, 1, pl)) return cudaErrorInvalidConfiguration;
    MmvqParams prm = {};
    prm.W[0] = static_cast<const uint8_t *>(w);
    prm.X = static_cast<const uint8_t *>(x_q8);
    prm.Y = y;
    prm.N = static_cast<int>(N);
    prm.nsb = nsb;
    prm.ldy = N;
    prm.P = P;
    prm.M = M;
    if (!apply_tp(prm, nullptr)) return cudaErrorInvalidValue;
    return launch_plan(t->partials[ki], pl, false, prm, stream);
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq)
