// mmvq_q6k.cu -- host side of the Q6_K x Q8_1 MMVQ: candidate table, launch
// planning (grid, ring depth, stage pitch, shared-memory layout) and dispatch
// to the per-batch-width kernel tables (mmvq_q6k_c<N>.cu; kernel in
// mmvq_q6k_impl.cuh).
#include "kernels.cuh"
#include "mmvq_q6k_impl.cuh"

namespace abra {

// id = 1000*mode' + 10*ks + ctas_per_sm (mode' = 1 per-row copies, 2 whole
// unit, 3 direct), the numbering of the Q4_K family.
static const MmvqConfig kQ6Candidates[] = {
    // id, mode, ks, ctas_per_sm, stage_kb
    {1011, Q6_ROWS, 1, 1, 200},  {1012, Q6_ROWS, 1, 2, 100},  {1021, Q6_ROWS, 2, 1, 200},
    {1022, Q6_ROWS, 2, 2, 100},  {1041, Q6_ROWS, 4, 1, 200},  {1042, Q6_ROWS, 4, 2, 100},
    {1081, Q6_ROWS, 8, 1, 200},  {1082, Q6_ROWS, 8, 2, 100},  {2011, Q6_WHOLE, 1, 1, 200},
    {2012, Q6_WHOLE, 1, 2, 100}, {3012, Q6_DIRECT, 1, 2, 0},  {3014, Q6_DIRECT, 1, 4, 0},
    {3022, Q6_DIRECT, 2, 2, 0},  {3024, Q6_DIRECT, 2, 4, 0},  {3042, Q6_DIRECT, 4, 2, 0},
    {3044, Q6_DIRECT, 4, 4, 0},  {3082, Q6_DIRECT, 8, 2, 0},  {3084, Q6_DIRECT, 8, 4, 0},
};

const MmvqConfig *q6k_candidates(int *count) {
    *count = static_cast<int>(sizeof(kQ6Candidates) / sizeof(kQ6Candidates[0]));
    return kQ6Candidates;
}

const MmvqConfig *q6k_candidate_by_id(int id) {
    int n = 0;
    const MmvqConfig *c = q6k_candidates(&n);
    for (int i = 0; i < n; ++i)
        if (c[i].id == id) return &c[i];
    return nullptr;
}

// More k-parts when there are too few row groups to fill the GPU; whole-unit
// copies once every CTA has several units.  Measured on B200 at batch 1:
// attn_v 1024 x 2560 -> 1041/1042 (2.6 us), ffn_down 2560 x 9728 -> 1021
// (10.1 us), output 151936 x 2560 -> 2011 (75 us, 4.25 TB/s).
int q6k_default_candidate(int64_t N, int64_t K, int ncols) {
    (void)ncols;
    const int64_t rg = (N + 7) / 8;
    const int64_t nsb = K / QK_K;
    if (rg < 148) return nsb >= 16 ? 1081 : 1042;
    if (rg < 4 * 148) return 1021;
    return 2011;
}

static const Q6Table *q6_table_for(int ncols) {
    switch (ncols) {
        case 1: return &q6_table_c1();
        case 2: return &q6_table_c2();
        case 3: return &q6_table_c3();
        case 4: return &q6_table_c4();
        case 5: return &q6_table_c5();
        case 6: return &q6_table_c6();
        case 7: return &q6_table_c7();
        case 8: return &q6_table_c8();
        default: return nullptr;
    }
}

static int q6_ks_index(int ks) { return ks == 1 ? 0 : ks == 2 ? 1 : ks == 4 ? 2 : ks == 8 ? 3 : -1; }

struct Q6Plan {
    int grid, block, nstage, pitch, stage_bytes, smem, rg_total;
};

// sms: the SM count to plan for (0: this device's).
static bool plan_q6(const MmvqConfig &cfg, int64_t N, int nsb, int ncols, const MmvqOpts *tp,
                    Q6Plan &pl, int sms = 0) {
    const int ks = cfg.ks;
    const bool staged = cfg.mode != Q6_DIRECT;
    if (cfg.mode == Q6_WHOLE && ks != 1) return false;
    const int nsl = 8 / ks;
    int sl_nsb, sl_base, sl_shift;
    if (!mmvq_shard_of(tp, nsb, sl_nsb, sl_base, sl_shift)) return false;
    int max_sb = 0;
    for (int j = 0; j < ks; ++j) {
        const int w = shard_slice(sl_nsb, sl_base, sl_shift, (j + 1) * nsl) -
                      shard_slice(sl_nsb, sl_base, sl_shift, j * nsl);
        max_sb = w > max_sb ? w : max_sb;
    }
    // per-row stage: the part's bytes plus up to 14 before (the copy starts
    // on the 16-byte boundary below) and 15 after; an odd number of 16-byte
    // chunks spreads the eight rows over the banks
    int pitch = align_up(max_sb * Q6K_BYTES + 30, 16);
    if (((pitch / 16) & 1) == 0) pitch += 16;
    const int stage_bytes = cfg.mode == Q6_WHOLE ? 8 * nsb * Q6K_BYTES : 8 * pitch;
    pl.pitch = pitch;
    pl.stage_bytes = stage_bytes;
    pl.rg_total = static_cast<int>((N + 7) / 8);
    if (sms <= 0) sms = device_sm_count();
    pl.grid = pl.rg_total < sms * cfg.ctas_per_sm ? pl.rg_total : sms * cfg.ctas_per_sm;
    pl.block = (ABRA_Q6_NCW + (staged ? 1 : 0)) * 32;
    // Ring depth: every unit of a CTA has its own stage, or nstage is a
    // multiple of the consumer-warp count so each stage always has the same
    // consumer (unit u is consumed by warp u % NCW), which awaits its phases
    // in order -- the rule of the Q4_K planner.
    constexpr int W = ABRA_Q6_NCW;
    int nstage = 1, units = 1;
    if (staged) {
        const int rg_per_cta = (pl.rg_total + pl.grid - 1) / pl.grid;
        units = rg_per_cta * ks;
        const int want = (cfg.stage_kb * 1024) / stage_bytes;
        nstage = want >= units ? units : (want / W > 0 ? want / W * W : (units < W ? units : W));
    }
    for (;;) {
        const Q6Layout L = q6_layout(ncols, ks, W, nsb, nstage, stage_bytes, staged);
        if (L.bytes <= kMmvqMaxSmem) {
            pl.nstage = nstage;
            pl.smem = L.bytes;
            return true;
        }
        if (!staged) return false;
        if (nstage >= units && units <= W) return false;
        const int next = (nstage - 1) / W * W;
        if (next < W) return false;
        nstage = next;
    }
}

bool q6k_plan_info(const MmvqConfig &cfg, int64_t N, int64_t K, int ncols, const MmvqOpts *tp,
                   int sms, int64_t out[8]) {
    Q6Plan pl;
    const int nsb = static_cast<int>(K / QK_K);
    if (!plan_q6(cfg, N, nsb, ncols, tp, pl, sms)) return false;
    const bool staged = cfg.mode != Q6_DIRECT;
    const Q6Layout L = q6_layout(ncols, cfg.ks, ABRA_Q6_NCW, nsb, pl.nstage, pl.stage_bytes, staged);
    const int64_t v[8] = {pl.grid, pl.block, pl.nstage, pl.pitch, staged ? pl.stage_bytes : 0,
                          pl.smem, pl.rg_total, L.off_stage};
    for (int i = 0; i < 8; ++i) out[i] = v[i];
    return true;
}

static cudaError_t launch_q6_plan(Q6Fn fn, const Q6Plan &pl, bool pdl, Q6Params prm,
                                  cudaStream_t stream) {
    cudaError_t e = ensure_smem_attr_ptr(reinterpret_cast<const void *>(fn));
    if (e != cudaSuccess) return e;
    prm.rg_total = pl.rg_total;
    prm.nstage = pl.nstage;
    prm.pitch = pl.pitch;
    prm.stage_bytes = pl.stage_bytes;
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

static bool q6_params(Q6Params &prm, const void *w, const void *x_q8, float *y, int64_t N,
                      int nsb, int64_t ldy, const MmvqOpts *tp) {
    prm.W = static_cast<const uint8_t *>(w);
    prm.X = static_cast<const uint8_t *>(x_q8);
    prm.Y = y;
    prm.N = static_cast<int>(N);
    prm.nsb = nsb;
    prm.ldy = ldy;
    prm.w_bytes = N * nsb * Q6K_BYTES;
    if (!mmvq_shard_of(tp, nsb, prm.sl_nsb, prm.sl_base, prm.sl_shift)) return false;
    prm.row_offset = tp ? tp->row_offset : 0;
    if (!tp) return true;
    for (int r = 0; r < 2; ++r) {
        if (tp->pf_bytes[r] <= 0) continue;
        if ((reinterpret_cast<uintptr_t>(tp->pf_ptr[r]) & 15) || (tp->pf_bytes[r] & 15)) return false;
        prm.pf_ptr[r] = static_cast<const uint8_t *>(tp->pf_ptr[r]);
        prm.pf_bytes[r] = tp->pf_bytes[r];
    }
    return tp->npeer == 0 && !tp->wait_cnt;  // no tensor-parallel push or wait on this path
}

cudaError_t launch_mmvq_q6k(const MmvqConfig &cfg, const void *w, const void *x_q8, float *y,
                            int64_t N, int64_t K, int ncols, int64_t ldy, int flags,
                            cudaStream_t stream, unsigned long long *amax, const MmvqOpts *tp) {
    const int nsb = static_cast<int>(K / QK_K);
    const Q6Table *t = q6_table_for(ncols);
    const int ki = q6_ks_index(cfg.ks);
    if (!t || ki < 0 || cfg.mode < 0 || cfg.mode > 2) return cudaErrorInvalidValue;
    Q6Fn fn = t->fn[cfg.mode][ki];
    if (!fn) return cudaErrorInvalidValue;
    Q6Plan pl;
    if (!plan_q6(cfg, N, nsb, ncols, tp, pl)) return cudaErrorInvalidConfiguration;
    Q6Params prm = {};
    if (!q6_params(prm, w, x_q8, y, N, nsb, ldy, tp)) return cudaErrorInvalidValue;
    prm.amax = amax;
    return launch_q6_plan(fn, pl, (flags & MMVQ_PDL) != 0, prm, stream);
}

cudaError_t launch_mmvq_q6k_partials(const void *w, const void *x_q8, float *y, int32_t *P,
                                     int64_t N, int64_t K, int ncols, cudaStream_t stream) {
    const int nsb = static_cast<int>(K / QK_K);
    const Q6Table *t = q6_table_for(ncols);
    if (!t || !t->partials) return cudaErrorInvalidValue;
    const MmvqConfig cfg = {0, Q6_ROWS, 1, 1, 200};
    Q6Plan pl;
    if (!plan_q6(cfg, N, nsb, ncols, nullptr, pl)) return cudaErrorInvalidConfiguration;
    Q6Params prm = {};
    if (!q6_params(prm, w, x_q8, y, N, nsb, N, nullptr)) return cudaErrorInvalidValue;
    prm.P = P;
    return launch_q6_plan(t->partials, pl, false, prm, stream);
}

cudaError_t prepare_mmvq_q6k(const MmvqConfig &cfg, int ncols) {
    const Q6Table *t = q6_table_for(ncols);
    const int ki = q6_ks_index(cfg.ks);
    if (!t || ki < 0 || cfg.mode < 0 || cfg.mode > 2) return cudaErrorInvalidValue;
    Q6Fn fn = t->fn[cfg.mode][ki];
    return fn ? ensure_smem_attr_ptr(reinterpret_cast<const void *>(fn)) : cudaErrorInvalidValue;
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq_q6k)
