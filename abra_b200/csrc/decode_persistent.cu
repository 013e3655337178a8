// decode_persistent.cu -- one decode token of the batch-1 Q4_K model as ONE
// cooperative kernel: one CTA per SM, eight warps each.
//
// The kernel-chain step (model.cu, record_step) is ~290 dependent launches
// per token, each paying launch, ramp and drain.  Here the token is a
// sequence of phases separated by grid-wide barriers, and the weights of
// every GEMV phase stream into a shared-memory ring AHEAD of the data
// dependency: weights do not depend on activations, so each CTA's ring
// always holds the next NSLOT units of its whole token's share of the weight
// rows -- layer by layer, phase by phase: the warp that finishes a slot
// refills it with the unit NSLOT tickets ahead.  While the warps work through
// attention or wait at a barrier, the copies already issued keep HBM
// streaming the next phases' rows.
//
// Phases of layer l (a grid barrier after each):
//   QKV   residual add + RMSNorm + Q8_1 in every CTA's shared memory (layer 0:
//         the token's embedding row dequantized in place), then the fused
//         q|k|v MMVQ -> qkv
//   ATT   per (q heads, 256-position chunk c) item -- a kv group's heads, or
//         one q head while the context is short: QK-RMSNorm + NEOX RoPE of
//         the item's q heads; on the chunk holding the current position also
//         the group's k/v heads (appended to the fp16 cache by the group's
//         first item); the chunk's softmax partials; one chunk: the CTA merges
//         its heads itself; more: the last chunk of the item's heads to
//         finish (arrival counter) merges them -> oq (Q8_1)
//   O     MMVQ of oq -> delta
//   GU    residual add + RMSNorm + Q8_1, fused gate/up SwiGLU MMVQ -> act
//   DOWN  Q8_1 of act in every CTA's shared memory, MMVQ -> delta
// then OUT: residual add + RMSNorm + Q8_1, the tied output MMVQ with the
// argmax keys; the last CTA to arrive appends the greedy pick and advances
// the position.
//
// Every value is computed by the same arithmetic, in the same order, as the
// kernel chain (mmvq_impl.cuh, decode_kernels.cu, gen_quant.cu) and so as the
// CPU oracle (oracle/model_oracle.c): logits and tokens are bit-identical to
// both.  Data written inside the launch is read through L2 (ld.global.cg) or
// from this CTA's shared memory, never through the non-coherent path.
//
// GEMV units: a unit is R consecutive rows (R = 8, 4, 2 or 1 per phase, so
// that a unit fits one ring slot), staged by ONE bulk copy per matrix (the
// rows are contiguous in HBM; many small copies cap an SM's copy rate); the
// lane owning (row r, superblock p) of the consuming warp computes
// superblocks p, p + 32/R, ... of row r, each whole superblock value in
// registers (the eight exact int32 sub-block dots by dp4a and the canonical
// fp32 tree); lanes 0 .. R-1 then sum one row each over the eight canonical
// K-slices.
//
// Ring protocol: ticket t of a CTA (its t-th unit over the token) goes to
// slot t % NSLOT (16 slots, or 8 when the activations of a wide or many-head
// shape leave less shared memory), phase t / NSLOT of that slot's full
// mbarrier; the warp that consumed ticket t - NSLOT issued t.  Within a GEMV
// phase unit u goes to warp u % 8 (NSLOT is a multiple of 8, so ticket
// t - NSLOT of the same phase belongs to the same warp, which consumed it
// before waiting on t; across phases all warps pass a CTA barrier) -- so no
// parity wait can alias a phase two ahead.
//
// Every wait is bounded (1 s of %globaltimer): a grid barrier that gives up
// sets ERR_GRID_TIMEOUT in the device error word, later barriers of the
// launch then pass at once, and named CTA barriers are never skipped, so the
// kernel always ends.  Every ticket issued is consumed (waited for) before
// the CTA exits, so no copy is in flight at exit.  No copy uses cluster
// multicast.
#include <algorithm>
#include <cmath>
#include <vector>

#include "common.cuh"
#include "decode.cuh"
#include "kernels.cuh"
#include "mmvq_impl.cuh"
#include "quant_common.cuh"
#include "lane_gemv.cuh"

namespace abra {

namespace {

constexpr int ATT_CHUNK_P = 256;              // attention positions per chunk (as the kernel chain)
constexpr int PK_NCW = 8;                      // warps: the canonical 256 lanes
constexpr int PK_THREADS = PK_NCW * 32;        // every warp consumes and refills the ring
constexpr int PK_NSLOT = 16;                   // ring slots (8 when shared memory is short)
// One ring slot: 8 rows x 10 superblocks at an odd pitch of 16-byte chunks
// (eight rows of a 2560-wide Q4_K matrix); every phase picks its rows per
// unit so that a unit fits.
constexpr int PK_SLOT_BYTES = 8 * 1456;
static_assert(PK_NSLOT % PK_NCW == 0 && PK_NSLOT / 2 == PK_NCW, "slots: 16 or 8, multiples of the warps");
// Activation record of one superblock in shared memory (lane_gemv.cuh).
constexpr int PK_AREC = LG_AREC;
// Per-warp staging of the superblock values of one unit (rows x superblocks
// x matrices <= 80: a unit fits an 11,648-byte slot).
constexpr int PK_VMAX = 80;

// GEMV kinds (index of the per-phase plan) and consumer phases.
enum : int { PK_QKV = 0, PK_O = 1, PK_GU = 2, PK_DOWN = 3, PK_OUT = 4, PK_KINDS = 5 };
enum : int { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_OUT = 5 };

struct PkParams {
    const PersistLayer *layers;  // device array, n_layers entries
    const uint8_t *embd;
    const float *out_norm;
    int n_layers, hidden, n_heads, n_kv, ffn, vocab, max_ctx, max_chunks;
    float eps, scale;
    float *h[2];
    float *delta, *qkv, *att, *part_m, *part_l, *part_o, *act, *logits;
    uint8_t *oq;
    __half *kc, *vc;
    const float *rope;
    int32_t *tokens, *picks, *pos;
    const int32_t *nprompt;
    unsigned long long *amax;
    unsigned long long *bar, *gen;  // grid barrier arrivals, launches completed
    unsigned *head_cnt;             // merge arrivals per attention item's first q head
    int lr[PK_KINDS], pitch[PK_KINDS];  // log2 rows per unit and staged row pitch per GEMV kind
    int slot_shift;                     // log2 of the ring slots (4: 16 slots, 3: 8)
    int off_vbuf, off_arec, off_x, off_ring, smem;  // dynamic shared memory layout
};

#ifdef ABRA_PK_TRACE
// Diagnostic build only: %globaltimer stamps of each CTA's phase starts,
// ends and end of inputs.
constexpr int PK_TRACE_EV = 512;
__device__ unsigned long long g_pk_trace[160][5][PK_TRACE_EV];
__shared__ unsigned long long g_pk_wait_ns;  // this CTA's warps' waits on ring slots, per phase
__device__ unsigned long long g_pk_att[12];         // CTA 0 thread 0: steps of layer 1's first attention item
#define PK_ASTAMP(layer, k)                                                   \
    do {                                                                      \
        if (blockIdx.x == 0 && threadIdx.x == 0 && (layer) == 1 && it == 0)   \
            g_pk_att[k] = globaltimer_ns();                                   \
    } while (0)
#define PK_STAMP(kind, idx)                                                                            \
    do {                                                                                               \
        if ((idx) < PK_TRACE_EV && blockIdx.x < 160) g_pk_trace[blockIdx.x][kind][idx] = globaltimer_ns(); \
    } while (0)
#else
#define PK_ASTAMP(layer, k) \
    do {                    \
    } while (0)
#define PK_STAMP(kind, idx) \
    do {                    \
    } while (0)
#endif

// ------------------------------------------------------------ helpers ---
__device__ __forceinline__ bool pk_aborted() {
    return (*static_cast<volatile unsigned *>(&g_abra_device_error) & ERR_GRID_TIMEOUT) != 0;
}
// Thread 0 of a CTA whose consumers have passed a CTA barrier after their
// last writes of the phase: publish the CTA's arrival with one release add at
// GPU scope (cumulative: it orders every write the CTA barrier made visible
// to this thread).  A separate fence.acq_rel before a relaxed add, the same
// ordering, measured 6 % slower over the token's 181 barriers.
__device__ __forceinline__ void pk_arrive(unsigned long long *bar) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(bar), "l"(1ull) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void cta_sync() { named_bar_sync(1, PK_NCW * 32); }

// Thread 0: wait until every CTA has arrived, polling with acquire loads (the
// load that sees the last arrival orders this CTA's later reads after every
// CTA's released writes; the CTA barrier that follows passes that on).
// Bounded; after one timeout in this launch the remaining barriers pass at
// once.
__device__ __forceinline__ void pk_wait(const unsigned long long *bar, unsigned long long target) {
    if (ld_acquire_gpu(bar) >= target || pk_aborted()) return;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (ld_acquire_gpu(bar) >= target) return;
        if ((i & 63u) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
            report_error(ERR_GRID_TIMEOUT);
            return;
        }
    }
}

struct PkMm {
    const uint8_t *w0, *w1;
    int N, nsb, lr, pitch;
};

// The weight matrix (or gate/up pair) of GEMV `kind` of `layer`.
__device__ __forceinline__ PkMm pk_mm(const PkParams &P, int layer, int kind) {
    PkMm mm;
    mm.w1 = nullptr;
    mm.lr = P.lr[kind];
    mm.pitch = P.pitch[kind];
    const int nsb_h = P.hidden / QK_K;
    if (kind == PK_OUT) {
        mm.w0 = P.embd;
        mm.N = P.vocab;
        mm.nsb = nsb_h;
        return mm;
    }
    const PersistLayer &L = P.layers[layer];
    if (kind == PK_QKV) {
        mm.w0 = L.wqkv;
        mm.N = (P.n_heads + 2 * P.n_kv) * 128;
        mm.nsb = nsb_h;
    } else if (kind == PK_O) {
        mm.w0 = L.wo;
        mm.N = P.hidden;
        mm.nsb = P.n_heads * 128 / QK_K;
    } else if (kind == PK_GU) {
        mm.w0 = L.wgate;
        mm.w1 = L.wup;
        mm.N = P.ffn;
        mm.nsb = nsb_h;
    } else {
        mm.w0 = L.wdown;
        mm.N = P.hidden;
        mm.nsb = P.ffn / QK_K;
    }
    return mm;
}

// This CTA's contiguous share [u_begin, u_begin + nu) of the GEMV's units.
__device__ __forceinline__ void pk_range(const PkMm &mm, int &u_begin, int &nu) {
    const int total = (mm.N + (1 << mm.lr) - 1) >> mm.lr;
    u_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * total / gridDim.x);
    nu = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * total / gridDim.x) - u_begin;
}

// ------------------------------------------------------ weight stream ---
// There is no producer warp: the warp that finishes with ring slot s
// (ticket t) refills it with ticket t + NSLOT, and the CTA's first NSLOT
// tickets are issued at launch.  A producer warp refilled a slot as soon as it
// was released and was otherwise blocked NSLOT tickets ahead, so the stream's
// timing is the same; what changes is the warp count: eight warps put two on
// each SM sub-partition (a ninth put three on one, whose 16K registers then
// capped every thread at 168 and spilled).
//
// Ticket map of a CTA: its unit count and first unit per GEMV kind (the same
// in every layer), the units of one layer, the token's total.
struct PkTickets {
    int nu[PK_KINDS], ub[PK_KINDS];
    int per_layer;
    uint32_t total;
};
// For CTA b of G, rows N[kind] in units of 2^lr[kind] rows (pk_range's split).
__host__ __device__ __forceinline__ void pk_tickets_for(const int (&N)[PK_KINDS], const int (&lr)[PK_KINDS],
                                                        int n_layers, int b, int G, PkTickets &k) {
    k.per_layer = 0;
    for (int kind = 0; kind < PK_KINDS; ++kind) {
        const int total = (N[kind] + (1 << lr[kind]) - 1) >> lr[kind];
        k.ub[kind] = static_cast<int>(static_cast<int64_t>(b) * total / G);
        k.nu[kind] = static_cast<int>(static_cast<int64_t>(b + 1) * total / G) - k.ub[kind];
        if (kind < PK_OUT) k.per_layer += k.nu[kind];
    }
    k.total = static_cast<uint32_t>(n_layers) * static_cast<uint32_t>(k.per_layer) + static_cast<uint32_t>(k.nu[PK_OUT]);
}
__device__ __forceinline__ void pk_tickets(const PkParams &P, PkTickets &k) {
    const int N[PK_KINDS] = {(P.n_heads + 2 * P.n_kv) * 128, P.hidden, P.ffn, P.hidden, P.vocab};
    const int lr[PK_KINDS] = {P.lr[0], P.lr[1], P.lr[2], P.lr[3], P.lr[4]};
    pk_tickets_for(N, lr, P.n_layers, blockIdx.x, gridDim.x, k);
}

// Position of a ticket in the token: GEMV kind, layer (P.n_layers for the
// output) and unit within the CTA's share.
struct PkTicketPos {
    int kind, layer, u;
};
// The position `ahead` tickets after `at` (walks forward over the phases).
__host__ __device__ __forceinline__ PkTicketPos pk_ticket_ahead(const PkTickets &k, int n_layers, PkTicketPos at, int ahead) {
    int rem = at.u + ahead;
    while (at.kind != PK_OUT && rem >= k.nu[at.kind]) {
        rem -= k.nu[at.kind];
        if (at.kind < PK_DOWN) {
            ++at.kind;
        } else if (at.layer + 1 < n_layers) {
            ++at.layer;
            at.kind = PK_QKV;
        } else {
            at.layer = n_layers;
            at.kind = PK_OUT;
        }
    }
    at.u = rem;  // past nu[PK_OUT]: beyond the token
    return at;
}

// One lane: the rows of the unit at `pos` into ring slot s (one bulk copy per
// matrix), the slot's full barrier expecting their bytes.
__device__ __forceinline__ void pk_issue_mm(const PkMm &mm, const PkTickets &k, PkTicketPos pos, int s, uint8_t *ring,
                                            uint64_t *full, uint64_t pol) {
    const int nmat = mm.w1 ? 2 : 1, R = 1 << mm.lr;
    const uint32_t row_bytes = static_cast<uint32_t>(mm.nsb) * Q4K_BYTES;
    const int row0 = (k.ub[pos.kind] + pos.u) * R, nvalid = min(R, mm.N - row0);
    const uint32_t bytes = static_cast<uint32_t>(nvalid) * row_bytes;
    mbar_arrive_expect_tx(&full[s], nmat * bytes);
    for (int m = 0; m < nmat; ++m)
        bulk_g2s(ring + s * PK_SLOT_BYTES + m * R * row_bytes, (m ? mm.w1 : mm.w0) + static_cast<int64_t>(row0) * row_bytes,
                 bytes, &full[s], pol);
}
__device__ __forceinline__ void pk_issue(const PkParams &P, const PkTickets &k, PkTicketPos pos, int s, uint8_t *ring,
                                         uint64_t *full, uint64_t pol) {
    pk_issue_mm(pk_mm(P, pos.kind == PK_OUT ? 0 : pos.layer, pos.kind), k, pos, s, ring, full, pol);
}

// The CTA's q|k|v rows of layer 0 -- where the next token starts -- into L2
// (one lane; asynchronous).
__device__ __forceinline__ void pk_prefetch_next(const PkParams &P, const PkTickets &k) {
    if (P.n_layers <= 0) return;
    const PkMm mm = pk_mm(P, 0, PK_QKV);
    const int64_t row_bytes = static_cast<int64_t>(mm.nsb) * Q4K_BYTES;
    const int64_t row0 = static_cast<int64_t>(k.ub[PK_QKV]) << mm.lr;
    const int64_t rows = min(static_cast<int64_t>(k.nu[PK_QKV]) << mm.lr, static_cast<int64_t>(mm.N) - row0);
    const uint8_t *base = mm.w0 + row0 * row_bytes;
    const int64_t bytes = rows > 0 ? rows * row_bytes : 0;  // a multiple of 16 (144 per block)
    constexpr int64_t PIECE = 16384;
    for (int64_t o = 0; o < bytes; o += PIECE) prefetch_l2_bulk(base + o, static_cast<uint32_t>(min(PIECE, bytes - o)));
}

// --------------------------------------------------- consumer: GEMV units ---
// The units of one GEMV phase that belong to this warp (unit u of the CTA's
// range -> warp u % 8, ring slot (T + u) % NSLOT).  The superblock values
// meet in this warp's staging buffer; eight lanes per row form the canonical
// K-slice sums and their fixed tree; the row's first lane stores y (and
// merges the argmax key).
template <int NMAT>
__device__ __forceinline__ void pk_units(const PkParams &P, const PkTickets &tk, PkTicketPos at, uint64_t pol,
                                         const PkMm &mm, int u_begin, int nu, uint32_t T, uint8_t *ring,
                                         uint64_t *full, float *vbuf, const uint8_t *arec,
                                         float *Y, unsigned long long *s_amax, int sh, bool &poisoned) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lr = mm.lr, R = 1 << lr, LP = 32 >> lr;  // LP lanes per row
    // lane -> (row r, first superblock p); rows are staged back to back
    // (pitch nsb * 144 B = 9 nsb chunks of 16 B), so the chunk of (r, b) is
    // 9 nsb r + 9 b + c == (nsb r + b) mod 8 bank groups.  LP >= 8: a
    // quarter warp is one row and eight consecutive superblocks (distinct);
    // LP == 4 (eight rows): a quarter warp is four rows x two superblocks,
    // distinct for nsb == 2 mod 8 (the 2560-wide matrices)
    int r, p;
    if (LP >= 8) {
        r = lane / LP;
        p = lane % LP;
    } else {
        const int q4 = lane >> 3, w8 = lane & 7;
        r = (w8 >> 1) + 4 * (q4 & 1);
        p = (w8 & 1) + 2 * (q4 >> 1);
    }
    const int nsb = mm.nsb, N = mm.N;
    const uint32_t smask = (1u << sh) - 1u;
    for (int u = warp; u < nu; u += PK_NCW) {
        const uint32_t t = T + static_cast<uint32_t>(u);
        const int s = static_cast<int>(t & smask);
#ifdef ABRA_PK_TRACE
        const uint64_t tw0 = globaltimer_ns();
#endif
        // the ticket this slot is refilled with and its weight pointers (read
        // from the layer table in global memory), fetched now so that the
        // load overlaps this unit's superblocks
        const bool refill = t + (1u << sh) < tk.total;
        PkTicketPos nx = at;
        PkMm nmm = mm;
        if (refill) {
            at.u = u;
            nx = pk_ticket_ahead(tk, P.n_layers, at, 1 << sh);
            nmm = pk_mm(P, nx.kind == PK_OUT ? 0 : nx.layer, nx.kind);
        }
        if (!poisoned && !mbar_wait(&full[s], (t >> sh) & 1)) poisoned = true;
#ifdef ABRA_PK_TRACE
        if (lane == 0) atomicAdd(&g_pk_wait_ns, static_cast<unsigned long long>(globaltimer_ns() - tw0));
#endif
        const uint8_t *wrow[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) wrow[m] = ring + s * PK_SLOT_BYTES + (m * R + r) * mm.pitch;
        for (int b = p; b < nsb; b += LP) {
            const uint8_t *wsb[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) wsb[m] = wrow[m] + b * Q4K_BYTES;
            float v[NMAT];
            pk_sb_value<NMAT>(wsb, arec + b * PK_AREC, v);
#pragma unroll
            for (int m = 0; m < NMAT; ++m) vbuf[(m * R + r) * nsb + b] = v[m];
        }
        __syncwarp();
        // the slot's weights are consumed: lane 31 refills it with the ticket
        // NSLOT ahead (ordered after the lanes' reads of the slot: the warp
        // barrier, then a proxy fence before the asynchronous copy)
        if (lane == 31 && refill) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            pk_issue_mm(nmm, tk, nx, s, ring, full, pol);
        }
        // row sums: lane 8g + i forms slice i of rows g, g + 4 of the unit,
        // the slice tree runs across the group's eight lanes, lane 8g stores
        const int i = lane & 7, g = lane >> 3;
        unsigned long long key = 0ull;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int rr = g + 4 * half;
            if (half == 1 && R <= 4) break;  // warp-uniform
            const int row = ((u_begin + u) << lr) + rr;
            const bool live = rr < R;
            float yv = pk_slice_tree(live ? pk_slice_sum(vbuf + rr * nsb, nsb, i) : 0.0f);
            if constexpr (NMAT == 2) {
                const float up = pk_slice_tree(live ? pk_slice_sum(vbuf + (R + rr) * nsb, nsb, i) : 0.0f);
                yv = __fmul_rn(up, abra_silu(yv));
            }
            if (i == 0 && live && row < N) {
                Y[row] = yv;
                const unsigned long long k = argmax_key(yv, row);
                key = k > key ? k : key;
            }
        }
        __syncwarp();
        if (s_amax) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                key = k2 > key ? k2 : key;
            }
            if (lane == 0) atomicMax(s_amax, key);
        }
        __syncwarp();  // the staging buffer is reused by the next unit
    }
}

// --------------------------------------- consumer: activation prologues ---
// Immutable RMSNorm weights into shared memory (done before the barrier that
// releases the phase).
__device__ __forceinline__ void pk_stage_norm(const float *w, float *s_w, int K) {
    for (int i = threadIdx.x * 4; i < K; i += PK_NCW * 32 * 4)
        *reinterpret_cast<float4 *>(s_w + i) = __ldg(reinterpret_cast<const float4 *>(w + i));
}

// 16 bytes from global memory (through L2, not L1) into shared memory without
// passing through registers; complete for this thread after cp_async_wait,
// for the CTA after a CTA barrier that follows it.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                 "l"(static_cast<uint64_t>(__cvta_generic_to_global(src)))
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// The next residual prologue's inputs -- its RMSNorm weights and the residual
// stream h (written before the last grid barrier this CTA passed) -- copied
// into shared memory in the background while this CTA works on or waits for
// other phases; the prologue waits for them.  Issued as early as the data is
// stable and s_x / s_w are free, so that a CTA arriving last at a barrier
// does not start its loads only then.  Warp 0 issues none: its thread 0
// arrives at and polls the grid barriers, and its fences would otherwise wait
// for these copies to land.
__device__ __forceinline__ void pk_stage_xin_async(const float *w, const float *h, float *s_w, float *s_x, int K) {
    if (threadIdx.x < 32) return;
    for (int i = (threadIdx.x - 32) * 4; i < K; i += (PK_NCW - 1) * 32 * 4) {
        cp_async16(s_w + i, w + i);
        cp_async16(s_x + i, h + i);
    }
}

// Element i of the token's embedding row (embed_kernel's arithmetic).
__device__ __forceinline__ float pk_embed(const uint8_t *row, int i) {
    const int b = i >> 8, r = i & 255, p = r >> 6, hh = (r >> 5) & 1, l = r & 31;
    const uint8_t *blk = row + b * Q4K_BYTES;
    const float d = __half2float(*reinterpret_cast<const __half *>(blk));
    const float dmin = __half2float(*reinterpret_cast<const __half *>(blk + 2));
    int sc, m;
    scale_min_one(blk + 4, 2 * p + hh, sc, m);
    const int byte = blk[16 + 32 * p + l];
    const int q = hh ? (byte >> 4) : (byte & 15);
    const float a = __fmul_rn(d, static_cast<float>(sc));
    const float bm = __fmul_rn(dmin, static_cast<float>(m));
    return __fmaf_rn(a, static_cast<float>(q), -bm);
}

// The reference Q8_1 rounding of one 32-value block (d = amax / 127,
// q = roundf(x / d), the block's integer sum; the bytes quantize_q8_1_kernel
// writes) by a lane pair, lane h (= lane & 1) holding values 16 h .. 16 h + 15
// (max and integer sum are exact in any order), into the activation records:
// quants, d8, A = d8 * sum.  Every lane of the warp calls it (the shuffles
// span the warp); `store` is false for a pair past the last block.
__device__ __forceinline__ void pk_quant16(uint8_t *arec, int i, int h, const float (&x)[16], bool store) {
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(x[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[4];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x[4 * k + j], id)))));
            sum += q;
            word |= (static_cast<uint32_t>(q) & 0xffu) << (8 * j);
        }
        w[k] = word;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    if (!store) return;
    uint8_t *rec = arec + (i >> 3) * PK_AREC;
    const int s = i & 7;
    *reinterpret_cast<uint4 *>(rec + 32 * s + 16 * h) = make_uint4(w[0], w[1], w[2], w[3]);
    if (h == 0) {
        const float d8 = __half2float(__float2half_rn(d));
        reinterpret_cast<float *>(rec + 256)[s] = d8;
        reinterpret_cast<float *>(rec + 288)[s] = __fmul_rn(d8, __int2float_rn(sum));
    }
}

// Before the phase's barrier: the residual stream h_in (stable since an
// earlier phase), or the token's embedding row, into s_x.
__device__ __forceinline__ void pk_xin_stage(int K, const float *h_in, const uint8_t *erow, float *s_x) {
    constexpr int U = 8;
    for (int i0 = threadIdx.x; i0 < K; i0 += 256 * U) {
        float v[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + k * 256;
            v[k] = i < K ? (erow ? pk_embed(erow, i) : __ldcg(h_in + i)) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + k * 256;
            if (i < K) s_x[i] = v[k];
        }
    }
}

// After it: x = s_x + delta (all of this thread's delta loads issued
// first), written to h_out (each CTA its contiguous share); then RMSNorm * w and Q8_1 into the
// activation records -- the XIN prologue of mmvq_q4k_kernel, operation for
// operation (thread t sums x[t + 256 k]^2 with fmaf in k order).
__device__ __forceinline__ void pk_xin(int K, const float *delta, float *h_out, float *s_x, const float *s_w,
                                       float eps, uint8_t *arec, float *s_nred) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    constexpr int U = 10;
    // this CTA's share of the write-back: every CTA holds the same x
    const int own0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * K / gridDim.x);
    const int own1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * K / gridDim.x);
    float acc = 0.0f;
    for (int i0 = t; i0 < K; i0 += 256 * U) {
        float d[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + k * 256;
            d[k] = (delta && i < K) ? __ldcg(delta + i) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + k * 256;
            if (i < K) {
                float v = s_x[i];
                if (delta) v = __fadd_rn(v, d[k]);
                if (i >= own0 && i < own1) h_out[i] = v;
                s_x[i] = v;
                acc = __fmaf_rn(v, v, acc);
            }
        }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
    if (lane == 0) s_nred[warp] = acc;
    cta_sync();
    float total = s_nred[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) total = __fadd_rn(total, s_nred[w]);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), eps)));
    const int nblk = K / QK8_1, h = t & 1;
    for (int i0 = 0; i0 < nblk; i0 += PK_NCW * 16) {  // a lane pair per block, 128 blocks per pass
        const int i = i0 + (t >> 1);
        const bool in = i < nblk;
        float v[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int j = i * QK8_1 + 16 * h + 4 * k;
            const float4 xv = in ? *reinterpret_cast<const float4 *>(s_x + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const float4 wv = in ? *reinterpret_cast<const float4 *>(s_w + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            v[4 * k] = __fmul_rn(__fmul_rn(xv.x, r), wv.x);
            v[4 * k + 1] = __fmul_rn(__fmul_rn(xv.y, r), wv.y);
            v[4 * k + 2] = __fmul_rn(__fmul_rn(xv.z, r), wv.z);
            v[4 * k + 3] = __fmul_rn(__fmul_rn(xv.w, r), wv.w);
        }
        pk_quant16(arec, i, h, v, in);
    }
    cta_sync();
}

// Q8_1 of an fp32 activation written earlier in this launch (the SwiGLU
// output), straight into the records: the bytes quantize_q8_1_kernel writes
// and mmvq_q4k_kernel stages.  A lane pair per block, 16 values each; all
// loads of up to three passes of 128 blocks are issued before the first block
// is rounded, so the 304 blocks of a 9728-wide FFN cost one L2 round trip.
__device__ __forceinline__ void pk_quant_f32(const float *x, int K, uint8_t *arec) {
    constexpr int U = 3;  // passes in flight
    const int nblk = K / QK8_1, t = threadIdx.x, h = t & 1;
    for (int g0 = 0; g0 < nblk; g0 += U * PK_NCW * 16) {
        float4 f[U][4];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = g0 + k * PK_NCW * 16 + (t >> 1);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                f[k][c] = i < nblk ? __ldcg(reinterpret_cast<const float4 *>(x + i * QK8_1 + 16 * h + 4 * c))
                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = g0 + k * PK_NCW * 16 + (t >> 1);
            if (g0 + k * PK_NCW * 16 >= nblk) break;  // CTA-uniform
            float v[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                v[4 * c] = f[k][c].x;
                v[4 * c + 1] = f[k][c].y;
                v[4 * c + 2] = f[k][c].z;
                v[4 * c + 3] = f[k][c].w;
            }
            pk_quant16(arec, i, h, v, i < nblk);
        }
    }
    cta_sync();
}

// Q8_1 blocks written earlier in this launch (oq) into the records (the
// staging loop of mmvq_q4k_kernel, loads through L2): one lane per block.
__device__ __forceinline__ void pk_stage_q8(const uint8_t *X, int K, uint8_t *arec) {
    const int nblk = K / QK8_1;
    for (int i = threadIdx.x; i < nblk; i += PK_NCW * 32) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(X + static_cast<int64_t>(i) * Q81_BYTES);
        uint32_t q[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) q[k] = __ldcg(src + k);
        int msum = 0;
#pragma unroll
        for (int k = 1; k < 9; ++k) msum = dp4a_ss(0x01010101, static_cast<int>(q[k]), msum);
        uint8_t *rec = arec + (i >> 3) * PK_AREC;
        const int s = i & 7;
        uint4 *dst = reinterpret_cast<uint4 *>(rec + 32 * s);
        dst[0] = make_uint4(q[1], q[2], q[3], q[4]);
        dst[1] = make_uint4(q[5], q[6], q[7], q[8]);
        const float d8 = half_lo(q[0]);
        reinterpret_cast<float *>(rec + 256)[s] = d8;
        reinterpret_cast<float *>(rec + 288)[s] = __fmul_rn(d8, __int2float_rn(msum));
    }
    cta_sync();
}

// ------------------------------------------------ consumer: attention ---
// QK-RMSNorm + NEOX RoPE of one head (qk_norm_rope_kv_kernel's arithmetic):
// lane owns elements 4 lane .. 4 lane + 3; nw and cs staged in shared memory.
__device__ __forceinline__ void pk_norm_rope(const float *x128, const float *nw, const float *cs,
                                             float eps, int lane, float (&o)[4]) {
    const float4 xv = __ldcg(reinterpret_cast<const float4 *>(x128 + 4 * lane));
    const float x[4] = {xv.x, xv.y, xv.z, xv.w};
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc = __fmaf_rn(x[k], x[k], acc);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, 128.0f), eps)));
    float y[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) y[k] = __fmul_rn(__fmul_rn(x[k], r), nw[4 * lane + k]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float partner = __shfl_xor_sync(0xffffffffu, y[k], 16);
        const int i = 4 * (lane & 15) + k;
        const float c = cs[2 * i], s = cs[2 * i + 1];
        if (lane < 16)
            o[k] = __fmaf_rn(y[k], c, -__fmul_rn(partner, s));
        else
            o[k] = __fmaf_rn(partner, s, __fmul_rn(y[k], c));
    }
}

// The merged output x of one q head (lane: dims 4 lane .. 4 lane + 3) to
// att and its four Q8_1 blocks to oq (attention_merge_quant_kernel's
// epilogue).
__device__ __forceinline__ void pk_head_out(const PkParams &P, int hq, const float (&x)[4], int lane) {
    *reinterpret_cast<float4 *>(P.att + static_cast<int64_t>(hq) * 128 + 4 * lane) = make_float4(x[0], x[1], x[2], x[3]);
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    amax = fmaxf(0.0f, amax);
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int qv[4], sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        qv[k] = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x[k], id)))));
        sum += qv[k];
    }
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
    uint32_t *o32 = reinterpret_cast<uint32_t *>(P.oq + (static_cast<int64_t>(hq) * 4 + (lane >> 3)) * Q81_BYTES);
    o32[1 + (lane & 7)] = (static_cast<uint32_t>(qv[0]) & 0xffu) | ((static_cast<uint32_t>(qv[1]) & 0xffu) << 8) |
                          ((static_cast<uint32_t>(qv[2]) & 0xffu) << 16) | ((static_cast<uint32_t>(qv[3]) & 0xffu) << 24);
    if ((lane & 7) == 0) {
        const uint32_t hd = __half_as_ushort(__float2half_rn(d));
        const uint32_t hs = __half_as_ushort(__float2half_rn(__fmul_rn(d, static_cast<float>(sum))));
        o32[0] = hd | (hs << 16);
    }
}

// Merge of one q head over nch chunks from the partials in global memory
// (attention_merge_quant_kernel's arithmetic, read through L2).
__device__ __forceinline__ void pk_merge_head(const PkParams &P, int hq, int nch, int lane) {
    const int mc = P.max_chunks;
    const float *pm = P.part_m + static_cast<int64_t>(hq) * mc;
    const float *pl = P.part_l + static_cast<int64_t>(hq) * mc;
    float M = __ldcg(pm);
    for (int c = 1; c < nch; ++c) M = fmaxf(M, __ldcg(pm + c));
    float Ls = 0.0f, O[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c = 0; c < nch; ++c) {
        const float wc = abra_expf(__fsub_rn(__ldcg(pm + c), M));
        Ls = __fmaf_rn(__ldcg(pl + c), wc, Ls);
        const float4 o = __ldcg(reinterpret_cast<const float4 *>(
            P.part_o + (static_cast<int64_t>(hq) * mc + c) * 128 + 4 * lane));
        O[0] = __fmaf_rn(o.x, wc, O[0]);
        O[1] = __fmaf_rn(o.y, wc, O[1]);
        O[2] = __fmaf_rn(o.z, wc, O[2]);
        O[3] = __fmaf_rn(o.w, wc, O[3]);
    }
    float x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = __fdiv_rn(O[k], Ls);
    pk_head_out(P, hq, x, lane);
}

// Shared-memory plan of the attention phase for items of hpi q heads
// (floats): q[hpi][128], e[hpi][256], red[hpi][8], o[8][hpi][128], then the
// staged q/k norm weights and RoPE row (3 x 128), then the new k and v rows
// (fp16, 2 x 128 = 128 floats).
__host__ __device__ constexpr int pk_att_floats(int hpi) {
    return hpi * (128 + ATT_CHUNK_P + 8) + 8 * hpi * 128 + 3 * 128 + 128;
}

// Attention items of a token at position pos: (q heads per item, items).
// Whole kv groups per item (hpi = gq) read each K/V row once per group; one
// q head per item (hpi = 1) spreads a short context over 4x the CTAs and is
// used while all its items fit one round of the grid.
__device__ __forceinline__ int pk_att_hpi(const PkParams &P, int pos, int gq) {
    const int nch = (pos + ATT_CHUNK_P) / ATT_CHUNK_P;
    return P.n_heads * nch <= static_cast<int>(gridDim.x) ? 1 : gq;
}

// Inputs of the attention phase that do not depend on the previous phase,
// staged before its barrier.
__device__ __forceinline__ void pk_stage_att(const PkParams &P, int layer, int pos, int gq, int hpi, float *scr) {
    float *s_in = scr + hpi * (128 + ATT_CHUNK_P + 8) + 8 * hpi * 128;
    const PersistLayer &Ly = P.layers[layer];
    const int t = threadIdx.x;
    if (t >= 32 && t < 128) {  // 16-byte pieces of the q and k norm weights and the RoPE row (not warp 0)
        const int j = t - 32;
        const float *src = j < 32 ? Ly.q_norm : j < 64 ? Ly.k_norm : P.rope + static_cast<int64_t>(pos) * 128;
        cp_async16(s_in + 4 * j, src + 4 * (j & 31));
    }
    // the cached K and V rows of this CTA's items into L2 (positions before
    // pos: written by earlier launches), so that the phase's loads do not
    // queue behind the weight stream in HBM
    if (t < 32) {
        const int L = pos, nch = (pos + ATT_CHUNK_P) / ATT_CHUNK_P;
        const size_t kv_layer = static_cast<size_t>(P.n_kv) * P.max_ctx * 128;
        const int nu = P.n_heads / hpi;
        for (int it = blockIdx.x; it < nu * nch; it += gridDim.x) {
            const int g = (it % nu) * hpi / gq, c = it / nu;
            const int j0 = c * ATT_CHUNK_P, nrow = min(ATT_CHUNK_P, L - j0);
            if (nrow <= 0) continue;
            const int64_t off = layer * kv_layer + (static_cast<int64_t>(g) * P.max_ctx + j0) * 128;
            const uint32_t bytes = static_cast<uint32_t>(nrow) * 256u;  // fp16 rows of 128
            const __half *base = (t & 16) ? P.vc + off : P.kc + off;
            const uint32_t piece = 16384u, lo = (t & 15) * piece;
            if (lo < bytes) prefetch_l2_bulk(reinterpret_cast<const uint8_t *>(base) + lo, min(piece, bytes - lo));
        }
    }
}

// Attention of layer `layer` at position pos: items (HPI consecutive q heads
// of kv group g, chunk c) over the CTAs; each item is attention_chunk_kernel's
// arithmetic on 256 positions for its heads (every head's operations in the
// same order whatever HPI is), its q heads normed and rotated in place.  On
// the chunk holding pos the item also forms the group's new k and v rows and
// keeps them in shared memory; the group's first item appends them to the
// cache.  One chunk: the CTA merges its own heads; more: the last chunk of
// each item's heads to finish merges them from the partials.
template <int HPI>
__device__ __forceinline__ void pk_attention(const PkParams &P, int layer, int pos, int gq, float *scr,
                                             unsigned *s_flag) {
    constexpr int GQ = HPI;  // q heads of this item
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float(*s_q)[128] = reinterpret_cast<float(*)[128]>(scr);                              // [GQ][128]
    float(*s_e)[ATT_CHUNK_P] = reinterpret_cast<float(*)[ATT_CHUNK_P]>(scr + GQ * 128);    // [GQ][256]
    float(*s_red)[8] = reinterpret_cast<float(*)[8]>(scr + GQ * (128 + ATT_CHUNK_P));      // [GQ][8]
    float *s_o = scr + GQ * (128 + ATT_CHUNK_P + 8);                                       // [8][GQ][128]
    float *s_in = s_o + 8 * GQ * 128;                                                      // norms, rope row
    __half *s_knew = reinterpret_cast<__half *>(s_in + 3 * 128);                           // [128]
    __half *s_vnew = s_knew + 128;                                                         // [128]
    const int L = pos + 1, nch = (L + ATT_CHUNK_P - 1) / ATT_CHUNK_P;
    const int nkv = P.n_kv, max_ctx = P.max_ctx, mc = P.max_chunks;
    const size_t kv_layer = static_cast<size_t>(nkv) * max_ctx * 128;
    __half *kc = P.kc + layer * kv_layer, *vc = P.vc + layer * kv_layer;
    const int nu = P.n_heads / HPI, items = nu * nch;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        PK_ASTAMP(layer, 0);
        const int u = it % nu, c = it / nu;
        const int h0 = u * HPI, g = h0 / gq;  // first q head, kv group
        const bool tail = c == nch - 1, first = h0 % gq == 0;
        // the group's q heads; on the chunk holding pos also the k and v
        // heads, appended to the cache (rounded to fp16) and kept here
        for (int hv = warp; hv < GQ + (tail ? 2 : 0); hv += PK_NCW) {
            if (hv < GQ) {
                float o[4];
                pk_norm_rope(P.qkv + static_cast<int64_t>(h0 + hv) * 128, s_in, s_in + 256, P.eps, lane, o);
                *reinterpret_cast<float4 *>(&s_q[hv][4 * lane]) = make_float4(o[0], o[1], o[2], o[3]);
            } else if (hv == GQ) {
                float o[4];
                pk_norm_rope(P.qkv + static_cast<int64_t>(P.n_heads + g) * 128, s_in + 128, s_in + 256, P.eps, lane, o);
                __half *dst = kc + (static_cast<int64_t>(g) * max_ctx + pos) * 128 + 4 * lane;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (first) dst[k] = __float2half_rn(o[k]);
                    s_knew[4 * lane + k] = __float2half_rn(o[k]);
                }
            } else {
                const float4 xv = __ldcg(reinterpret_cast<const float4 *>(
                    P.qkv + static_cast<int64_t>(P.n_heads + nkv + g) * 128 + 4 * lane));
                const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
                __half *dst = vc + (static_cast<int64_t>(g) * max_ctx + pos) * 128 + 4 * lane;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (first) dst[k] = __float2half_rn(xs[k]);
                    s_vnew[4 * lane + k] = __float2half_rn(xs[k]);
                }
            }
        }
        cta_sync();
        PK_ASTAMP(layer, 1);
        const int j = c * ATT_CHUNK_P + t;
        const bool valid = j < L;
        float s[GQ];
#pragma unroll
        for (int h = 0; h < GQ; ++h) s[h] = 0.0f;
        if (valid) {
            // earlier positions come from the cache (written by earlier
            // launches), the current one from shared memory
            const uint4 *krow = j == pos ? reinterpret_cast<const uint4 *>(s_knew)
                                         : reinterpret_cast<const uint4 *>(kc + (static_cast<int64_t>(g) * max_ctx + j) * 128);
            // the row's 16 loads issued together (two halves of 8 for eight
            // heads, to bound registers); the fmaf order over d is unchanged
            constexpr int KP = GQ > 4 ? 8 : 16;
#pragma unroll
            for (int h0 = 0; h0 < 16; h0 += KP) {
                uint4 kv[KP];
#pragma unroll
                for (int d8 = 0; d8 < KP; ++d8) kv[d8] = krow[h0 + d8];
#pragma unroll
                for (int d8 = 0; d8 < KP; ++d8) {
                    const __half2 *k2 = reinterpret_cast<const __half2 *>(&kv[d8]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 kf = __half22float2(k2[e]);
#pragma unroll
                        for (int h = 0; h < GQ; ++h) {
                            const float2 qv = *reinterpret_cast<const float2 *>(&s_q[h][(h0 + d8) * 8 + 2 * e]);
                            s[h] = __fmaf_rn(qv.x, kf.x, s[h]);
                            s[h] = __fmaf_rn(qv.y, kf.y, s[h]);
                        }
                    }
                }
            }
        }
        PK_ASTAMP(layer, 2);
        float mxs[GQ];
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
            const float sv = valid ? __fmul_rn(s[h], P.scale) : -INFINITY;
            float mx = sv;
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
            if (lane == 0) s_red[h][warp] = mx;
            s[h] = sv;
        }
        cta_sync();
        PK_ASTAMP(layer, 3);
        float ev[GQ];
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
            float mx = s_red[h][0];
#pragma unroll
            for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_red[h][w]);
            mxs[h] = mx;
            ev[h] = valid ? abra_expf(__fsub_rn(s[h], mx)) : 0.0f;
            s_e[h][t] = ev[h];
            if (t == 0 && nch > 1) P.part_m[static_cast<int64_t>(h0 + h) * mc + c] = mx;
        }
        cta_sync();  // s_red is reused for the sums
        PK_ASTAMP(layer, 4);
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
            float v = ev[h];
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
            if (lane == 0) s_red[h][warp] = v;
        }
        __syncwarp();
        float acc[GQ][4];
#pragma unroll
        for (int h = 0; h < GQ; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[h][k] = 0.0f;
        const int j0 = c * ATT_CHUNK_P + warp * 32;
        const int nv = max(0, min(32, L - j0));
        const __half *vbase = vc + (static_cast<int64_t>(g) * max_ctx + j0) * 128 + 4 * lane;
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
            if (g8 * 8 >= nv) break;
            uint2 vv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int jj = j0 + g8 * 8 + u;
                if (g8 * 8 + u < nv)
                    vv[u] = *reinterpret_cast<const uint2 *>(jj == pos ? s_vnew + 4 * lane : vbase + (g8 * 8 + u) * 128);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (g8 * 8 + u < nv) {
                    const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv[u].x));
                    const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv[u].y));
                    const float vf[4] = {v01.x, v01.y, v23.x, v23.y};
#pragma unroll
                    for (int h = 0; h < GQ; ++h) {
                        const float e = s_e[h][warp * 32 + g8 * 8 + u];
#pragma unroll
                        for (int k = 0; k < 4; ++k) acc[h][k] = __fmaf_rn(e, vf[k], acc[h][k]);
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < GQ; ++h)
            *reinterpret_cast<float4 *>(s_o + (warp * GQ + h) * 128 + 4 * lane) =
                make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        cta_sync();
        PK_ASTAMP(layer, 5);
        if (nch == 1) {
            // one chunk: merge this CTA's heads in place (the merge's
            // arithmetic on the chunk's own max, sum and output)
            if (warp < GQ) {
                const int h = warp;
                float l = s_red[h][0];
#pragma unroll
                for (int w = 1; w < 8; ++w) l = __fadd_rn(l, s_red[h][w]);
                const float wc = abra_expf(__fsub_rn(mxs[h], mxs[h]));
                const float Ls = __fmaf_rn(l, wc, 0.0f);
                float x[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int d = 4 * lane + k;
                    float o = s_o[h * 128 + d];
#pragma unroll
                    for (int w = 1; w < 8; ++w) o = __fadd_rn(o, s_o[(w * GQ + h) * 128 + d]);
                    x[k] = __fdiv_rn(__fmaf_rn(o, wc, 0.0f), Ls);
                }
                pk_head_out(P, h0 + h, x, lane);
            }
            PK_ASTAMP(layer, 6);
            cta_sync();  // the scratch is reused by the next item
            PK_ASTAMP(layer, 7);
            continue;
        }
        for (int i = t; i < GQ * 128; i += 256) {
            const int h = i / 128, d = i % 128;
            float o = s_o[h * 128 + d];
#pragma unroll
            for (int w = 1; w < 8; ++w) o = __fadd_rn(o, s_o[(w * GQ + h) * 128 + d]);
            P.part_o[(static_cast<int64_t>(h0 + h) * mc + c) * 128 + d] = o;
        }
        if (t < GQ) {
            float l = s_red[t][0];
#pragma unroll
            for (int w = 1; w < 8; ++w) l = __fadd_rn(l, s_red[t][w]);
            P.part_l[static_cast<int64_t>(h0 + t) * mc + c] = l;
        }
        // the last chunk of the item's heads to finish merges them: one
        // acquire-release add publishes this chunk's partials (the CTA barrier
        // made them visible to thread 0) and, for the last, acquires the others'
        cta_sync();
        if (t == 0) {
            unsigned old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(P.head_cnt + h0) : "memory");
            const unsigned last = old + 1u == static_cast<unsigned>(nch) ? 1u : 0u;
            if (last) P.head_cnt[h0] = 0u;
            *s_flag = last;
        }
        cta_sync();
        if (*s_flag && warp < GQ) pk_merge_head(P, h0 + warp, nch, lane);
        cta_sync();  // the scratch is reused by the next item
    }
}

// --------------------------------------------------------------- kernel ---
template <int GQ>
__global__ void __launch_bounds__(PK_THREADS, 1) decode_token_kernel(const PkParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_nred[8];
    __shared__ unsigned long long s_amax;
    __shared__ unsigned s_flag;
    __shared__ PkTickets s_tk;  // this CTA's ticket map (indexed by GEMV kind at run time)
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + P.off_ring;
    const int pos = __ldcg(P.pos);
    if (pos < 0 || pos >= P.max_ctx) return;  // the host never steps past max_ctx
    if (threadIdx.x == 0) {
        for (int s = 0; s < (1 << P.slot_shift); ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
        pk_tickets(P, s_tk);
    }
    __syncthreads();
    const int t = threadIdx.x;
    const int L = P.n_layers;
    const PkTickets &tk = s_tk;
    const uint64_t pol = policy_evict_first();
    const PkTicketPos start = {L > 0 ? PK_QKV : PK_OUT, 0, 0};
    if ((t & 31) == 0) {  // the first NSLOT tickets, lane 0 of warp w: w, w + 8
        const uint32_t first = min(tk.total, 1u << P.slot_shift);
        for (uint32_t tt = t >> 5; tt < first; tt += PK_NCW)
            pk_issue(P, tk, pk_ticket_ahead(tk, L, start, static_cast<int>(tt)), static_cast<int>(tt), ring, full, pol);
    }
    float *vbuf = reinterpret_cast<float *>(smem + P.off_vbuf) + (t >> 5) * PK_VMAX;
    uint8_t *arec = smem + P.off_arec;
    float *scr = reinterpret_cast<float *>(smem + P.off_x);
    const int hidden = P.hidden;
    float *s_x = scr, *s_w = scr + hidden;
    const unsigned long long G = gridDim.x;
    const int nev = 5 * L + 1;  // phases of the token; a grid barrier between consecutive ones
    unsigned long long kb = *reinterpret_cast<volatile unsigned long long *>(P.gen) * static_cast<unsigned long long>(nev);
    uint32_t T = 0;
    bool poisoned = false;
    int cur = 0;
    int tok = __ldcg(P.tokens + pos);
    if (tok < 0 || tok >= P.vocab) {  // never from a valid pick or prompt: flag it, read row 0
        if (t == 0) report_error(ERR_BAD_INDEX);
        tok = 0;
    }
    const uint8_t *erow = P.embd + static_cast<int64_t>(tok) * (hidden / QK_K) * Q4K_BYTES;
    for (int e = 0; e < nev; ++e) {
        const int l = e / 5;
        const int ph = e == nev - 1 ? PH_OUT : e % 5;
        const bool xin = ph == PH_QKV || ph == PH_GU || ph == PH_OUT;
        const bool first = xin && (ph == PH_QKV ? l == 0 : L == 0);  // the embedding row, no residual delta
        // inputs that do not depend on the previous phase, staged before its
        // barrier: norm weights, the residual stream (written two or more
        // phases back) or the embedding row, the attention's norms and RoPE row
        if (first) {  // the embedding row: no earlier phase to stage it in
            pk_stage_norm(ph == PH_OUT ? P.out_norm : P.layers[l].attn_norm, s_w, hidden);
            pk_xin_stage(hidden, nullptr, erow, s_x);
        } else if (ph == PH_ATT)
            pk_stage_att(P, l, pos, GQ, pk_att_hpi(P, pos, GQ), scr);
        if (ph == PH_OUT && t == 0) s_amax = 0ull;
        if (e > 0) {
            ++kb;
            if (t == 0) pk_wait(P.bar, kb * G);
        }
        if (t == 0) PK_STAMP(0, e);
        cp_async_wait();  // this thread's staged inputs (the barrier below shares them)
        cta_sync();
        // the phase's activation
        if (xin) {
            pk_xin(hidden, first ? nullptr : P.delta, P.h[cur ^ 1], s_x, s_w, P.eps, arec, s_nred);
            cur ^= 1;
        } else if (ph == PH_O) {
            pk_stage_q8(P.oq, P.n_heads * 128, arec);
        } else if (ph == PH_DOWN) {
            pk_quant_f32(P.act, P.ffn, arec);
            // the next prologue's inputs: the residual stream written in this
            // layer's GU prologue (visible since this phase's barrier), behind
            // this prologue's own loads
            pk_stage_xin_async(l + 1 < L ? P.layers[l + 1].attn_norm : P.out_norm, P.h[cur], s_w, s_x, hidden);
        }
        if (t == 0) PK_STAMP(3, e);
#ifdef ABRA_PK_TRACE
        if (t == 0) g_pk_wait_ns = 0;
        cta_sync();
#endif
        // the phase's work
        if (ph == PH_ATT) {
            if (GQ > 1 && pk_att_hpi(P, pos, GQ) == 1)
                pk_attention<1>(P, l, pos, GQ, scr, &s_flag);
            else
                pk_attention<GQ>(P, l, pos, GQ, scr, &s_flag);
        } else {
            const int kind = ph == PH_QKV ? PK_QKV : ph == PH_O ? PK_O : ph == PH_GU ? PK_GU : ph == PH_DOWN ? PK_DOWN : PK_OUT;
            float *Y = ph == PH_QKV ? P.qkv : ph == PH_GU ? P.act : ph == PH_OUT ? P.logits : P.delta;
            const PkMm mm = pk_mm(P, l, kind);
            int u_begin, nu;
            pk_range(mm, u_begin, nu);
            unsigned long long *amax = ph == PH_OUT ? &s_amax : nullptr;
            const PkTicketPos at = {kind, ph == PH_OUT ? L : l, 0};
            if (ph == PH_OUT && t == PK_NCW * 32 - 1) pk_prefetch_next(P, tk);
            if (mm.w1)
                pk_units<2>(P, tk, at, pol, mm, u_begin, nu, T, ring, full, vbuf, arec, Y, amax, P.slot_shift, poisoned);
            else
                pk_units<1>(P, tk, at, pol, mm, u_begin, nu, T, ring, full, vbuf, arec, Y, amax, P.slot_shift, poisoned);
            T += static_cast<uint32_t>(nu);
        }
        cta_sync();
        if (t == 0) PK_STAMP(1, e);
#ifdef ABRA_PK_TRACE
        if (t == 0 && e < PK_TRACE_EV && blockIdx.x < 160) g_pk_trace[blockIdx.x][4][e] = g_pk_wait_ns;
#endif
        if (e < nev - 1 && t == 0) pk_arrive(P.bar);
        // the attention scratch is free: the GU prologue's inputs (the residual
        // stream written in this layer's QKV prologue) in the background
        if (ph == PH_ATT) pk_stage_xin_async(P.layers[l].ffn_norm, P.h[cur], s_w, s_x, hidden);
    }
    // the greedy pick: the last CTA to arrive decodes the merged key
    if (t == 0) {
        atomicMax(P.amax, s_amax);
        __threadfence();
        const unsigned long long old = atom_add_acq_rel_gpu(P.bar, 1ull);
        if (old + 1ull == (kb + 1ull) * G) {  // the last CTA of the launch
            __threadfence();
            const unsigned long long key = __ldcg(P.amax);
            *P.amax = 0ull;
            int bi = static_cast<int>(0xFFFFFFFFu - static_cast<unsigned>(key & 0xFFFFFFFFull));
            if (bi < 0 || bi >= P.vocab) {  // no key was merged: flag it, pick row 0
                report_error(ERR_BAD_INDEX);
                bi = 0;
            }
            P.picks[pos] = bi;
            if (pos + 1 >= __ldcg(P.nprompt)) P.tokens[pos + 1] = bi;
            *P.pos = pos + 1;
            *P.gen = *reinterpret_cast<volatile unsigned long long *>(P.gen) + 1ull;
            __threadfence();
        }
    }
}

using PkKernel = void (*)(const PkParams);

PkKernel pk_kernel_for(int gq) {
    switch (gq) {
        case 1: return decode_token_kernel<1>;
        case 2: return decode_token_kernel<2>;
        case 4: return decode_token_kernel<4>;
        case 8: return decode_token_kernel<8>;
        default: return nullptr;
    }
}

// ------------------------------------------------------------ planning ---
struct PkPlan {
    int rows[PK_KINDS], pitch[PK_KINDS];
    int slot_shift;
    int off_vbuf, off_arec, off_x, off_ring, smem;
};

int pk_align(int v, int a) { return (v + a - 1) / a * a; }

int log2i(int v) {
    int l = 0;
    while ((1 << l) < v) ++l;
    return l;
}

// Rows per unit and row pitch of each GEMV, chosen by the critical path of
// the phase on `sms` CTAs (superblock passes of the busiest warp plus its row
// sums), and the shared-memory layout.
bool pk_plan(int hidden, int n_heads, int n_kv, int ffn, int head_dim, int vocab, int sms, PkPlan &pl,
             const char **why) {
    auto no = [&](const char *w) {
        if (why) *why = w;
        return false;
    };
    if (head_dim != 128 || n_kv <= 0 || n_heads % n_kv) return no("head layout");
    const int gq = n_heads / n_kv;
    if (gq != 1 && gq != 2 && gq != 4 && gq != 8) return no("q heads per kv head must be 1, 2, 4 or 8");
    if (hidden % QK_K || ffn % QK_K || (n_heads * 128) % QK_K || hidden <= 0 || ffn <= 0 || vocab <= 0)
        return no("dimensions must be multiples of 256");
    if (sms < 1) sms = 1;
    const int nsb[PK_KINDS] = {hidden / QK_K, n_heads * 128 / QK_K, hidden / QK_K, ffn / QK_K, hidden / QK_K};
    const int nmat[PK_KINDS] = {1, 1, 2, 1, 1};
    const int64_t N[PK_KINDS] = {static_cast<int64_t>(n_heads + 2 * n_kv) * 128, hidden, ffn, hidden, vocab};
    for (int k = 0; k < PK_KINDS; ++k) {
        pl.rows[k] = 0;
        int64_t best = -1;
        for (int R : {8, 4, 2, 1}) {
            const int pitch = nsb[k] * Q4K_BYTES;  // rows back to back, as in HBM
            if (nmat[k] * R * pitch > PK_SLOT_BYTES || nmat[k] * R * nsb[k] > PK_VMAX) continue;
            const int64_t units = (N[k] + R - 1) / R;
            const int64_t per_cta = (units + sms - 1) / sms;
            const int64_t per_warp = (per_cta + PK_NCW - 1) / PK_NCW;
            const int64_t passes = (nsb[k] + 32 / R - 1) / (32 / R);
            const int64_t cost = per_warp * (16 * passes * nmat[k] + nsb[k] * nmat[k]);
            if (best < 0 || cost < best) {
                best = cost;
                pl.rows[k] = R;
                pl.pitch[k] = pitch;
            }
        }
        if (!pl.rows[k]) return no("a row does not fit a ring slot");
    }
    const int nsb_max = std::max(std::max(hidden, n_heads * 128), ffn) / QK_K;
    const int scratch = std::max(8 * hidden, 4 * pk_att_floats(gq));
    int o = 16 * PK_NSLOT;  // the slots' full mbarriers (room reserved for two per slot)
    pl.off_vbuf = pk_align(o, 16);
    o = pl.off_vbuf + PK_NCW * PK_VMAX * 4;
    pl.off_arec = pk_align(o, 128);
    o = pl.off_arec + nsb_max * PK_AREC;
    pl.off_x = pk_align(o, 16);
    o = pl.off_x + scratch;
    pl.off_ring = pk_align(o, 128);
    for (int shift : {4, 3}) {  // 16 slots, or 8 when the activations leave less room
        pl.slot_shift = shift;
        pl.smem = pl.off_ring + (1 << shift) * PK_SLOT_BYTES;
        if (pl.smem <= kMmvqMaxSmem) return true;
    }
    return no("shared memory");
}

}  // namespace

size_t persist_sync_bytes(int n_heads) { return static_cast<size_t>(pk_align(16 + 4 * n_heads, 256)); }

bool persist_supported(int hidden, int n_heads, int n_kv, int ffn, int head_dim, const char **why) {
    PkPlan pl;
    return pk_plan(hidden, n_heads, n_kv, ffn, head_dim, 1, 148, pl, why);
}

cudaError_t persist_prepare(int hidden, int n_heads, int n_kv, int ffn) {
    PkPlan pl;
    if (!pk_plan(hidden, n_heads, n_kv, ffn, 128, 1, device_sm_count(), pl, nullptr)) return cudaErrorInvalidValue;
    PkKernel fn = pk_kernel_for(n_heads / n_kv);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = ensure_smem_attr_ptr(reinterpret_cast<const void *>(fn));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, PK_THREADS, pl.smem);
    if (e != cudaSuccess) return e;
    return per_sm < 1 ? cudaErrorCooperativeLaunchTooLarge : cudaSuccess;
}

cudaError_t launch_persist_step(const PersistModel &pm, cudaStream_t st) {
    PkPlan pl;
    const int sms = device_sm_count();
    if (!pk_plan(pm.hidden, pm.n_heads, pm.n_kv, pm.ffn, 128, pm.vocab, sms, pl, nullptr))
        return cudaErrorInvalidValue;
    PkKernel fn = pk_kernel_for(pm.n_heads / pm.n_kv);
    if (!fn) return cudaErrorInvalidValue;
    PkParams P = {};
    P.layers = pm.layers;
    P.embd = pm.embd;
    P.out_norm = pm.out_norm;
    P.n_layers = pm.n_layers;
    P.hidden = pm.hidden;
    P.n_heads = pm.n_heads;
    P.n_kv = pm.n_kv;
    P.ffn = pm.ffn;
    P.vocab = pm.vocab;
    P.max_ctx = pm.max_ctx;
    P.max_chunks = (pm.max_ctx + ATT_CHUNK_P - 1) / ATT_CHUNK_P;
    P.eps = pm.eps;
    P.scale = static_cast<float>(1.0 / std::sqrt(128.0));
    P.h[0] = pm.h0;
    P.h[1] = pm.h1;
    P.delta = pm.delta;
    P.qkv = pm.qkv;
    P.att = pm.att;
    P.part_m = pm.part_m;
    P.part_l = pm.part_l;
    P.part_o = pm.part_o;
    P.act = pm.act;
    P.logits = pm.logits;
    P.oq = pm.oq;
    P.kc = static_cast<__half *>(pm.kc);
    P.vc = static_cast<__half *>(pm.vc);
    P.rope = pm.rope;
    P.tokens = pm.tokens;
    P.picks = pm.picks;
    P.pos = pm.pos;
    P.nprompt = pm.nprompt;
    P.amax = pm.amax;
    uint8_t *sync = static_cast<uint8_t *>(pm.sync);
    P.bar = reinterpret_cast<unsigned long long *>(sync);
    P.gen = P.bar + 1;
    P.head_cnt = reinterpret_cast<unsigned *>(sync + 16);
    for (int k = 0; k < PK_KINDS; ++k) {
        P.lr[k] = log2i(pl.rows[k]);
        P.pitch[k] = pl.pitch[k];
    }
    P.slot_shift = pl.slot_shift;
    P.off_vbuf = pl.off_vbuf;
    P.off_arec = pl.off_arec;
    P.off_x = pl.off_x;
    P.off_ring = pl.off_ring;
    P.smem = pl.smem;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(PK_THREADS);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, P);
}

// Host-side walk of every bulk copy the warps of `sms` CTAs would issue
// for a model shape, checked against the ring slot and the weight tensors:
// out = {smem, ring bytes, units of the busiest CTA, copies checked, rows per
// unit of the five GEMVs}.  Returns false with *why set when a copy would
// leave its slot or its tensor.
bool persist_plan_check(int n_layers, int hidden, int n_heads, int n_kv, int ffn, int vocab, int sms,
                        int64_t out[9], const char **why) {
    PkPlan pl;
    if (!pk_plan(hidden, n_heads, n_kv, ffn, 128, vocab, sms, pl, why)) return false;
    const int nsb[PK_KINDS] = {hidden / QK_K, n_heads * 128 / QK_K, hidden / QK_K, ffn / QK_K, hidden / QK_K};
    const int rows[PK_KINDS] = {(n_heads + 2 * n_kv) * 128, hidden, ffn, hidden, vocab};
    const int nmat[PK_KINDS] = {1, 1, 2, 1, 1};
    const int64_t nslot = int64_t(1) << pl.slot_shift;
    int64_t max_tickets = 0, copies = 0;
    auto fail = [&](const char *w) {
        if (why) *why = w;
        return false;
    };
    // the consumer side of a unit (the same for every unit of a GEMV kind):
    // every lane's superblock reads inside its slot, its staging-buffer
    // writes and the row sums' reads inside PK_VMAX, its activation records
    // inside the staged K -- the lane map of pk_units, restated
    for (int kind = 0; kind < PK_KINDS; ++kind) {
        const int R = pl.rows[kind], lr = R == 8 ? 3 : R == 4 ? 2 : R == 2 ? 1 : 0, LP = 32 >> lr;
        const int nb = nsb[kind], nm = nmat[kind];
        for (int lane = 0; lane < 32; ++lane) {
            int r, p0;
            if (LP >= 8) {
                r = lane / LP;
                p0 = lane % LP;
            } else {
                const int q4 = lane >> 3, w8 = lane & 7;
                r = (w8 >> 1) + 4 * (q4 & 1);
                p0 = (w8 & 1) + 2 * (q4 >> 1);
            }
            if (r >= R) return fail("lane row outside its unit");
            for (int bb = p0; bb < nb; bb += LP)
                for (int m = 0; m < nm; ++m) {
                    const int64_t off = static_cast<int64_t>(m * R + r) * pl.pitch[kind] + bb * Q4K_BYTES;
                    if (off + Q4K_BYTES > static_cast<int64_t>(nm) * R * pl.pitch[kind] || off + Q4K_BYTES > PK_SLOT_BYTES ||
                        (m * R + r) * nb + bb >= PK_VMAX)
                        return fail("a lane's superblock leaves its slot or staging buffer");
                }
            for (int half = 0; half < 2; ++half) {  // row sums: rows g, g + 4 of the unit
                const int rr = (lane >> 3) + 4 * half;
                if (rr < R && ((nm - 1) * R + rr + 1) * nb > PK_VMAX) return fail("row sums leave the staging buffer");
            }
        }
    }
    // the ticket walk the warps refill the ring with: from the start,
    // and NSLOT ahead of every ticket, it must name the unit of the sequential
    // phase-by-phase order
    const int Nk[PK_KINDS] = {rows[0], rows[1], rows[2], rows[3], rows[4]};
    int lrk[PK_KINDS];
    for (int k = 0; k < PK_KINDS; ++k) lrk[k] = pl.rows[k] == 8 ? 3 : pl.rows[k] == 4 ? 2 : pl.rows[k] == 2 ? 1 : 0;
    for (int b = 0; b < sms; ++b) {
        PkTickets tk;
        pk_tickets_for(Nk, lrk, n_layers, b, sms, tk);
        std::vector<PkTicketPos> seq;
        for (int l = 0; l < n_layers; ++l)
            for (int k = 0; k < PK_OUT; ++k)
                for (int u = 0; u < tk.nu[k]; ++u) seq.push_back({k, l, u});
        for (int u = 0; u < tk.nu[PK_OUT]; ++u) seq.push_back({PK_OUT, n_layers, u});
        if (seq.size() != tk.total) return fail("ticket count");
        const PkTicketPos start = {n_layers > 0 ? PK_QKV : PK_OUT, 0, 0};
        const int ahead = 1 << pl.slot_shift;
        auto same = [](const PkTicketPos &x, const PkTicketPos &y) {
            return x.kind == y.kind && x.layer == y.layer && x.u == y.u;
        };
        for (size_t i = 0; i < seq.size(); ++i) {
            if (i < static_cast<size_t>(ahead) && !same(pk_ticket_ahead(tk, n_layers, start, static_cast<int>(i)), seq[i]))
                return fail("first tickets of the ring");
            if (i + ahead < seq.size() && !same(pk_ticket_ahead(tk, n_layers, seq[i], ahead), seq[i + ahead]))
                return fail("ring refill ticket");
        }
    }
    for (int b = 0; b < sms; ++b) {
        int64_t t = 0;
        const int nph = 4 * n_layers + 1;
        for (int ph = 0; ph < nph; ++ph) {
            const int kind = ph == nph - 1 ? PK_OUT : (ph & 3);
            const int N = rows[kind], R = pl.rows[kind], pitch = pl.pitch[kind];
            const int64_t row_bytes = static_cast<int64_t>(nsb[kind]) * Q4K_BYTES;
            const int64_t total = (N + R - 1) / R;
            const int u0 = static_cast<int>(b * total / sms), u1 = static_cast<int>((b + 1) * total / sms);
            if (nmat[kind] * R * nsb[kind] > PK_VMAX || (R != 1 && R != 2 && R != 4 && R != 8))
                return fail("unit exceeds the staging buffer");
            for (int u = u0; u < u1; ++u, ++t) {
                const int row0 = u * R, nvalid = std::min(R, N - row0);
                if (nvalid <= 0 || row_bytes != pitch || (pitch & 15) || nmat[kind] * nvalid * row_bytes > (1 << 20) - 1)
                    return fail("unit does not fit its row pitch");
                for (int m = 0; m < nmat[kind]; ++m) {  // one copy per (unit, matrix)
                    const int64_t bytes = nvalid * row_bytes;
                    const int64_t dst = (t % nslot) * PK_SLOT_BYTES + m * R * row_bytes;
                    const int64_t src = static_cast<int64_t>(row0) * row_bytes;
                    const int64_t tensor = static_cast<int64_t>(N) * row_bytes;
                    if (dst + bytes > nslot * PK_SLOT_BYTES || (dst & 15) || (bytes & 15) || src + bytes > tensor ||
                        (src & 15) || (m + 1) * R * row_bytes > PK_SLOT_BYTES)
                        return fail("copy leaves its slot or its tensor");
                    ++copies;
                }
            }
        }
        max_tickets = std::max(max_tickets, t);
    }
    const int64_t v[9] = {pl.smem, int64_t(PK_SLOT_BYTES) << pl.slot_shift, max_tickets, copies,
                          pl.rows[0], pl.rows[1], pl.rows[2], pl.rows[3], pl.rows[4]};
    for (int i = 0; i < 9; ++i) out[i] = v[i];
    return true;
}

}  // namespace abra

#ifdef ABRA_PK_TRACE
extern "C" int abra_pk_trace(unsigned long long *out, long long n) {
    const long long all = static_cast<long long>(sizeof(abra::g_pk_trace) / 8);
    return cudaMemcpyFromSymbol(out, abra::g_pk_trace, 8 * (n < all ? n : all)) == cudaSuccess ? 0 : -2;
}
extern "C" int abra_pk_att(unsigned long long *out) {
    return cudaMemcpyFromSymbol(out, abra::g_pk_att, sizeof(abra::g_pk_att)) == cudaSuccess ? 0 : -2;
}
#endif

ABRA_ERROR_WORD_ACCESSOR(error_word_persist)
