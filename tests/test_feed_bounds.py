"""Host-side index checks of the MMVQ kernels' weight feeds (no GPU).

For every launch plan the dispatch would make (abra_mmvq_plan_info: grid,
ring depth, stage pitch, shared-memory layout, for B200's 148 SMs), this
file follows each address the kernels form -- the producer warp's bulk
copies (cp.async.bulk, global -> shared), its plain tail copies, the
consumers' shared-memory and direct global loads -- and checks what the
hardware requires of them:

* every global read lies inside the weight tensor;
* every bulk copy starts on a 16-byte boundary at both ends and moves a
  multiple of 16 bytes; one stage's expected transaction bytes stay below
  the mbarrier's 2^20 limit;
* every shared-memory write and read stays inside its stage (its row's
  pitch) and the ring stays inside the dynamic shared memory, which stays
  within the opt-in limit;
* the CTAs' row-group ranges tile the rows exactly once, and the ring depth
  obeys the parity rule of the planner (each CTA's units get their own
  stages, or the depth is a multiple of the eight consumer warps).

The address arithmetic restated here is that of mmvq_impl.cuh (Q4_K) and
mmvq_q6k_impl.cuh (Q6_K); a change there that breaks one of these rules for
any shape below fails here, on the CPU, before the kernel runs on a GPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from abra_b200 import _lib

SMS = 148
NCW = 8
MAX_SMEM = 227 * 1024 - 1024
TX_LIMIT = (1 << 20) - 1
Q4K, Q6K = 144, 210
MODE_NAMES = {0: "rows", 1: "whole", 2: "direct", 3: "lane"}


def slice_start(nsb: int, i: int) -> int:
    q, r = divmod(nsb, 8)
    return i * q + min(i, r)


def shard_slice(sl_nsb: int, sl_base: int, sl_shift: int, i: int) -> int:
    return slice_start(sl_nsb, sl_base + ((i + (1 << sl_shift) - 1) >> sl_shift)) - slice_start(sl_nsb, sl_base)


def plan(ggml_type, cand, N, K, ncols=1, nmat=1, xin=0, K_full=0, sl_base=0, sl_cnt=8):
    out = np.zeros(8, dtype=np.int64)
    rc = _lib.lib.abra_mmvq_plan_info(ggml_type, cand, N, K, ncols, nmat, xin, K_full, sl_base,
                                      sl_cnt, SMS, out.ctypes.data)
    if rc == _lib.ABRA_E_UNSUPPORTED:
        return None
    assert rc == _lib.ABRA_OK, _lib.last_error()
    keys = ("grid", "block", "nstage", "pitch", "stage_bytes", "smem", "rg_total", "off_stage")
    return dict(zip(keys, (int(v) for v in out)))


def _cands(kind):
    n = _lib.lib.abra_candidate_count() if kind == "q4k" else _lib.lib.abra_q6k_candidate_count()
    out = []
    for i in range(n):
        v = [C.c_int32() for _ in range(6)]
        if kind == "q4k":
            _lib.lib.abra_candidate_info(i, *[C.byref(x) for x in v])
            cid, mode, ks, _, cps, _ = (x.value for x in v)
        else:
            _lib.lib.abra_q6k_candidate_info(i, *[C.byref(x) for x in v[:5]])
            cid, mode, ks, cps, _ = (x.value for x in v[:5])
        out.append((cid, mode, ks, cps))
    return out


def _units(pl, ks, staged):
    """Every (cta, unit u, row group) each CTA walks."""
    G, R = pl["grid"], pl["rg_total"]
    b = np.arange(G, dtype=np.int64)
    rb, re = b * R // G, (b + 1) * R // G
    nrg = re - rb
    assert nrg.min() >= 1 and nrg.sum() == R and rb[0] == 0 and re[-1] == R
    U = nrg * ks
    nst = pl["nstage"]
    assert nst >= 1
    if staged:
        assert np.all((nst >= U) | (nst % NCW == 0)), "ring depth breaks the parity rule"
    cta = np.repeat(b, U)
    u = np.arange(U.sum(), dtype=np.int64) - np.repeat(np.cumsum(U) - U, U)
    rg = rb[cta] + u // ks
    j = u % ks
    return cta, u, rg, j


def _part_bounds(nsb, ks, shard):
    sl_nsb, sl_base, sl_cnt = shard if shard else (nsb, 0, 8)
    shift = {8: 0, 4: 1, 2: 2, 1: 3}[sl_cnt]
    nsl = 8 // ks
    lo = np.array([shard_slice(sl_nsb, sl_base, shift, jj * nsl) for jj in range(ks)], dtype=np.int64)
    hi = np.array([shard_slice(sl_nsb, sl_base, shift, (jj + 1) * nsl) for jj in range(ks)], dtype=np.int64)
    assert shard_slice(sl_nsb, sl_base, shift, 8) == nsb
    return lo, hi


def check_q4k_lane(pl, N, K, nmat):
    """The lane-mapped kernel (mmvq_lane.cu): units of R consecutive rows,
    one bulk copy per (unit, matrix) of nvalid whole rows into slot u % nslot
    of the ring; lanes read whole superblocks of rows < R from the slot."""
    nsb = K // 256
    row_bytes = nsb * Q4K
    G, total, nslot = pl["grid"], pl["rg_total"], pl["nstage"]
    slot, off = pl["stage_bytes"], pl["off_stage"]
    assert pl["pitch"] == row_bytes and slot % (nmat * row_bytes) == 0
    R = slot // (nmat * row_bytes)
    assert R in (1, 2, 4, 8) and R * nmat * nsb <= 80, "a unit does not fit the warp's staging buffer"
    assert total == (N + R - 1) // R and G <= total and pl["block"] == (NCW + 1) * 32
    assert pl["smem"] <= MAX_SMEM and off % 128 == 0 and off + nslot * slot <= pl["smem"]
    b = np.arange(G, dtype=np.int64)
    ub, ue = b * total // G, (b + 1) * total // G
    nu = ue - ub
    assert nu.min() >= 1 and nu.sum() == total
    assert np.all((nslot >= nu) | (nslot % NCW == 0)), "ring depth breaks the parity rule"
    cta = np.repeat(b, nu)
    u = np.arange(total, dtype=np.int64) - np.repeat(np.cumsum(nu) - nu, nu)
    row0 = (ub[cta] + u) * R
    nvalid = np.minimum(R, N - row0)
    assert nvalid.min() >= 1
    s = u % nslot
    src, nbytes = row0 * row_bytes, nvalid * row_bytes
    for m in range(nmat):
        dst = off + s * slot + m * R * row_bytes
        assert np.all(src % 16 == 0) and np.all(nbytes % 16 == 0) and np.all(dst % 16 == 0)
        assert (src + nbytes).max() <= N * row_bytes
        assert np.all(dst + nbytes <= off + (s + 1) * slot)
    assert (nmat * nbytes).max() <= TX_LIMIT
    return True


def check_q4k(cand, mode, ks, cps, N, K, ncols, nmat=1, xin=0, shard=None):
    kf, sb, sc = (shard[0] * 256, shard[1], shard[2]) if shard else (0, 0, 8)
    pl = plan(12, cand, N, K, ncols, nmat, xin, kf, sb, sc)
    if pl is None:
        return False
    if mode == 3:
        if ncols == 1 and not xin and not shard:
            return check_q4k_lane(pl, N, K, nmat)
        # elsewhere the candidate runs a template plan (mmvq_classic)
        mode, ks, cps = (1, 1, min(cps, 2)) if ks >= 4 else (0, 2, 1)
    nsb = K // 256
    staged = mode != 2
    assert pl["block"] == (NCW + staged) * 32
    assert pl["rg_total"] == (N + 7) // 8 and pl["grid"] <= min(pl["rg_total"], SMS * cps)
    assert pl["smem"] <= MAX_SMEM
    lo, hi = _part_bounds(nsb, ks, shard)
    part = (hi - lo) * Q4K
    w_bytes = N * nsb * Q4K
    cta, u, rg, j = _units(pl, ks, staged)
    row0 = rg * 8
    nvalid = np.minimum(8, N - row0)
    if not staged:
        # lanes (p, g) load 16-byte vectors at +0, +16+32p, +32+32p of each
        # superblock of their (clamped) row: inside the block, 16-aligned
        assert (32 + 32 * 3 + 16) <= Q4K and Q4K % 16 == 0
        rr = np.minimum(row0 + 7, N - 1)
        last = (rr * nsb + hi[j]) * Q4K
        assert last.max() <= w_bytes
        return True
    pitch, nst, sbytes, off = pl["pitch"], pl["nstage"], pl["stage_bytes"], pl["off_stage"]
    assert sbytes == 8 * nmat * pitch and pitch % 16 == 0 and off % 128 == 0
    assert off + nst * sbytes <= pl["smem"]
    assert pitch >= part.max(), "a row's part does not fit its pitch"
    s = u % nst
    if mode == 1:  # whole unit: nvalid rows of the full width, contiguous
        assert ks == 1 and pitch == nsb * Q4K
        src = row0 * nsb * Q4K
        nbytes = nvalid * part[j]
        for m in range(nmat):
            dst = off + (s * nmat + m) * 8 * pitch
            assert np.all(src % 16 == 0) and np.all(nbytes % 16 == 0) and np.all(dst % 16 == 0)
            assert (src + nbytes).max() <= w_bytes
            assert np.all(dst + nbytes <= off + (s * nmat + m + 1) * 8 * pitch)
    else:  # one bulk copy per valid row
        for lane in range(8):
            ok = lane < nvalid
            src = ((row0 + lane) * nsb + lo[j]) * Q4K
            for m in range(nmat):
                dst = off + ((s * nmat + m) * 8 + lane) * pitch
                assert np.all(src[ok] % 16 == 0) and np.all(part % 16 == 0) and np.all(dst % 16 == 0)
                assert np.all((src + part[j])[ok] <= w_bytes)
                assert np.all(dst + part[j] <= dst + pitch)
    tx = nmat * nvalid * part[j]
    assert tx.max() <= TX_LIMIT
    # consumers read 16-byte vectors up to the part's end from each row's pitch
    assert (part.max() // Q4K - 1) * Q4K + 32 + 32 * 3 + 16 <= pitch
    return True


def _q6_copy(start, end, w_bytes):
    a = start & ~15
    lim = w_bytes & ~15
    b = np.maximum(np.minimum((end + 15) & ~15, lim), a)
    return a, b


def check_q6k(cand, mode, ks, cps, N, K, ncols, shard=None):
    kf, sb, sc = (shard[0] * 256, shard[1], shard[2]) if shard else (0, 0, 8)
    pl = plan(14, cand, N, K, ncols, 1, 0, kf, sb, sc)
    if pl is None:
        return False
    nsb = K // 256
    RB = nsb * Q6K
    staged = mode != 2
    assert pl["block"] == (NCW + staged) * 32
    assert pl["rg_total"] == (N + 7) // 8 and pl["grid"] <= min(pl["rg_total"], SMS * cps)
    assert pl["smem"] <= MAX_SMEM
    lo, hi = _part_bounds(nsb, ks, shard)
    w_bytes = N * RB
    cta, u, rg, j = _units(pl, ks, staged)
    row0 = rg * 8
    nvalid = np.minimum(8, N - row0)
    # a lane's reads inside one 210-byte block at an even address p0: the
    # ql run [64h+32s, +32) and the qh run [128+32h, +32), each as nine
    # aligned words from the word holding its first byte, so within
    # [run - 2, run + 36); the scales [192, 208) and d [208, 210) as 16-bit
    # loads.  Reads end by the block's end and begin at most 2 bytes before
    # it, and only when p0 = 2 (mod 4), i.e. never at the tensor's 16-aligned
    # start or a stage row's start.
    reach = max([64 * h + 32 * s + 36 for h in (0, 1) for s in (0, 1)] +
                [128 + 32 * h + 36 for h in (0, 1)] + [208, 210])
    assert reach == Q6K
    if not staged:
        rr = np.minimum(row0 + 7, N - 1)
        first = rr * RB + lo[j] * Q6K
        last = rr * RB + hi[j] * Q6K
        assert np.all((first == 0) | (first >= 2)) and last.max() <= w_bytes
        return True
    pitch, nst, sbytes, off = pl["pitch"], pl["nstage"], pl["stage_bytes"], pl["off_stage"]
    assert pitch % 16 == 0 and off % 128 == 0 and sbytes % 16 == 0
    assert off + nst * sbytes <= pl["smem"]
    s = u % nst
    base = off + s * sbytes
    if mode == 1:
        assert ks == 1 and sbytes == 8 * RB
        start, end = row0 * RB, (row0 + nvalid) * RB
        a, b = _q6_copy(start, end, w_bytes)
        assert np.all(a % 16 == 0) and np.all((b - a) % 16 == 0) and np.all(base % 16 == 0)
        assert np.all(b <= w_bytes) and np.all(end <= w_bytes)
        assert np.all(np.maximum(b, end) - a <= sbytes)  # bulk run and plain tail inside the stage
        tx = b - a
    else:
        tx = np.zeros_like(row0)
        for lane in range(8):
            ok = lane < nvalid
            start = (row0 + lane) * RB + lo[j] * Q6K
            end = (row0 + lane) * RB + hi[j] * Q6K
            a, b = _q6_copy(start, end, w_bytes)
            dst = base + lane * pitch
            assert np.all(a[ok] % 16 == 0) and np.all((b - a)[ok] % 16 == 0) and np.all(dst % 16 == 0)
            assert np.all(b[ok] <= w_bytes) and np.all(end[ok] <= w_bytes)
            assert np.all((np.maximum(b, end) - a)[ok] <= pitch)  # run + tail inside the row's pitch
            # consumer reads: from (start & 15), less 2 when that is 2 mod 4,
            # up to the last block's reach
            assert np.all((start & 15) - np.where((start & 3) != 0, 2, 0) >= 0)
            assert np.all(((start & 15) + (hi[j] - lo[j] - 1) * Q6K + reach)[ok] <= pitch)
            tx = tx + np.where(ok, b - a, 0)
    assert tx.max() <= TX_LIMIT
    return True


Q4K_MODEL = [(6144, 2560), (4096, 2560), (1024, 2560), (2560, 4096), (9728, 2560), (2560, 9728),
             (151936, 2560)]
K_EDGES = [256, 512, 768, 1024, 2048, 2304, 2560, 4096, 4864, 8192, 9728]
N_EDGES = [1, 2, 7, 9, 33, 127, 129, 1183, 4097]


@pytest.mark.parametrize("N,K", Q4K_MODEL)
def test_q4k_model_shapes_every_candidate(N, K):
    planned = 0
    for cid, mode, ks, cps in _cands("q4k"):
        for ncols in (1, 2, 5, 8):
            planned += check_q4k(cid, mode, ks, cps, N, K, ncols)
        if (N, K) in ((9728, 2560),):
            planned += check_q4k(cid, mode, ks, cps, N, K, 1, nmat=2)
        if K == 2560:
            planned += check_q4k(cid, mode, ks, cps, N, K, 1, nmat=2 if N == 9728 else 1, xin=1)
    assert planned > 0


@pytest.mark.parametrize("K", K_EDGES)
def test_q4k_edge_shapes_every_candidate(K):
    for cid, mode, ks, cps in _cands("q4k"):
        for N in N_EDGES:
            for ncols in (1, 8):
                check_q4k(cid, mode, ks, cps, N, K, ncols)
            # the fused RMSNorm prologue (abra_q4k_mmvq_rmsnorm), MMVQ and gate/up
            check_q4k(cid, mode, ks, cps, N, K, 1, xin=1)
            check_q4k(cid, mode, ks, cps, N, K, 1, nmat=2, xin=1)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_q4k_tensor_parallel_shards(world):
    """o (K_full 4096) and down (K_full 9728) K-shards of every rank."""
    per = 8 // world
    for cid, mode, ks, cps in _cands("q4k"):
        for kfull in (4096, 9728):
            nsb_g = kfull // 256
            for r in range(world):
                k = (slice_start(nsb_g, (r + 1) * per) - slice_start(nsb_g, r * per)) * 256
                check_q4k(cid, mode, ks, cps, 2560, k, 1, shard=(nsb_g, r * per, per))
        # row-split q|k|v and gate/up with the fused prologue
        check_q4k(cid, mode, ks, cps, 6144 // world, 2560, 1, xin=1)
        check_q4k(cid, mode, ks, cps, 9728 // world, 2560, 1, nmat=2, xin=1)


@pytest.mark.parametrize("N,K", [(1024, 2560), (2560, 9728), (151936, 2560)])
def test_q6k_model_shapes_every_candidate(N, K):
    planned = 0
    for cid, mode, ks, cps in _cands("q6k"):
        for ncols in (1, 2, 3, 8):
            planned += check_q6k(cid, mode, ks, cps, N, K, ncols)
    assert planned > 0


@pytest.mark.parametrize("K", K_EDGES)
def test_q6k_edge_shapes_every_candidate(K):
    for cid, mode, ks, cps in _cands("q6k"):
        for N in N_EDGES + [64]:
            for ncols in (1, 8):
                check_q6k(cid, mode, ks, cps, N, K, ncols)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_q6k_tensor_parallel_shards(world):
    per = 8 // world
    nsb_g = 9728 // 256
    for cid, mode, ks, cps in _cands("q6k"):
        for r in range(world):
            k = (slice_start(nsb_g, (r + 1) * per) - slice_start(nsb_g, r * per)) * 256
            check_q6k(cid, mode, ks, cps, 2560, k, 1, shard=(nsb_g, r * per, per))


def test_the_product_shapes_have_plans():
    """The tuned and default candidates of every shape the decode runtime
    launches have a plan (the dispatch never refuses them)."""
    for N, K in Q4K_MODEL:
        assert plan(12, 0, N, K) is not None
    assert plan(12, 0, 9728, 2560, nmat=2, xin=1) is not None
    assert plan(12, 0, 6144, 2560, xin=1) is not None
    for N, K in [(1024, 2560), (2560, 9728), (151936, 2560)]:
        assert plan(14, 0, N, K) is not None


def test_plan_info_rejects_bad_arguments():
    out = np.zeros(8, dtype=np.int64)
    lib = _lib.lib
    assert lib.abra_mmvq_plan_info(13, 0, 64, 256, 1, 1, 0, 0, 0, 8, SMS, out.ctypes.data) == _lib.ABRA_E_INVALID
    assert lib.abra_mmvq_plan_info(12, 0, 64, 300, 1, 1, 0, 0, 0, 8, SMS, out.ctypes.data) == _lib.ABRA_E_INVALID
    assert lib.abra_mmvq_plan_info(14, 0, 64, 256, 1, 2, 0, 0, 0, 8, SMS, out.ctypes.data) == _lib.ABRA_E_INVALID
    assert lib.abra_mmvq_plan_info(12, 0, 64, 256, 2, 1, 1, 0, 0, 8, SMS, out.ctypes.data) == _lib.ABRA_E_INVALID
    assert lib.abra_mmvq_plan_info(12, 12345, 64, 256, 1, 1, 0, 0, 0, 8, SMS, out.ctypes.data) == _lib.ABRA_E_INVALID
    assert lib.abra_mmvq_plan_info(12, 0, 64, 256, 1, 1, 0, 9728, 0, 3, SMS, out.ctypes.data) == _lib.ABRA_E_INVALID
    assert lib.abra_mmvq_plan_info(12, 0, 64, 256, 1, 1, 0, 0, 0, 8, SMS, None) == _lib.ABRA_E_INVALID


def test_python_plan_info():
    import abra_b200 as A

    p = A.plan_info(9728, 2560)
    from abra_b200.q4k import PLAN_FIELDS

    assert tuple(p) == PLAN_FIELDS
    assert p["row_groups"] == 1216 and p["threads"] in (256, 288) and p["smem"] <= MAX_SMEM
    assert A.plan_info(151936, 2560, q6k=True)["row_groups"] == 18992
    assert A.plan_info(2560, 9728, ncols=8, candidate=1021, q6k=True) is None  # does not fit
    with pytest.raises(ValueError):
        A.plan_info(64, 300)


def test_random_shapes_keep_every_feed_rule():
    """Random shapes, batch widths, k-splits and K-shards (hypothesis): every
    plan the dispatch makes keeps the rules above, for both weight types."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    q4, q6 = _cands("q4k"), _cands("q6k")

    @settings(max_examples=60, deadline=None)
    @given(kind=st.sampled_from(["q4k", "q6k"]), N=st.integers(1, 40000), nsb=st.integers(1, 48),
           ncols=st.integers(1, 8), pick=st.integers(0, 10**6), nmat=st.integers(1, 2),
           xin=st.booleans(), world=st.sampled_from([1, 2, 4, 8]), rank=st.integers(0, 7))
    def run(kind, N, nsb, ncols, pick, nmat, xin, world, rank):
        shard = None
        K = nsb * 256
        if world > 1 and nsb >= 8:  # a K-shard of a row nsb superblocks wide
            per, r = 8 // world, rank % world
            lo, hi = slice_start(nsb, r * per), slice_start(nsb, (r + 1) * per)
            shard, K = (nsb, r * per, per), (hi - lo) * 256
        if kind == "q4k":
            cid, mode, ks, cps = q4[pick % len(q4)]
            fused = xin and ncols == 1 and shard is None
            check_q4k(cid, mode, ks, cps, N, K, ncols, nmat=nmat, xin=int(fused), shard=shard)
        else:
            cid, mode, ks, cps = q6[pick % len(q6)]
            check_q6k(cid, mode, ks, cps, N, K, ncols, shard=shard)

    run()
