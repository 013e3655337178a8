#!/usr/bin/env python
"""Benchmark of the Q4_K x Q8_1 MMVQ path on B200.

Default workload ("qwen3_4b_q4k_decode_tg"): greedy decode of the seeded
Qwen3-4B-shaped model, all linear weights Q4_K, after a 16-token prompt; one
step is one token (one launch of the persistent decode kernel on one GPU),
``value`` is tok/s at depth 0, ``e2e`` the same through the per-token host
call, and ``roofline`` that kernel's algorithmic bytes per launch (the
token's weights, KV rows and logits) over its measured duration against
measured HBM bandwidth.  Under torchrun the model is tensor parallel over the
ranks (kernel chain).

GEMV workload (``--workload gemv``, "qwen3_4b_decode_weight_sweep"): one step is one pass of MMVQ over
the full Qwen3-4B-shaped decode weight set, in the operators a decode step
runs: per layer the fused q|k|v projection (6144 x 2560), o (2560 x 4096),
the fused gate/up SwiGLU (2 x 9728 x 2560) and down (2560 x 9728), for 36
layers, then the tied 151936 x 2560 output -- 145 launches, 2,262,528,000
bytes of Q4_K weights (d, dmin ~ U(0.001, 0.02), 6-bit scales/mins
~ U{0..63}, nibbles ~ U{0..15}; activations N(0,1) quantized to Q8_1; seed
0), at batch 1 (``--batch``).  The weights exceed L2, so every launch reads
HBM.  The metric is algorithmic bytes / time in GB/s (weights + Q8_1
activations + fp32 outputs, the reference's formula,
bench/micro/q4k_q8_bench.cu:330-333), aggregated over ranks (each rank runs
the full set on its own GPU: weak scaling, no collective).

Also reported: every decode matrix separately (q, k, v, o, gate, up, down,
output), the reference's own kernel family on the same GPU over the
unfused sweep, the sweep end to end through the C ABI with host buffers,
the quantize-once RMSNorm -> Q8_1 block in three forms (fused_rmsnorm_block),
and the CPU baseline on all host cores: llama.cpp's CPU Q4_K path restated in
oracle/ (activations quantized to Q8_K, the Q4_K x Q8_K dot; llama.cpp itself
is not in the image), beside the restatement of vec_dot_q4_K_q8_1.

``--impl reference`` times the CPU decode itself, token by token, on all
host threads (the GEMV workload: the CPU GEMV on a bounded sample).

Run: python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS = 36
# (name, N, K, nmat): nmat 2 = fused gate/up SwiGLU over two N x K matrices
LAYER_OPS = [("qkv", 6144, 2560, 1), ("o", 2560, 4096, 1), ("gate_up", 9728, 2560, 2),
             ("down", 2560, 9728, 1)]
OUTPUT_OP = ("output", 151936, 2560, 1)
# every decode matrix of the Qwen3-4B shape, separately
DECODE_MATRICES = [("q", 4096, 2560), ("k", 1024, 2560), ("v", 1024, 2560), ("o", 2560, 4096),
                  ("gate", 9728, 2560), ("up", 9728, 2560), ("down", 2560, 9728),
                  ("output", 151936, 2560)]
WORKLOAD = "qwen3_4b_decode_weight_sweep"
L2_BYTES = 126 * 1024 * 1024


def q4k_bytes(N, K):
    return N * (K // 256) * 144


def alg_bytes(N, K, B, nmat=1):
    """Reference formula: Q4_K weights + Q8_1 activations + fp32 outputs."""
    return nmat * q4k_bytes(N, K) + B * (K // 32) * 36 + B * N * 4


def sweep_ops():
    ops = []
    for layer in range(LAYERS):
        for i, (name, N, K, nmat) in enumerate(LAYER_OPS):
            ops.append((f"{name}.{layer}", N, K, nmat, layer * 16 + 2 * i + 1))
    ops.append((OUTPUT_OP[0], OUTPUT_OP[1], OUTPUT_OP[2], 1, 1))
    return ops


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks ---
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def __enter__(self):
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.tmp.flush()

    def summary(self):
        try:
            lines = Path(self.tmp.name).read_text().strip().splitlines()
        finally:
            os.unlink(self.tmp.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ distributed ---
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend: str):
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64,
                         device="cuda" if torch.cuda.is_available() else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# --------------------------------------------------------------- CPU arm ---
def simd_level() -> int:
    import oracle as O

    return int(O.lib.orc_simd_level())


CPU_PATHS = {
    "ggml": "llama.cpp's CPU Q4_K path restated (activations in Q8_K, vec_dot_q4_K_q8_K)",
    "q8_1": "the restatement of vec_dot_q4_K_q8_1 (the GPU path's formula)",
}


# the CPU sample: this many layers of decode matrices (56.8 MB each), more
# than a host's last-level cache, so every pass streams from DRAM as a token does
CPU_SAMPLE_LAYERS = 8
CPU_SAMPLE = (f"{CPU_SAMPLE_LAYERS} layers of decode matrices (q|k|v, o, gate, up, down; "
              f"{CPU_SAMPLE_LAYERS * 56.77:.0f} MB, more than the host's last-level cache)")


_CPU_SAMPLES: dict = {}


def cpu_sample_rate(batch: int, budget_s: float, seed: int = 0, path: str = "ggml"):
    """A CPU Q4_K GEMV (OpenMP, all host cores; integer sub-block dots on the
    host's AVX-512 VNNI or AVX2 when present) on a sample of the workload:
    CPU_SAMPLE, every matrix once per pass, passes repeated until
    ``budget_s`` seconds elapse.  ``path`` "ggml": llama.cpp's CPU path restated
    (activations quantized to Q8_K, the Q4_K x Q8_K dot), the CPU path the
    reference runs on the host; "q8_1": the restatement of
    vec_dot_q4_K_q8_1.  Returns GB/s by the reference's byte formula."""
    import oracle as O

    threads = os.cpu_count() or 1
    quant, gemv = (O.quantize_q8_K, O.gemv_q8k) if path == "ggml" else (O.quantize_q8_1, O.gemv)
    key = (batch, seed, path)
    if key not in _CPU_SAMPLES:  # built once per process: the passes time the GEMV alone
        xs = {K: quant(O.gen_normal_f32((batch, K), seed + 1000 + K)) for K in (2560, 4096, 9728)}
        sample = []
        for layer in range(CPU_SAMPLE_LAYERS):
            for name, N, K, nmat in LAYER_OPS:
                for m in range(nmat):
                    w = O.gen_q4k(N, K, seed, 16 * layer + 2 * len(sample) + m + 1)
                    sample.append((w, xs[K], N, K))
        _CPU_SAMPLES.clear()  # one sample held at a time (454 MB)
        _CPU_SAMPLES[key] = sample
    sample = _CPU_SAMPLES[key]
    nbytes = sum(alg_bytes(n, k, batch) for _, _, n, k in sample)
    gemv(sample[0][0], sample[0][1], sample[0][3], threads)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        for w, xq, n, k in sample:
            gemv(w, xq, k, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return reps * nbytes / el / 1e9, threads, reps, el


CPU_DECODE = ("the full 36-layer Qwen3-4B-shaped decode (seeded weights, the GPU model's), one "
              "token per step after a {prompt}-token prompt, on llama.cpp's CPU path restated in "
              "oracle/model_oracle.c (every Q4_K GEMV on Q8_K activations, ggml's "
              "vec_dot_q4_K_q8_K; integer dots at SIMD level {simd}: 0 scalar, 1 AVX2, "
              "2 AVX-512 VNNI), OpenMP on all host threads")


class CpuDecoder:
    """The CPU decode the reference runs when its model is on the host,
    token by token (orc_model_step_cpu), on all host threads."""

    def __init__(self, max_tokens: int, seed: int = 0):
        import oracle as O

        self.m = O.OrcModel(max_ctx=PROMPT + max_tokens + 1, seed=seed)
        self.prompt = np.random.default_rng(seed).integers(0, self.m.cfg.vocab, PROMPT).astype(np.int32)
        self.pos, self.tok = 0, int(self.prompt[0])
        self.threads = self.m.threads

    def step(self) -> float:
        """One token; returns its wall time in ms."""
        t0 = time.perf_counter()
        pick = self.m.step_cpu(self.tok, self.pos)
        el = (time.perf_counter() - t0) * 1e3
        self.pos += 1
        self.tok = int(self.prompt[self.pos]) if self.pos < PROMPT else pick
        return el

    def close(self):
        self.m.close()


def cpu_decode_rate(warmup: int, max_tokens: int, budget_s: float):
    """Tokens per second of the CPU decode: ``warmup`` untimed tokens, then
    tokens until ``max_tokens`` or ``budget_s`` seconds."""
    d = CpuDecoder(warmup + max_tokens)
    for _ in range(warmup):
        d.step()
    ms = []
    while len(ms) < max_tokens and sum(ms) < budget_s * 1e3:
        ms.append(d.step())
    d.close()
    return 1000.0 * len(ms) / sum(ms), d.threads, ms


# --------------------------------------------------------------- GPU arm ---
def launch_ops(plan, ncols: int, pdl: bool, stream=None):
    """Launch (w, w2, x, y, N, K, nmat) MMVQs through the C ABI with the least
    host overhead: the stream is resolved once, the symbols are pre-bound."""
    from abra_b200 import _lib
    from abra_b200.q4k import stream_handle

    f1 = _lib.lib.abra_q4k_mmvq_ex
    f2 = _lib.lib.abra_q4k_mmvq_swiglu
    st = stream_handle(stream)
    flags = _lib.ABRA_MMVQ_PDL if pdl else 0
    for w, w2, x, y, N, K, nmat in plan:
        if nmat == 1:
            rc = f1(w, x, y, N, K, ncols, N, 0, flags, st)
        else:
            rc = f2(w, w2, x, y, N, K, ncols, N, 0, flags, st)
        if rc:
            _lib.check(rc, "abra_q4k_mmvq")


def tc_ks(N: int) -> int:
    """k-parts of the batch-32 tensor-core MMVQ: enough CTAs for 148 SMs."""
    return 1 if N >= 16384 else 2 if N >= 4096 else 8


def launch_ops_tc(plan, ws_ptr: int, pdl: bool, stream=None):
    """The same decode weight set at batch 32 through the tcgen05 MMVQ
    (abra_q4k_mmvq_tc); a fused gate/up op is its two matrices."""
    from abra_b200 import _lib
    from abra_b200.q4k import stream_handle

    f = _lib.lib.abra_q4k_mmvq_tc
    st = stream_handle(stream)
    flags = _lib.ABRA_MMVQ_PDL if pdl else 0
    for w, w2, x, y, N, K, nmat in plan:
        for wm in ((w,) if nmat == 1 else (w, w2)):
            rc = f(wm, x, y, N, K, 32, N, tc_ks(N), ws_ptr, flags, st)
            if rc:
                _lib.check(rc, "abra_q4k_mmvq_tc")


class Sweep:
    def __init__(self, dev, batch: int, seed: int = 0):
        import torch

        import abra_b200 as A
        import oracle as O

        self.A, self.torch, self.dev, self.B = A, torch, dev, batch
        self.ops = sweep_ops()
        self.w = {}
        for name, N, K, nmat, tid in self.ops:
            nb = N * K // 256
            bufs = []
            for m in range(nmat):
                buf = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
                A.gen_q4k(buf, nb, seed, tid + m)
                bufs.append(buf)
            self.w[name] = bufs
        self.Ks = sorted({K for _, _, K, _, _ in self.ops})
        self.xq = {}
        for K in self.Ks:
            x = O.gen_normal_f32((batch, K), seed + 1000 + K)
            xq = torch.empty(batch * (K // 32) * 36, dtype=torch.uint8, device=dev)
            A.launch_quantize_f32_to_q8_1(torch.from_numpy(x.reshape(-1)).to(dev), xq, K,
                                          ncols=batch)
            self.xq[K] = xq
        maxn = max(N for _, N, _, _, _ in self.ops)
        self.y = torch.empty(batch * maxn, dtype=torch.float32, device=dev)
        self.bytes = sum(alg_bytes(N, K, batch, nmat) for _, N, K, nmat, _ in self.ops)
        self.weight_bytes = sum(nmat * q4k_bytes(N, K) for _, N, K, nmat, _ in self.ops)
        self.launches = len(self.ops)
        self.plan = []
        for name, N, K, nmat, _ in self.ops:
            b = self.w[name]
            self.plan.append((b[0].data_ptr(), b[1].data_ptr() if nmat == 2 else 0,
                              self.xq[K].data_ptr(), self.y.data_ptr(), N, K, nmat))
        torch.cuda.synchronize()

    def step(self, pdl=True):
        """One pass over the decode weight set, launched through the C ABI."""
        launch_ops(self.plan, self.B, pdl)

    def capture(self, fn=None):
        """Capture ``fn`` (default: one step) into a CUDA graph."""
        torch = self.torch
        fn = fn or self.step
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        return g

    def timed(self, steps: int, fn=None):
        torch = self.torch
        fn = fn or self.step
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / steps  # ms per step


class E2E:
    """The same sweep through the public API with host buffers: per step one
    H2D copy of every operator input (fp32, pinned), their quantization on
    the device, the MMVQs, and one D2H copy of every output."""

    def __init__(self, sw: Sweep):
        torch = sw.torch
        self.sw = sw
        B = sw.B
        total_x = sum(K for _, _, K, _, _ in sw.ops) * B
        self.h_x = torch.empty(total_x, dtype=torch.float32).pin_memory()
        self.h_x.numpy()[:] = np.random.default_rng(7).standard_normal(total_x, dtype=np.float32)
        self.d_x = torch.empty(total_x, dtype=torch.float32, device=sw.dev)
        self.d_q = torch.empty(sum(K // 32 * 36 for _, _, K, _, _ in sw.ops) * B,
                               dtype=torch.uint8, device=sw.dev)
        total_y = sum(N for _, N, _, _, _ in sw.ops) * B
        self.d_y = torch.empty(total_y, dtype=torch.float32, device=sw.dev)
        self.h_y = torch.empty(total_y, dtype=torch.float32).pin_memory()
        self.h2d, self.d2h = total_x * 4, total_y * 4
        xb, qb, yb = self.d_x.data_ptr(), self.d_q.data_ptr(), self.d_y.data_ptr()
        self.qplan, self.mplan = [], []
        xo = qo = yo = 0
        for name, N, K, nmat, _ in sw.ops:
            w = sw.w[name]
            self.qplan.append((xb + xo * 4, qb + qo, K))
            self.mplan.append((w[0].data_ptr(), w[1].data_ptr() if nmat == 2 else 0, qb + qo,
                               yb + yo * 4, N, K, nmat))
            xo += K * B
            qo += K // 32 * 36 * B
            yo += N * B

    def step(self):
        from abra_b200 import _lib
        from abra_b200.q4k import stream_handle

        B = self.sw.B
        st = stream_handle(None)
        self.d_x.copy_(self.h_x, non_blocking=True)
        fq = _lib.lib.abra_quantize_q8_1
        for x, q, K in self.qplan:
            rc = fq(x, q, K, B, st)
            if rc:
                _lib.check(rc, "abra_quantize_q8_1")
        launch_ops(self.mplan, B, pdl=False, stream=st)
        self.h_y.copy_(self.d_y, non_blocking=True)


def shape_table(sw: Sweep, reps: int = 3):
    """Each decode matrix (and the fused operators) alone: one CUDA graph of
    back-to-back launches over >= 4 x L2 (at least 8) distinct weight copies,
    best of ``reps`` replays."""
    torch, A = sw.torch, sw.A
    out = {}
    shapes = [(n, N, K, 1) for n, N, K in DECODE_MATRICES] + [
        ("qkv_fused", 6144, 2560, 1), ("gate_up_swiglu", 9728, 2560, 2)]
    for name, N, K, nmat in shapes:
        per = nmat * q4k_bytes(N, K)
        copies = max(8, -(-4 * L2_BYTES // per))
        nb = N * K // 256
        bufs = []
        for i in range(copies * nmat):
            t = torch.empty(nb * 144, dtype=torch.uint8, device=sw.dev)
            A.gen_q4k(t, nb, 0, 9000 + i)
            bufs.append(t)
        plan = [(bufs[i * nmat].data_ptr(), bufs[i * nmat + 1].data_ptr() if nmat == 2 else 0,
                 sw.xq[K].data_ptr(), sw.y.data_ptr(), N, K, nmat) for i in range(copies)]
        g = sw.capture(lambda: launch_ops(plan, sw.B, True))
        ms = min(sw.timed(1, g.replay) for _ in range(reps))
        us = ms * 1e3 / copies
        out[name] = {"N": N, "K": K, "nmat": nmat, "us": round(us, 3),
                     "GBps": round(alg_bytes(N, K, sw.B, nmat) / (us * 1e-6) / 1e9, 1),
                     "copies": copies,
                     "candidate": A.get_autotuned_candidate_for_shape(N, K, ncols=sw.B, nmat=nmat)}
        del g, bufs, plan
        torch.cuda.empty_cache()
    return out


def packed_table(sw: Sweep, reps: int = 3):
    """The reference's 148-byte prepack against the plain 144-byte layout on
    config 0 (gate 9728x2560) and the tied output: the same lane-mapped MMVQ
    (2 CTAs per SM, 8-row units) over each, one CUDA graph of back-to-back
    launches over >= 4 x L2 of weight copies, best of ``reps``."""
    torch, A = sw.torch, sw.A
    out = {}
    for name, N, K in (("gate", 9728, 2560), ("output", 151936, 2560)):
        nb = N * K // 256
        copies = max(8, -(-4 * L2_BYTES // (nb * 144)))
        plain, packed = [], []
        for i in range(copies):
            t = torch.empty(nb * 144, dtype=torch.uint8, device=sw.dev)
            A.gen_q4k(t, nb, 0, 9500 + i)
            p = torch.empty(nb * 148, dtype=torch.uint8, device=sw.dev)
            A.pack_q4k(t, p, nb)
            plain.append(t)
            packed.append(p)
        torch.cuda.synchronize()
        row = {"N": N, "K": K, "copies": copies}
        for form, bufs, nbytes in (("q4k_144", plain, 144), ("packed_148", packed, 148)):
            if form == "q4k_144":
                run = lambda: [A.mmvq(b, sw.xq[K], sw.y, N, K, candidate=4082, pdl=True) for b in bufs]
            else:
                run = lambda: [A.mmvq_packed(b, sw.xq[K], sw.y, N, K, pdl=True) for b in bufs]
            g = sw.capture(run)
            ms = min(sw.timed(1, g.replay) for _ in range(reps))
            us = ms * 1e3 / copies
            row[form] = {"us": round(us, 3), "GBps": round((nb * nbytes + K // 32 * 36 + N * 4) / (us * 1e-6) / 1e9, 1)}
            del g
        out[name] = row
        del plain, packed
        torch.cuda.empty_cache()
    return out


Q6K_SHAPES = [("attn_v", 1024, 2560), ("ffn_down", 2560, 9728), ("output", 151936, 2560)]


def shape_table_q6k(sw: Sweep, reps: int = 3):
    """The real model's Q6_K tensors (abra_q6k_mmvq, tuned candidate) alone,
    timed like shape_table: one graph over >= 4 x L2 of distinct weight copies."""
    torch, A = sw.torch, sw.A
    from abra_b200 import _lib
    from abra_b200.q4k import stream_handle

    out = {}
    for name, N, K in Q6K_SHAPES:
        per = N * K // 256 * 210
        copies = max(8, -(-4 * L2_BYTES // per))
        nb = N * K // 256
        bufs = []
        for i in range(copies):
            t = torch.empty(nb * 210, dtype=torch.uint8, device=sw.dev)
            A.gen_q6k(t, nb, 0, 9500 + i)
            bufs.append(t)
        xq, y = sw.xq[K].data_ptr(), sw.y.data_ptr()
        fn = _lib.lib.abra_q6k_mmvq_ex

        def run():
            st = stream_handle(None)
            for b in bufs:
                rc = fn(b.data_ptr(), xq, y, N, K, 1, N, 0, _lib.ABRA_MMVQ_PDL, st)
                if rc:
                    _lib.check(rc, "abra_q6k_mmvq_ex")

        g = sw.capture(run)
        ms = min(sw.timed(1, g.replay) for _ in range(reps))
        us = ms * 1e3 / copies
        alg = per + K // 32 * 36 + N * 4
        out[name] = {"N": N, "K": K, "us": round(us, 3), "GBps": round(alg / (us * 1e-6) / 1e9, 1),
                     "copies": copies, "candidate": A.q6k_tune_get(N, K, 1)}
        del g, bufs
        torch.cuda.empty_cache()
    return out


def ref_gpu_sweep(sw: Sweep, steps: int):
    """The reference's own kernel family (oracle/_ref) on the same weights,
    unfused (q, k, v, gate, up as separate launches -- it has no fused forms),
    batch 1, with the reference's dispatch rule
    (get_autotuned_candidate_for_shape), captured in a CUDA graph."""
    import oracle as O

    try:
        ref = O.RefFamily()
    except FileNotFoundError:
        return None
    if sw.B != 1:
        return None
    plan = []
    for name, N, K, nmat, _ in sw.ops:
        w = sw.w[name]
        if name.startswith("qkv"):
            base = w[0].data_ptr()
            for rows, off in ((4096, 0), (1024, 4096), (1024, 5120)):
                plan.append((base + off * q4k_bytes(1, K), sw.xq[K].data_ptr(), rows, K))
        else:
            for m in range(nmat):
                plan.append((w[m].data_ptr(), sw.xq[K].data_ptr(), N, K))
    plan = [(wp, xp, N, K, ref.autotuned_candidate(N, K, 61) or 204) for wp, xp, N, K in plan]
    yp = sw.y.data_ptr()

    def run():
        stream = sw.torch.cuda.current_stream().cuda_stream
        for wp, xp, N, K, cid in plan:
            ref.launch_candidate(cid, wp, xp, yp, N, K, stream)

    g = sw.capture(run)
    ms = sw.timed(steps, g.replay)
    return {"GBps": round(sw.bytes / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4),
            "launches_per_step": len(plan),
            "dispatch": "reference get_autotuned_candidate_for_shape(N, K, 61)"}


def run_case(a):
    """Profiling case: one operator, ``--copies`` weight copies, eager launches
    (warm-up passes then timed passes), for ncu captures."""
    import torch

    import abra_b200 as A
    import oracle as O

    table = {n: (N, K, 1) for n, N, K in DECODE_MATRICES}
    table.update({"qkv": (6144, 2560, 1), "gate_up": (9728, 2560, 2)})
    if a.case.startswith("q6k_"):
        return run_case_q6k(a)
    if a.case == "tc_b32_16384":
        return run_case_tc(a)
    if a.case in ("decode_token", "decode_chain"):
        return run_case_decode(a)
    if a.case == "fused_rmsnorm_block":
        torch.cuda.set_device(0)
        print(json.dumps({"case": a.case, **fused_rmsnorm_block(torch, a.steps, copies=max(8, a.copies))}),
              flush=True)
        return 0
    N, K, nmat = table[a.case]
    dev = torch.device("cuda:0")
    nb = N * K // 256
    bufs = []
    for i in range(a.copies * nmat):
        t = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
        A.gen_q4k(t, nb, 0, 500 + i)
        bufs.append(t)
    xq = torch.empty(a.batch * (K // 32) * 36, dtype=torch.uint8, device=dev)
    A.launch_quantize_f32_to_q8_1(
        torch.from_numpy(O.gen_normal_f32((a.batch, K), 1).reshape(-1)).to(dev), xq, K,
        ncols=a.batch)
    y = torch.empty(a.batch * N, dtype=torch.float32, device=dev)
    plan = [(bufs[i * nmat].data_ptr(), bufs[i * nmat + 1].data_ptr() if nmat == 2 else 0,
             xq.data_ptr(), y.data_ptr(), N, K, nmat) for i in range(a.copies)]
    for _ in range(a.warmup):
        launch_ops(plan, a.batch, True)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        launch_ops(plan, a.batch, True)
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / (a.steps * len(plan))
    print(json.dumps({"case": a.case, "N": N, "K": K, "nmat": nmat, "batch": a.batch,
                      "copies": a.copies, "us_per_launch_eager": round(us, 3),
                      "GBps_eager": round(alg_bytes(N, K, a.batch, nmat) / (us * 1e-6) / 1e9, 1),
                      "candidate": A.get_autotuned_candidate_for_shape(N, K, ncols=a.batch,
                                                                       nmat=nmat),
                      "device_error": A.device_error()}), flush=True)
    return 0


def run_case_q6k(a):
    """Profiling case for a Q6_K tensor of the real model (q6k_<name> of
    Q6K_SHAPES): ``--copies`` weight copies, eager tuned launches."""
    import torch

    import abra_b200 as A
    import oracle as O

    N, K = {f"q6k_{n}": (N, K) for n, N, K in Q6K_SHAPES}[a.case]
    dev = torch.device("cuda:0")
    nb = N * K // 256
    bufs = []
    for i in range(a.copies):
        t = torch.empty(nb * 210, dtype=torch.uint8, device=dev)
        A.gen_q6k(t, nb, 0, 700 + i)
        bufs.append(t)
    xq = torch.empty(a.batch * (K // 32) * 36, dtype=torch.uint8, device=dev)
    A.launch_quantize_f32_to_q8_1(
        torch.from_numpy(O.gen_normal_f32((a.batch, K), 1).reshape(-1)).to(dev), xq, K,
        ncols=a.batch)
    y = torch.empty(a.batch * N, dtype=torch.float32, device=dev)

    def run():
        for b in bufs:
            A.mmvq_q6k(b, xq, y, N, K, ncols=a.batch, pdl=True)

    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        run()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / (a.steps * len(bufs))
    alg = N * K // 256 * 210 + a.batch * (K // 32 * 36 + N * 4)
    print(json.dumps({"case": a.case, "N": N, "K": K, "batch": a.batch, "copies": a.copies,
                      "us_per_launch_eager": round(us, 3),
                      "GBps_eager": round(alg / (us * 1e-6) / 1e9, 1),
                      "candidate": A.q6k_tune_get(N, K, a.batch),
                      "device_error": A.device_error()}), flush=True)
    return 0


def run_case_decode(a):
    """Profiling case for the decode step at ``--depth``: the full-size
    Qwen3-4B-shaped model (2.3 GB of weights), the prompt and depth prefix fed
    token by token, ``--warmup`` then ``--steps`` tokens; decode_token is the
    persistent kernel (one launch per token), decode_chain the per-operation
    kernel chain (attention, QK-norm and merge kernels included)."""
    import torch

    from abra_b200.model import KERNEL_CHAIN

    torch.cuda.set_device(0)
    flags = KERNEL_CHAIN if a.case == "decode_chain" else 0
    r = decode_depth(torch, a.depth, a.warmup, a.steps, streaming=False, flags=flags,
                     n_layers=a.layers)
    print(json.dumps({"case": a.case, "layers": a.layers, **r}), flush=True)
    return 0


TC_CASE_SHAPE = (16384, 2560)


def run_case_tc(a):
    """Profiling case for the batch-32 tensor-core MMVQ: ``--copies`` (at
    least 3) copies of a 16384 x 2560 Q4_K matrix (23.6 MB each), 32 N(0,1)
    columns quantized to Q8_1, mmvq_tc (ks 1) on each copy, eager launches."""
    import torch

    import abra_b200 as A
    import oracle as O

    N, K = TC_CASE_SHAPE
    dev = torch.device("cuda:0")
    nb = N * K // 256
    bufs = []
    for i in range(max(3, a.copies)):
        t = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
        A.gen_q4k(t, nb, 0, 40 + i)
        bufs.append(t)
    xq = torch.empty(32 * (K // 32) * 36, dtype=torch.uint8, device=dev)
    A.launch_quantize_f32_to_q8_1(
        torch.from_numpy(O.gen_normal_f32((32, K), 1).reshape(-1)).to(dev), xq, K, ncols=32)
    y = torch.empty(32 * N, dtype=torch.float32, device=dev)

    def run():
        for b in bufs:
            A.mmvq_tc(b, xq, y, N, K, ks=1)

    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        run()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / (a.steps * len(bufs))
    alg = nb * 144 + 32 * (K // 32 * 36 + N * 4)
    print(json.dumps({"case": a.case, "N": N, "K": K, "batch": 32, "copies": len(bufs),
                      "us_per_launch_eager": round(us, 3),
                      "GBps_eager": round(alg / (us * 1e-6) / 1e9, 1),
                      "device_error": A.device_error()}), flush=True)
    return 0


DECODE_WORKLOAD = "qwen3_4b_q4k_decode_tg"
PROMPT = 16
# kernels per token: embed; per layer q|k|v (fused RMSNorm), QK-norm/RoPE/KV,
# attention, merge+Q8_1, o, gate/up (fused RMSNorm), Q8_1, down; output, argmax
LAUNCHES_PER_TOKEN = 1 + 36 * 8 + 2
# fp16 K and V of every layer and kv head, per position of context
KV_BYTES_PER_POS = 36 * 2 * 8 * 128 * 2


def decode_depth(torch, depth: int, warmup: int, steps: int, streaming: bool, seed: int = 0,
                 dist=None, flags: int = 0, n_layers: int = 36):
    """One decode measurement: a model sized for the prompt + depth prefix +
    warm-up + timed tokens; the prefix is fed untimed (token by token through
    the same step), then ``warmup`` untimed tokens, then ``steps`` timed
    tokens (one CUDA graph replay each), timed with CUDA events on the model's
    stream.  With ``streaming`` the timed tokens go through the per-token
    host round trip of abra_model_decode_streaming instead.  Under torchrun
    (world > 1) every rank holds its tensor-parallel shard of one model."""
    from abra_b200.model import DecodeModel

    n_prompt = PROMPT + depth
    rank, world = (dist.rank, dist.world) if dist else (0, 1)
    m = DecodeModel(rank=rank, world=world, max_ctx=n_prompt + warmup + steps, seed=seed,
                    flags=flags, n_layers=n_layers)
    prompt = np.random.default_rng(seed + depth).integers(0, m.cfg.vocab, n_prompt).astype(np.int32)
    m.reset(prompt)
    m.step(n_prompt - 1 + warmup)
    m.sync()
    if dist:
        dist.barrier()
    st = torch.cuda.ExternalStream(m.stream)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(st)
    if streaming:
        m.decode_streaming(steps)
    else:
        m.step(steps)
    e.record(st)
    e.synchronize()
    ms = s.elapsed_time(e) / steps
    info = m.info()
    persistent = m.persistent
    toks = m.tokens(n_prompt + warmup + steps)[n_prompt:]
    if dist:
        dist.barrier()  # peers push into this rank's arena until they finish
    m.close()
    return {"depth": depth, "ms_per_token": round(ms, 4), "tok_s": round(1000.0 / ms, 2),
            "weight_bytes": info["weight_bytes"],
            "kv_read_bytes_per_token": KV_BYTES_PER_POS * (n_prompt + warmup + steps // 2),
            "step": "persistent decode kernel" if persistent else "kernel chain",
            "tokens_head": toks[:4].tolist()}


def decode_samples(torch, warmup: int, steps: int, seed: int = 0):
    """Per-token decode times at depth 0 (a second pass after the headline
    measurement): one CUDA event pair per token on the model's stream,
    giving the median / min / max / spread / stddev and the raw samples the
    reference's methodology reports (docs/benchmark-methodology.md:41-62)."""
    from abra_b200.model import DecodeModel

    m = DecodeModel(max_ctx=PROMPT + warmup + steps + 1, seed=seed)
    prompt = np.random.default_rng(seed).integers(0, m.cfg.vocab, PROMPT).astype(np.int32)
    m.reset(prompt)
    m.step(PROMPT - 1 + warmup)
    m.sync()
    st = torch.cuda.ExternalStream(m.stream)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record(st)
    for i in range(steps):
        m.step(1)
        ev[i + 1].record(st)
    ev[-1].synchronize()
    ms = np.array([ev[i].elapsed_time(ev[i + 1]) for i in range(steps)])
    m.close()
    return {"unit": "ms/token", "n": steps, "median": round(float(np.median(ms)), 4),
            "min": round(float(ms.min()), 4), "max": round(float(ms.max()), 4),
            "spread": round(float(ms.max() - ms.min()), 4), "stddev": round(float(ms.std()), 4)}


def prompt_processing(torch, n: int = 512, reps: int = 3, seed: int = 0):
    """pp<n>: an n+1-token prompt: n tokens through abra_model_prefill (the
    tensor-core tiles) and the last through one decode step, which picks the
    first generated token; CUDA events on the model's stream around both,
    best of ``reps`` after one untimed pass (graph capture)."""
    from abra_b200.model import DecodeModel

    m = DecodeModel(max_ctx=n + 8, seed=seed)
    prompt = np.random.default_rng(seed + 1).integers(0, m.cfg.vocab, n + 1).astype(np.int32)
    st = torch.cuda.ExternalStream(m.stream)
    best = None
    for r in range(reps + 1):
        m.reset(prompt)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        m.prefill(n)
        m.step(1)
        e.record(st)
        e.synchronize()
        if r > 0:
            ms = s.elapsed_time(e)
            best = ms if best is None else min(best, ms)
    first = int(m.tokens(n + 2)[n + 1])
    m.close()
    return {"prompt_tokens": n + 1, "ms": round(best, 3), "tok_s": round((n + 1) * 1000.0 / best, 1),
            "first_token": first,
            "path": f"abra_model_prefill({n}): 32-column tcgen05 GEMV tiles, chunks of 256; "
                    "then one decode step"}


def lookup_verification(torch, n_prompt: int = 16, blocks: int = 12, seed: int = 0):
    """Prompt-lookup speculation's verification pass (abra_model_verify):
    per block 1 current + 15 drafted tokens, the drafts being the true greedy
    continuation (every draft accepted: the best case of the reference's
    lookup_decode loop), host round trip included; against plain decode
    steps.  The break-even point is decode_ms -> verify_ms / decode_ms
    accepted tokens per block."""
    from abra_b200.model import DecodeModel

    n_gen = blocks * 16 + 8
    m = DecodeModel(max_ctx=n_prompt + n_gen + 40, seed=seed)
    prompt = np.random.default_rng(seed + 2).integers(0, m.cfg.vocab, n_prompt).astype(np.int32)
    greedy = m.generate(prompt, n_gen)
    st = torch.cuda.ExternalStream(m.stream)
    m.reset(prompt)
    m.step(n_prompt)  # current = greedy[0]
    m.verify(greedy[1:16])  # warm-up: graph capture
    i = 16
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(st)
    kept_total = 0
    for _ in range(blocks - 1):
        kept, _ = m.verify(greedy[i + 1:i + 16])
        kept_total += kept
        i += kept
    e.record(st)
    e.synchronize()
    ms = s.elapsed_time(e) / (blocks - 1)
    ok = bool(np.array_equal(m.tokens(n_prompt + i + 1)[n_prompt:n_prompt + i + 1], greedy[:i + 1]))
    m.close()
    return {"verify_ms": round(ms, 3), "tokens_per_verify": kept_total / (blocks - 1),
            "tok_s_all_accepted": round(kept_total / (blocks - 1) * 1000.0 / ms, 1),
            "tokens_equal_greedy": ok,
            "path": "abra_model_verify: 32-column tcgen05 pass with logits, host commit"}


def _span(t, off: int, nbytes: int) -> int:
    """Device address of bytes [off, off + nbytes) of tensor t, checked to lie
    inside it (every pointer handed to a kernel below goes through here)."""
    size = t.numel() * t.element_size()
    assert 0 <= off and off + nbytes <= size, (off, nbytes, size)
    return t.data_ptr() + off


FB_K, FB_HQ, FB_HKV, FB_F = 2560, 4096, 1024, 9728
FB_NQKV = FB_HQ + 2 * FB_HKV
FB_EPS = 1e-6


def fused_block_buffers(torch, dev, copies: int) -> dict:
    """Buffers of the quantize-once block (weights uninitialised)."""
    K, NQKV, F = FB_K, FB_NQKV, FB_F
    q8 = K // 32 * 36

    def u8(n):
        return torch.empty(n, dtype=torch.uint8, device=dev)

    def f32(n):
        return torch.empty(n, dtype=torch.float32, device=dev)

    return {"wqkv": [u8(NQKV * (K // 256) * 144) for _ in range(copies)],
            "wg": [u8(F * (K // 256) * 144) for _ in range(copies)],
            "wu": [u8(F * (K // 256) * 144) for _ in range(copies)],
            "x": f32(K), "g": f32(K), "xn": f32(K),
            "xq": u8(6 * q8),  # [0]: the shared copy; [1..5]: one per consumer
            "y_sep": f32(NQKV + 2 * F), "y_once": f32(NQKV + F), "y_fused": f32(NQKV + F)}


def fused_block_forms(A, b: dict) -> dict:
    """The three forms of the block over buffers ``b``: name -> (fn(copy),
    launches, Q8_1 bytes written, Q8_1 bytes read, fp32 activation bytes).
    Every pointer goes through _span, checked against its tensor."""
    K, HQ, HKV, F, NQKV, eps = FB_K, FB_HQ, FB_HKV, FB_F, FB_NQKV, FB_EPS
    q8 = K // 32 * 36
    wq_bytes, wf_bytes = A.q4k_nbytes(NQKV, K), A.q4k_nbytes(F, K)
    x, g, xn, xq = b["x"], b["g"], b["xn"], b["xq"]
    rows = ((0, HQ), (HQ, HKV), (HQ + HKV, HKV))  # q, k, v: row ranges of q|k|v

    def per_consumer(r):
        A.rmsnorm_quantize_q8_1(_span(x, 0, K * 4), _span(g, 0, K * 4), eps, _span(xq, 0, q8), K,
                                d_xn_out=_span(xn, 0, K * 4))
        for i in range(5):
            A.launch_quantize_f32_to_q8_1(_span(xn, 0, K * 4), _span(xq, (i + 1) * q8, q8), K)
        yo = 0
        for i, (r0, n) in enumerate(rows):
            A.mmvq(_span(b["wqkv"][r], A.q4k_nbytes(r0, K), A.q4k_nbytes(n, K)),
                   _span(xq, (i + 1) * q8, q8), _span(b["y_sep"], yo * 4, n * 4), n, K)
            yo += n
        for i, w in ((3, b["wg"][r]), (4, b["wu"][r])):
            A.mmvq(_span(w, 0, wf_bytes), _span(xq, (i + 1) * q8, q8),
                   _span(b["y_sep"], yo * 4, F * 4), F, K)
            yo += F

    def quantize_once(r):
        A.rmsnorm_quantize_q8_1(_span(x, 0, K * 4), _span(g, 0, K * 4), eps, _span(xq, 0, q8), K)
        A.mmvq(_span(b["wqkv"][r], 0, wq_bytes), _span(xq, 0, q8),
               _span(b["y_once"], 0, NQKV * 4), NQKV, K)
        A.mmvq_swiglu(_span(b["wg"][r], 0, wf_bytes), _span(b["wu"][r], 0, wf_bytes),
                      _span(xq, 0, q8), _span(b["y_once"], NQKV * 4, F * 4), F, K)

    def fused_prologue(r):
        A.mmvq_rmsnorm(_span(b["wqkv"][r], 0, wq_bytes), _span(x, 0, K * 4), _span(g, 0, K * 4),
                       eps, _span(b["y_fused"], 0, NQKV * 4), NQKV, K)
        A.mmvq_rmsnorm(_span(b["wg"][r], 0, wf_bytes), _span(x, 0, K * 4), _span(g, 0, K * 4),
                       eps, _span(b["y_fused"], NQKV * 4, F * 4), F, K,
                       d_w_up=_span(b["wu"][r], 0, wf_bytes))

    act = 2 * K * 4  # x and the norm weight
    return {
        # the norm's fp32 output written once and read by 5 quantizations
        "per_consumer": (per_consumer, 11, 6 * q8, 5 * q8, act + K * 4 + 5 * K * 4),
        "quantize_once": (quantize_once, 3, q8, 2 * q8, act),
        "fused_prologue": (fused_prologue, 2, 0, 0, act),
    }


def fused_rmsnorm_block(torch, steps: int, copies: int = 8, seed: int = 0):
    """The quantize-once block on hidden 2560: x ~ N(0,1) fp32 and a norm
    weight ~ U(0.8, 1.2) (eps 1e-6); the normalized, Q8_1-quantized
    activation feeds q (4096), k, v (1024 each), gate and up (9728 each).
    Three forms of the same block, each as a CUDA graph over ``copies``
    copies of the layer's weights (36.9 MB a copy, 295 MB in all: every block
    reads its weights from HBM):

    * per_consumer -- RMSNorm to fp32, then one Q8_1 quantization and one
      MMVQ per consumer (the reference without its reuse cache: 5 Q8_1
      writes and 5 reads);
    * quantize_once -- abra_rmsnorm_quantize_q8_1 writes one Q8_1 copy that
      the fused q|k|v MMVQ and the gate/up SwiGLU MMVQ read (the reference's
      Q8 reuse, kernels/q4k/abra-q8-reuse.cuh:3-71);
    * fused_prologue -- abra_q4k_mmvq_rmsnorm: each CTA of the two MMVQs
      normalizes and quantizes in shared memory; no Q8_1 in HBM (the decode
      runtime's form).

    Reports time per block, launches, Q8_1 bytes through HBM and the bytes
    saved, and whether the three forms give the same outputs."""
    import abra_b200 as A
    import oracle as O

    K, NQKV, F = FB_K, FB_NQKV, FB_F
    dev = torch.device("cuda", torch.cuda.current_device())
    b = fused_block_buffers(torch, dev, copies)
    for r in range(copies):
        for name, tid in (("wqkv", 900), ("wg", 901), ("wu", 902)):
            t = b[name][r]
            A.gen_q4k(t, t.numel() // 144, seed, tid + 10 * r)
    b["x"].copy_(torch.from_numpy(O.gen_normal_f32((1, K), seed + 77).reshape(-1)))
    b["g"].copy_(torch.from_numpy(O.gen_uniform_f32(K, seed, 78, 0.4, 0.8)))  # U(0.8, 1.2)
    out = {"workload": "fused_rmsnorm_q8_1_block_2560", "copies": copies,
           "consumers": "q 4096, k 1024, v 1024, gate 9728, up 9728 (x 2560)", "forms": {}}
    for name, (fn, launches, qw, qr, fp32_bytes) in fused_block_forms(A, b).items():
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for r in range(copies):
                fn(r)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for r in range(copies):
                fn(r)
        for _ in range(3):
            graph.replay()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(5, steps // 8)
        torch.cuda.synchronize()
        s.record()
        for _ in range(n):
            graph.replay()
        e.record()
        torch.cuda.synchronize()
        del graph
        out["forms"][name] = {"us_per_block": round(s.elapsed_time(e) / n / copies * 1000.0, 2),
                              "launches": launches, "q8_1_bytes_written": qw,
                              "q8_1_bytes_read": qr, "fp32_activation_bytes": fp32_bytes}
    base = out["forms"]["per_consumer"]
    for name in ("quantize_once", "fused_prologue"):
        f = out["forms"][name]
        f["q8_1_bytes_saved"] = (base["q8_1_bytes_written"] + base["q8_1_bytes_read"]
                                 - f["q8_1_bytes_written"] - f["q8_1_bytes_read"])
    ys = b["y_sep"][:NQKV].cpu().numpy()
    out["qkv_outputs_identical"] = bool(
        np.array_equal(ys, b["y_once"][:NQKV].cpu().numpy())
        and np.array_equal(ys, b["y_fused"][:NQKV].cpu().numpy()))
    out["ffn_outputs_identical"] = bool(np.array_equal(b["y_once"][NQKV:].cpu().numpy(),
                                                       b["y_fused"][NQKV:].cpu().numpy()))
    del b
    torch.cuda.empty_cache()
    return out


def decode_batched(torch, warmup: int, steps: int, batch: int = 32, seed: int = 0, dist=None):
    """Batch-32 decode (32 sequences in lockstep, tcgen05 GEMVs): aggregate
    tok/s over ``steps`` graph replays after the 16-token prompts and
    ``warmup`` untimed steps, CUDA events on the model's stream.  Under
    torchrun (world > 1) every rank holds its tensor-parallel shard of the
    batch-32 model and the time is the max over ranks."""
    from abra_b200.model import BatchedDecodeModel

    rank, world = (dist.rank, dist.world) if dist else (0, 1)
    m = BatchedDecodeModel(batch, rank=rank, world=world, max_ctx=PROMPT + warmup + steps, seed=seed)
    prompts = np.random.default_rng(seed).integers(0, m.cfg.vocab, (batch, PROMPT)).astype(np.int32)
    m.reset(prompts)
    m.step(PROMPT - 1 + warmup)
    m.sync()
    if dist:
        dist.barrier()
    st = torch.cuda.ExternalStream(m.stream)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(st)
    m.step(steps)
    e.record(st)
    e.synchronize()
    ms = s.elapsed_time(e) / steps
    toks = m.tokens(PROMPT + warmup + steps)[:, PROMPT:]
    if dist:
        dist.barrier()  # peers push into this rank's arena until they finish
        ms = dist.max(ms)
    m.close()
    return {"batch": batch, "depth": 0, "ms_per_step": round(ms, 4),
            "tok_s_aggregate": round(batch * 1000.0 / ms, 1), "tokens_head_seq0": toks[0, :8].tolist(),
            "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "path": ("abra_model_create_batched_tp: every GEMV on tcgen05 kind::i8, o/down partial sums pushed "
                     "from the MMVQ epilogue over NVLink" if world > 1 else
                     "abra_model_create_batched: every GEMV on tcgen05 kind::i8 (abra_q4k_mmvq_tc)")}


def decode_alg_bytes(res: dict, vocab: int = 151936) -> int:
    """Algorithmic bytes of one decode step: every weight byte of the token,
    the KV rows attention reads at the run's mean context, the new K/V rows
    written, the fp32 logits written."""
    return int(res["weight_bytes"] + res["kv_read_bytes_per_token"] + KV_BYTES_PER_POS + 4 * vocab)


def decode_main(a, dist):
    import torch

    peak, peak_kind = measured_peaks()
    torch.cuda.set_device(dist.local)
    dist.init("nccl" if dist.world > 1 else "gloo")
    depths = [0] if a.quick else [0, 2048, 8192]
    dist.barrier()
    with ClockSampler(dist.local) as clk:
        res = decode_depth(torch, 0, a.warmup, a.steps, streaming=False, dist=dist)
        dist.barrier()
    clocks = clk.summary()
    ms = dist.max(res["ms_per_token"])
    tok_s = 1000.0 / ms  # one sequence, tensor parallel over all ranks
    persistent = res["step"].startswith("persistent")
    e2e = decode_depth(torch, 0, a.warmup, a.steps, streaming=True, dist=dist)
    e2e_ms = dist.max(e2e["ms_per_token"])
    extras = {"decode": {"depth0": res}}
    for d in depths[1:]:
        r = decode_depth(torch, d, a.warmup, a.steps, streaming=False, dist=dist)
        r["ms_per_token"] = dist.max(r["ms_per_token"])
        r["tok_s"] = round(1000.0 / r["ms_per_token"], 2)
        r["roofline_frac"] = round(decode_alg_bytes(r) / (r["ms_per_token"] * 1e-3) / 1e9 / peak, 4)
        extras["decode"][f"depth{d}"] = r
    # the dominant kernel: the persistent decode kernel is the whole step (one
    # launch per token), timed above with CUDA events on the model's stream
    alg = decode_alg_bytes(res)
    achieved = alg / (res["ms_per_token"] * 1e-3) / 1e9
    traffic = None
    tp = ROOT / "profiles" / "traffic_decode_token_kernel_qwen3_4b_depth0.json"
    if persistent and tp.exists():
        traffic = json.loads(tp.read_text()).get("bytes_per_launch")
    # the MMVQ family alone: the decode step's weight sweep as one graph of
    # 145 launches (batch 1), the same at batch 8
    sw = Sweep(torch.device("cuda", dist.local), 1)
    g = sw.capture()
    for _ in range(3):
        g.replay()
    ms_sw = sw.timed(max(3, a.steps // 16), g.replay)
    del g
    extras["gemv_sweep"] = {"workload": WORKLOAD, "batch": 1,
                            "GBps": round(sw.bytes / (ms_sw * 1e-3) / 1e9, 1),
                            "frac": round(sw.bytes / (ms_sw * 1e-3) / 1e9 / peak, 4),
                            "ms_per_step": round(ms_sw, 4), "launches_per_step": sw.launches}
    cpu = None
    if dist.world > 1:
        # batch 32 on the tensor cores, tensor parallel over the same ranks
        # (an error here is reported in the field; every rank raises alike)
        try:
            extras["decode_b32"] = decode_batched(torch, a.warmup, a.steps, dist=dist)
        except Exception as exc:
            extras["decode_b32"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    if dist.world == 1:
        # the same token through the per-operation kernel chain
        from abra_b200.model import KERNEL_CHAIN, Q4_K_M
        r = decode_depth(torch, 0, a.warmup, a.steps, streaming=False, flags=KERNEL_CHAIN)
        extras["decode_kernel_chain"] = {"tok_s": r["tok_s"], "ms_per_token": r["ms_per_token"],
                                         "launches_per_token": LAUNCHES_PER_TOKEN,
                                         "same_tokens": r["tokens_head"] == res["tokens_head"]}
        sw8 = Sweep(torch.device("cuda", dist.local), 8)
        g8 = sw8.capture()
        for _ in range(3):
            g8.replay()
        ms8 = sw8.timed(max(3, a.steps // 16), g8.replay)
        del g8
        extras["gemv_sweep_b8"] = {"GBps": round(sw8.bytes / (ms8 * 1e-3) / 1e9, 1),
                                   "frac": round(sw8.bytes / (ms8 * 1e-3) / 1e9 / peak, 4),
                                   "ms_per_step": round(ms8, 4)}
        del sw8
        # batch 32 on the tensor cores: the decode weight set as one graph, and
        # the batched decode step
        sw32 = Sweep(torch.device("cuda", dist.local), 32)
        ws = torch.empty(8 * 32 * 20480, dtype=torch.float32, device=sw32.dev)
        g32 = sw32.capture(lambda: launch_ops_tc(sw32.plan, ws.data_ptr(), True))
        for _ in range(3):
            g32.replay()
        ms32 = sw32.timed(max(3, a.steps // 16), g32.replay)
        del g32
        extras["gemv_sweep_b32_tc"] = {
            "GBps": round(sw32.bytes / (ms32 * 1e-3) / 1e9, 1),
            "weight_GBps": round(sw32.weight_bytes / (ms32 * 1e-3) / 1e9, 1),
            "ms_per_step": round(ms32, 4), "kernel": "mmvq_tc_kernel (tcgen05.mma kind::i8)"}
        del sw32, ws
        torch.cuda.empty_cache()
        extras["decode_b32"] = decode_batched(torch, a.warmup, a.steps)
        # the real Qwen3-4B-Q4_K_M type map: Q6_K attn_v/ffn_down in 18 layers
        # and a Q6_K tied table (kernel chain)
        r = decode_depth(torch, 0, a.warmup, a.steps, streaming=False, flags=Q4_K_M)
        extras["decode_q4_k_m"] = {"tok_s": r["tok_s"], "ms_per_token": r["ms_per_token"],
                                   "weight_bytes": r["weight_bytes"]}
        for name, fn in (("prompt_pp512", lambda: prompt_processing(torch, 512)),
                         ("lookup_verify", lambda: lookup_verification(torch)),
                         ("decode_samples", lambda: decode_samples(torch, a.warmup, a.steps))):
            try:
                extras[name] = fn()
            except Exception as exc:  # an extra must not cost the main line
                extras[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    if dist.rank == 0 and dist.world == 1:
        if not a.no_extras:
            extras["per_shape"] = shape_table(sw)
            extras["per_shape_q6k"] = shape_table_q6k(sw)
            try:
                extras["packed_q4k"] = packed_table(sw)
            except Exception as exc:
                extras["packed_q4k"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            r = ref_gpu_sweep(sw, 5)
            if r:
                extras["reference_kernels_on_b200"] = r
            try:  # the last GPU work of the run: an error here costs nothing else
                extras["fused_rmsnorm_block"] = fused_rmsnorm_block(torch, a.steps)
            except Exception as exc:
                extras["fused_rmsnorm_block"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        rate, threads, cms = cpu_decode_rate(2, 64, a.cpu_budget)
        cpu = {"value": round(rate, 3), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{len(cms)} tokens timed after 2 warm-up tokens: "
                         + CPU_DECODE.format(prompt=PROMPT, simd=simd_level())}
        gbs, t2, reps, el = cpu_sample_rate(1, max(1.0, a.cpu_budget / 4))
        extras["cpu_gemv_rate"] = {"GBps": round(gbs, 2), "cores": t2,
                                   "tok_s_if_weight_bound": round(gbs * 1e9 / res["weight_bytes"], 3),
                                   "sample": f"{CPU_SAMPLE}, {reps} passes in {el:.1f}s"}
    del sw
    if dist.rank == 0:
        line = {
            "metric": "Qwen3-4B-shape decode tok/s", "value": round(tok_s, 2), "unit": "tok/s",
            "n_gpus": dist.world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u4 x s8 dot, fp32 accumulate",
            "data": "synthetic (seeded random-init Qwen3-4B shape, all linear weights Q4_K)",
            "config": {"workload": DECODE_WORKLOAD, "model": "qwen3-4b-shape-q4k",
                       "global_batch": 1, "batch_per_gpu": 1, "seq_len": PROMPT + a.warmup + a.steps,
                       "depth": 0, "prompt": PROMPT, "gen": a.steps,
                       "parallelism": f"tp{dist.world}" if dist.world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (2.26 GB of weights per token)",
                       "step": res["step"]},
            "gpu_launches": a.steps * (1 if persistent else LAUNCHES_PER_TOKEN * dist.world),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic,
                         "kernel": "decode_token_kernel" if persistent else "decode step (kernel chain)",
                         "alg_bytes_per_launch": alg},
            "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "ms_per_step": round(e2e_ms, 4), "path": "abra_model_decode_streaming"},
            "clocks": clocks,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        line.update(extras)
        print(json.dumps(line, separators=(",", ":")), flush=True)
    dist.close()
    return 0


def reference_arm(a, dist):
    if dist.rank != 0:
        return 0
    if a.workload == "decode":
        # one step = one token of the full CPU decode, timed on all host threads
        d = CpuDecoder(a.warmup + a.steps)
        for _ in range(a.warmup):
            d.step()
        ms = [d.step() for _ in range(a.steps)]
        d.close()
        val = 1000.0 * len(ms) / sum(ms)
        sample = f"{a.steps} tokens after {a.warmup} warm-up tokens: " + CPU_DECODE.format(
            prompt=PROMPT, simd=simd_level())
        line = {
            "impl": "reference", "metric": "Qwen3-4B-shape decode tok/s", "value": round(val, 3),
            "unit": "tok/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(sum(ms) / len(ms), 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u4 x s8 dot, fp32 accumulate", "data": "synthetic",
            "config": {"workload": DECODE_WORKLOAD, "model": "qwen3-4b-shape-q4k", "global_batch": 1,
                       "batch_per_gpu": 1, "seq_len": PROMPT + a.warmup + a.steps, "depth": 0,
                       "prompt": PROMPT, "gen": a.steps,
                       "parallelism": f"CPU, {d.threads} host threads"},
            "cpu_baseline": {"value": round(val, 3), "unit": "tok/s", "cores": d.threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(val, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    for _ in range(a.warmup):
        cpu_sample_rate(a.batch, budget_s=0.5)
    # each step a bounded sample: the whole --steps/--warmup run stays within minutes
    per = max(0.5, min(20.0, 150.0 / max(1, a.steps)))
    rates = [cpu_sample_rate(a.batch, budget_s=per) for _ in range(a.steps)]
    gbs = statistics.median(r[0] for r in rates)
    threads = rates[0][1]
    sample = (f"{CPU_SAMPLE}, batch {a.batch}, {per:.1f}s per step; "
              f"{CPU_PATHS['ggml']}, integer dots at SIMD level {simd_level()} "
              "(0 scalar, 1 AVX2, 2 AVX-512 VNNI)")
    if a.workload == "decode":
        weight_bytes = sum(nmat * q4k_bytes(N, K) for _, N, K, nmat, _ in sweep_ops())
        val, unit, metric = gbs * 1e9 / weight_bytes, "tok/s", "Qwen3-4B-shape decode tok/s"
        cfg = {"workload": DECODE_WORKLOAD, "model": "qwen3-4b-shape-q4k", "global_batch": 1,
               "batch_per_gpu": 1, "seq_len": PROMPT + a.warmup + a.steps, "depth": 0,
               "prompt": PROMPT, "gen": a.steps,
               "parallelism": f"CPU restatement on {threads} host threads"}
        sample += ", scaled to the 2.26 GB of Q4_K weights a token reads"
    else:
        val, unit, metric = gbs, "GB/s", "Q4_K GEMV HBM GB/s"
        cfg = {"workload": WORKLOAD, "batch": a.batch}
    line = {
        "impl": "reference", "metric": metric, "value": round(val, 3),
        "unit": unit, "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(1000.0 / val, 3) if a.workload == "decode" else None,
        "higher_is_better": True, "scaling": "strong" if a.workload == "decode" else "weak",
        "vs_baseline": None, "dtype": "u4 x s8 dot, fp32 scale", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {"value": round(val, 3), "unit": unit, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(val, 3), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", choices=["decode", "gemv"], default="decode",
                    help="decode: Qwen3-4B-shape tg at depths 0/2048/8192 (headline: depth 0); "
                         "gemv: the decode weight sweep alone")
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps: tokens for decode (default 128), sweeps for gemv (20)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the per-shape table and the reference kernel family")
    ap.add_argument("--quick", action="store_true", help="decode: depth 0 only")
    ap.add_argument("--case", choices=[n for n, _, _ in DECODE_MATRICES] + ["qkv", "gate_up"]
                    + [f"q6k_{n}" for n, _, _ in Q6K_SHAPES]
                    + ["tc_b32_16384", "fused_rmsnorm_block", "decode_token", "decode_chain"],
                    help="profiling mode: one operator, eager launches")
    ap.add_argument("--copies", type=int, default=2, help="weight copies in --case mode")
    ap.add_argument("--depth", type=int, default=0, help="context depth in the decode_* cases")
    ap.add_argument("--layers", type=int, default=36, help="transformer layers in the decode_* cases")
    a = ap.parse_args()
    if a.warmup < 3:
        ap.error("--warmup must be >= 3")
    if a.steps is None:
        a.steps = 128 if a.workload == "decode" else 20
    if a.case:
        return run_case(a)
    dist = Dist()
    if a.impl == "reference":
        return reference_arm(a, dist)
    if a.workload == "decode":
        return decode_main(a, dist)

    import torch

    peak, peak_kind = measured_peaks()
    torch.cuda.set_device(dist.local)
    dist.init("nccl" if dist.world > 1 else "gloo")
    dev = torch.device("cuda", dist.local)
    sw = Sweep(dev, a.batch)
    sw.step()
    graph = sw.capture()  # one CUDA graph per step: 145 MMVQ launches
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    with ClockSampler(dist.local) as clk:
        ms = sw.timed(a.steps, graph.replay)
        dist.barrier()
    clocks = clk.summary()
    ms_max = dist.max(ms)
    value = dist.world * sw.bytes / (ms_max * 1e-3) / 1e9
    achieved = sw.bytes / (ms * 1e-3) / 1e9  # per GPU; only MMVQ launches in the step
    err = sw.A.device_error()
    del graph

    e2e = E2E(sw)
    for _ in range(3):
        e2e.step()
    ms_e2e = dist.max(sw.timed(max(3, a.steps // 2), e2e.step))
    e2e_val = dist.world * sw.bytes / (ms_e2e * 1e-3) / 1e9

    extras = {}
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not a.no_extras:
        extras["per_shape"] = shape_table(sw)
        r = ref_gpu_sweep(sw, max(3, a.steps // 2))
        if r:
            extras["reference_kernels_on_b200"] = r
    if dist.rank == 0 and dist.world == 1:
        gbs, threads, reps, el = cpu_sample_rate(a.batch, a.cpu_budget)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{CPU_SAMPLE}, batch {a.batch}, {reps} passes "
                         f"in {el:.1f}s; {CPU_PATHS['ggml']}, integer dots at SIMD level "
                         f"{simd_level()} (0 scalar, 1 AVX2, 2 AVX-512 VNNI)"}

    traffic = None
    tp = ROOT / "profiles" / f"traffic_{WORKLOAD}_b{a.batch}.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get("bytes_per_launch")

    if dist.rank == 0:
        line = {
            "metric": "Q4_K GEMV HBM GB/s", "value": round(value, 1), "unit": "GB/s",
            "n_gpus": dist.world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u4 x s8 dot, fp32 scale", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": a.batch, "layers": LAYERS,
                       "launches_per_step": sw.launches, "weight_bytes_per_step": sw.weight_bytes,
                       "alg_bytes_per_step": sw.bytes,
                       "l2": "inputs larger than L2 (2.26 GB of weights per step)",
                       "parallelism": f"replica x{dist.world}",
                       "launch": "one CUDA graph per step, programmatic dependent launch"},
            "gpu_launches": sw.launches * a.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": "mmvq_q4k_kernel"},
            "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": e2e.h2d,
                    "d2h_bytes_per_step": e2e.d2h, "ms_per_step": round(ms_e2e, 4)},
            "clocks": clocks,
            "device_error": err,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        line.update(extras)
        print(json.dumps(line), flush=True)
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
