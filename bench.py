#!/usr/bin/env python
"""Benchmark of the Q4_K x Q8_1 MMVQ path on B200.

Workload ("qwen3_4b_decode_gemv_sweep"): one step is one pass of MMVQ over
every Qwen3-4B-shaped decode matrix of the model -- per layer q 4096x2560,
k and v 1024x2560, o 2560x4096, gate and up 9728x2560, down 2560x9728, for
36 layers, then the tied 151936x2560 output -- at batch 1 (``--batch``),
all Q4_K with d, dmin ~ U(0.001, 0.02), 6-bit scales/mins ~ U{0..63},
nibbles ~ U{0..15}, activations N(0,1) quantized to Q8_1 (seed 0).  That is
2,262,528,000 bytes of weights per step, larger than L2, so every launch
reads HBM.  The metric is algorithmic bytes / time in GB/s (weights +
Q8_1 activations + fp32 outputs, the reference's formula,
bench/micro/q4k_q8_bench.cu:330-333), aggregated over ranks.

``--impl reference`` times the CPU restatement of the reference's
vec_dot_q4_K_q8_1 (oracle/, OpenMP on all host cores) on a bounded sample of
the same workload; the reference's ggml CPU path is not available.

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
LAYER_SHAPES = [("q", 4096, 2560), ("k", 1024, 2560), ("v", 1024, 2560), ("o", 2560, 4096),
                ("gate", 9728, 2560), ("up", 9728, 2560), ("down", 2560, 9728)]
OUTPUT_SHAPE = ("output", 151936, 2560)
WORKLOAD = "qwen3_4b_decode_gemv_sweep"
L2_BYTES = 126 * 1024 * 1024


def q4k_bytes(N, K):
    return N * (K // 256) * 144


def alg_bytes(N, K, B):
    """Reference formula: Q4_K weights + Q8_1 activations + fp32 outputs."""
    return q4k_bytes(N, K) + B * (K // 32) * 36 + B * N * 4


def sweep_shapes():
    out = []
    for layer in range(LAYERS):
        for i, (name, N, K) in enumerate(LAYER_SHAPES):
            out.append((f"{name}.{layer}", N, K, layer * 16 + i + 1))
    out.append((OUTPUT_SHAPE[0], OUTPUT_SHAPE[1], OUTPUT_SHAPE[2], 1))
    return out


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
def cpu_sample_rate(batch: int, budget_s: float, seed: int = 0):
    """CPU restatement of vec_dot_q4_K_q8_1 (OpenMP, all host cores) on a
    sample of the workload: the first 512 rows of every layer-0 matrix and of
    the output, repeated until ``budget_s`` seconds elapse.  Returns GB/s by
    the same byte formula."""
    import oracle as O

    threads = os.cpu_count() or 1
    rows = 512
    sample = []
    for i, (name, N, K) in enumerate(LAYER_SHAPES + [OUTPUT_SHAPE]):
        tid = i + 1 if name != "output" else 1
        w = O.gen_q4k(min(rows, N), K, seed, tid)
        xq = O.quantize_q8_1(O.gen_normal_f32((batch, K), seed + 1000 + K))
        sample.append((w, xq, min(rows, N), K))
    nbytes = sum(alg_bytes(n, k, batch) for _, _, n, k in sample)
    O.gemv(sample[0][0], sample[0][1], sample[0][3], threads)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        for w, xq, n, k in sample:
            O.gemv(w, xq, k, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    gbs = reps * nbytes / el / 1e9
    return gbs, threads, reps, el


# --------------------------------------------------------------- GPU arm ---
class Sweep:
    def __init__(self, dev, batch: int, seed: int = 0):
        import torch

        import abra_b200 as A
        import oracle as O

        self.A = A
        self.torch = torch
        self.dev = dev
        self.B = batch
        self.shapes = sweep_shapes()
        self.w = {}
        for name, N, K, tid in self.shapes:
            nb = N * K // 256
            buf = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
            A.gen_q4k(buf, nb, seed, tid)
            self.w[name] = buf
        self.Ks = sorted({K for _, _, K, _ in self.shapes})
        self.x = {K: O.gen_normal_f32((batch, K), seed + 1000 + K) for K in self.Ks}
        self.xq = {}
        for K in self.Ks:
            xq = torch.empty(batch * (K // 32) * 36, dtype=torch.uint8, device=dev)
            A.launch_quantize_f32_to_q8_1(torch.from_numpy(self.x[K].reshape(-1)).to(dev), xq, K,
                                          ncols=batch)
            self.xq[K] = xq
        maxn = max(N for _, N, _, _ in self.shapes)
        self.y = torch.empty(batch * maxn, dtype=torch.float32, device=dev)
        self.bytes = sum(alg_bytes(N, K, batch) for _, N, K, _ in self.shapes)
        self.launches = len(self.shapes)
        torch.cuda.synchronize()

    def step(self, pdl=True):
        A, B = self.A, self.B
        for name, N, K, _ in self.shapes:
            A.mmvq(self.w[name], self.xq[K], self.y, N, K, ncols=B, pdl=pdl)

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
    H2D copy of every activation (fp32, pinned) and one D2H copy of every
    output; quantization on the device inside the step."""

    def __init__(self, sw: Sweep):
        torch = sw.torch
        self.sw = sw
        B = sw.B
        # one activation column per distinct layer input (q/k/v share, o,
        # gate/up share, down) plus the output's input
        self.inputs = []
        for layer in range(LAYERS):
            self.inputs += [(f"attn.{layer}", 2560), (f"o.{layer}", 4096),
                            (f"ffn.{layer}", 2560), (f"down.{layer}", 9728)]
        self.inputs.append(("out", 2560))
        total_x = sum(K for _, K in self.inputs) * B
        self.h_x = torch.empty(total_x, dtype=torch.float32).pin_memory()
        rng = np.random.default_rng(7)
        self.h_x.numpy()[:] = rng.standard_normal(total_x, dtype=np.float32)
        self.d_x = torch.empty(total_x, dtype=torch.float32, device=sw.dev)
        self.off = {}
        o = 0
        for name, K in self.inputs:
            self.off[name] = (o, K)
            o += K * B
        self.d_q = torch.empty(sum(K // 32 * 36 for _, K in self.inputs) * B, dtype=torch.uint8,
                               device=sw.dev)
        self.qoff = {}
        o = 0
        for name, K in self.inputs:
            self.qoff[name] = o
            o += K // 32 * 36 * B
        total_y = sum(N for _, N, _, _ in sw.shapes) * B
        self.d_y = torch.empty(total_y, dtype=torch.float32, device=sw.dev)
        self.h_y = torch.empty(total_y, dtype=torch.float32).pin_memory()
        self.h2d = total_x * 4
        self.d2h = total_y * 4

    def step(self):
        sw, A, B = self.sw, self.sw.A, self.sw.B
        self.d_x.copy_(self.h_x, non_blocking=True)
        for name, K in self.inputs:
            o, _ = self.off[name]
            A.launch_quantize_f32_to_q8_1(self.d_x[o:o + K * B], self.d_q[self.qoff[name]:], K,
                                          ncols=B)
        yo = 0
        for name, N, K, _ in sw.shapes:
            kind, _, layer = name.partition(".")
            src = {"q": "attn", "k": "attn", "v": "attn", "o": "o", "gate": "ffn", "up": "ffn",
                   "down": "down"}.get(kind)
            key = f"{src}.{layer}" if src else "out"
            A.mmvq(sw.w[name], self.d_q[self.qoff[key]:], self.d_y[yo:], N, K, ncols=B)
            yo += N * B
        self.h_y.copy_(self.d_y, non_blocking=True)


def per_shape_table(sw: Sweep, reps: int = 3):
    """GB/s of each distinct shape, back-to-back over >= 4 x L2 of weight copies."""
    torch, A = sw.torch, sw.A
    out = {}
    for name, N, K in LAYER_SHAPES + [OUTPUT_SHAPE]:
        nb = N * K // 256
        per = nb * 144
        copies = max(8, -(-4 * L2_BYTES // per))
        bufs = [sw.w[f"{name}.{i}"] if f"{name}.{i}" in sw.w else None for i in range(LAYERS)]
        bufs = [b for b in bufs if b is not None][:copies]
        if name == "output":
            bufs = [sw.w["output"]]
        extra = []
        while len(bufs) + len(extra) < copies:
            t = torch.empty(per, dtype=torch.uint8, device=sw.dev)
            A.gen_q4k(t, nb, 0, 9000 + len(extra))
            extra.append(t)
        allb = bufs + extra

        def run():
            for b in allb:
                A.mmvq(b, sw.xq[K], sw.y, N, K, ncols=sw.B, pdl=True)

        run()
        ms = min(sw.timed(1, run) for _ in range(reps))
        per_launch_us = ms * 1e3 / len(allb)
        out[name] = {"N": N, "K": K, "us": round(per_launch_us, 3),
                     "GBps": round(alg_bytes(N, K, sw.B) / (per_launch_us * 1e-6) / 1e9, 1),
                     "copies": len(allb)}
        del extra
    return out


def ref_gpu_sweep(sw: Sweep, steps: int):
    """The reference's own kernel family (oracle/_ref) on the same sweep, batch 1,
    with the reference's dispatch rule (get_autotuned_candidate_for_shape)."""
    import oracle as O

    try:
        ref = O.RefFamily()
    except FileNotFoundError:
        return None
    if sw.B != 1:
        return None
    stream = sw.torch.cuda.current_stream().cuda_stream
    plan = []
    for name, N, K, _ in sw.shapes:
        cid = ref.autotuned_candidate(N, K, 61)
        if cid == 0:
            cid = 204
        plan.append((sw.w[name].data_ptr(), sw.xq[K].data_ptr(), N, K, cid))
    yp = sw.y.data_ptr()

    def run():
        for w, x, N, K, cid in plan:
            ref.launch_candidate(cid, w, x, yp, N, K, stream)

    run()
    ms = sw.timed(steps, run)
    return {"GBps": round(sw.bytes / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4),
            "dispatch": "reference get_autotuned_candidate_for_shape(N, K, 61)"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-extras", action="store_true", help="skip per-shape table and reference GPU family")
    a = ap.parse_args()
    if a.warmup < 3:
        ap.error("--warmup must be >= 3")
    peak, peak_kind = measured_peaks()
    dist = Dist()

    if a.impl == "reference":
        if dist.rank != 0:
            return 0
        rates = []
        for _ in range(a.warmup):
            cpu_sample_rate(a.batch, budget_s=0.5)
        per = max(1.0, min(20.0, 150.0 / max(1, a.steps)))
        for _ in range(a.steps):
            rates.append(cpu_sample_rate(a.batch, budget_s=per))
        gbs = statistics.median(r[0] for r in rates)
        threads = rates[0][1]
        line = {
            "impl": "reference", "metric": "Q4_K GEMV HBM GB/s", "value": round(gbs, 3),
            "unit": "GB/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/u4 dot, fp32 scale", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": a.batch},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                             "kind": "port",
                             "sample": f"first 512 rows of each layer-0 matrix and of the output, "
                                       f"batch {a.batch}, {per:.0f}s per step; CPU restatement of "
                                       "vec_dot_q4_K_q8_1 (ggml CPU path unavailable)"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0

    import torch

    torch.cuda.set_device(dist.local)
    dist.init("nccl" if dist.world > 1 else "gloo")
    dev = torch.device("cuda", dist.local)
    sw = Sweep(dev, a.batch)
    for _ in range(a.warmup):
        sw.step()
    torch.cuda.synchronize()
    dist.barrier()
    with ClockSampler(dist.local) as clk:
        ms = sw.timed(a.steps)
        dist.barrier()
    clocks = clk.summary()
    ms_max = dist.max(ms)
    value = dist.world * sw.bytes / (ms_max * 1e-3) / 1e9
    achieved = sw.bytes / (ms * 1e-3) / 1e9  # per GPU: only MMVQ launches in the step
    err = sw.A.device_error()

    # end to end through the C ABI with host buffers
    e2e = E2E(sw)
    for _ in range(3):
        e2e.step()
    ms_e2e = dist.max(sw.timed(max(3, a.steps // 2), e2e.step))
    e2e_val = dist.world * sw.bytes / (ms_e2e * 1e-3) / 1e9

    extras = {}
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not a.no_extras:
        extras["per_shape"] = per_shape_table(sw)
        r = ref_gpu_sweep(sw, max(3, a.steps // 2))
        if r:
            extras["reference_kernels_on_b200"] = r
    if dist.rank == 0 and dist.world == 1:
        gbs, threads, reps, el = cpu_sample_rate(a.batch, a.cpu_budget)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"first 512 rows of each layer-0 matrix and of the output, batch "
                         f"{a.batch}, {reps} reps in {el:.1f}s; CPU restatement of "
                         "vec_dot_q4_K_q8_1 (ggml CPU path unavailable)"}

    traffic = None
    tp = ROOT / "profiles" / f"traffic_{WORKLOAD}_b{a.batch}.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get("bytes_per_launch")

    if dist.rank == 0:
        line = {
            "metric": "Q4_K GEMV HBM GB/s", "value": round(value, 1), "unit": "GB/s",
            "n_gpus": dist.world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/u4 dot, fp32 scale", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": a.batch, "layers": LAYERS,
                       "launches_per_step": sw.launches,
                       "weight_bytes_per_step": sum(q4k_bytes(N, K) for _, N, K, _ in sw.shapes),
                       "alg_bytes_per_step": sw.bytes,
                       "l2": "inputs larger than L2 (2.26 GB of weights per step)",
                       "parallelism": f"replica x{dist.world}"},
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
