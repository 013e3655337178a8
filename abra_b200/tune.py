"""Autotuner for the sm_100a MMVQ family.

For every (N, K, ncols, nmat) in the shape list it times every candidate of
the family as one CUDA graph of back-to-back launches (programmatic
dependent launch on) over enough distinct weight copies that their total is
at least 4 x L2 (at least 4 copies), keeps the best of a few replays, and
writes the winners -- with every candidate's time -- to
``abra_b200/tuning/sm100.json``, which ``abra_b200`` loads at import.

This replaces the reference's offline tuner (tools/run-m4-autotune.py,
synthesize_tuning_table at :168-240) and its hand-copied table
(kernels/q4k/q4k_family.cu:378-397).  Ties within 0.5 % go to the lower
candidate id, mirroring the reference's tie-break rule (:200-206).

    python -m abra_b200.tune [--ncols 1 8] [--out PATH] [--quick]
    python -m abra_b200.tune --tp --ncols 1 --merge   # tensor-parallel shard shapes
    python -m abra_b200.tune --decode                 # decode slots, by whole-token time
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

from . import _lib
from .q4k import TUNING_FILE, get_all_candidate_ids, get_candidate_spec, stream_handle

L2_BYTES = 126 * 1024 * 1024

# Qwen3-4B decode shapes: q, k/v, o, gate/up, down, output, fused q|k|v;
# nmat 2 = fused gate/up SwiGLU (9728 x 2560 each).
DECODE_SHAPES = [
    (4096, 2560, 1), (1024, 2560, 1), (2560, 4096, 1), (9728, 2560, 1), (2560, 9728, 1),
    (151936, 2560, 1), (6144, 2560, 1), (9728, 2560, 2),
]


def tp_shapes(worlds=(2, 4, 8)):
    """Per-rank shapes of the tensor-parallel decode: (N, K, nmat, K_full,
    sl_base, sl_cnt); K_full > 0 marks a K-shard (o, down), timed through the
    K-shard entry point with the shard's slicing."""
    from .model import shard_info

    out = []
    for w in worlds:
        for r in range(w):
            s = shard_info(r, w)
            qkv = (s.q_heads + 2 * s.kv_heads) * 128
            ffn = s.ffn_hi - s.ffn_lo
            for shp in ((qkv, 2560, 1, 0, 0, 8),
                        (2560, s.q_heads * 128, 1, 4096, s.sl_base, s.sl_cnt),
                        (ffn, 2560, 2, 0, 0, 8), (2560, ffn, 1, 9728, s.sl_base, s.sl_cnt),
                        (int(s.vocab_hi - s.vocab_lo), 2560, 1, 0, 0, 8)):
                if shp[:3] not in [o[:3] for o in out]:
                    out.append(shp)
    return out


def q4k_bytes(N: int, K: int) -> int:
    return N * (K // 256) * 144


def pick_winner(times: dict) -> int:
    """The candidate a shape's entry names: among those within 0.5 % of the
    fastest, the lowest id.  The reference keeps the same 0.5 % band and
    breaks ties by its own geometry order, then the id
    (tools/run-m4-autotune.py:196-206); the id is this family's order."""
    if not times:
        raise ValueError("no candidate times")
    fastest = min(times.values())
    return min(c for c, t in times.items() if t <= fastest * 1.005)


def time_candidate(torch, plan, ncols, nmat, cid, reps=3, failures=None, kshard=(0, 0, 8)):
    from .q4k import device_error

    f_mm = _lib.lib.abra_q4k_mmvq_ex
    f_sw = _lib.lib.abra_q4k_mmvq_swiglu
    f_ks = _lib.lib.abra_q4k_mmvq_kshard
    K_full, sl_base, sl_cnt = kshard

    def run(items=plan):
        st = stream_handle(None)
        for w, w2, x, y, N, K in items:
            if K_full:
                rc = f_ks(w, x, y, N, K, ncols, K_full, sl_base, sl_cnt, cid, _lib.ABRA_MMVQ_PDL, st)
            elif nmat == 1:
                rc = f_mm(w, x, y, N, K, ncols, N, cid, _lib.ABRA_MMVQ_PDL, st)
            else:
                rc = f_sw(w, w2, x, y, N, K, ncols, N, cid, _lib.ABRA_MMVQ_PDL, st)
            if rc:
                return rc
        return 0

    # one launch, then two back to back, each checked before anything longer runs
    for items in (plan[:1], plan[:2], plan):
        rc = run(items)
        torch.cuda.synchronize()
        err = device_error(clear=True)
        if rc or err:
            if failures is not None and err:
                failures.append({"candidate": cid, "device_error": err, "launches": len(items)})
            return None
    return graph_time(torch, run, len(plan), reps)


def graph_time(torch, run, launches: int, reps: int = 3) -> float:
    """Microseconds per launch of ``run`` (``launches`` launches) captured in
    one CUDA graph, best of ``reps`` replays."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    best = float("inf")
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e) * 1e3 / launches)
    del g
    return best


# the real Qwen3-4B-Q4_K_M Q6_K tensors: attn_v, ffn_down, tied output
Q6K_SHAPES = [(1024, 2560), (2560, 9728), (151936, 2560)]


def tune_q6k(shapes, ncols_list, out: Path, reps: int = 3) -> dict:
    """Time every Q6_K candidate (abra_q6k_mmvq_ex) per shape and batch
    width, as tune() does for Q4_K, and store the winners under
    ``q6k_entries`` of ``out`` (other keys kept)."""
    import torch

    import abra_b200 as A
    from .q4k import device_error

    dev = torch.device("cuda:0")
    ids = sorted(A.q6k_candidates())
    f = _lib.lib.abra_q6k_mmvq_ex
    entries = []
    for N, K in shapes:
        per = N * (K // 256) * 210
        copies = max(4, -(-4 * L2_BYTES // per))
        nb = N * K // 256
        bufs = []
        for i in range(copies):
            t = torch.empty(nb * 210, dtype=torch.uint8, device=dev)
            A.gen_q6k(t, nb, 0, 7500 + i)
            bufs.append(t)
        for ncols in ncols_list:
            x = torch.from_numpy(np.random.default_rng(K).standard_normal(ncols * K, dtype=np.float32)).to(dev)
            xq = torch.empty(ncols * (K // 32) * 36, dtype=torch.uint8, device=dev)
            A.launch_quantize_f32_to_q8_1(x, xq, K, ncols=ncols)
            y = torch.empty(ncols * N, dtype=torch.float32, device=dev)
            times = {}
            for cid in ids:
                def run(n=copies, cid=cid):
                    st = stream_handle(None)
                    for b in bufs[:n]:
                        rc = f(b.data_ptr(), xq.data_ptr(), y.data_ptr(), N, K, ncols, N, cid,
                               _lib.ABRA_MMVQ_PDL, st)
                        if rc:
                            return rc
                    return 0
                if run(1) or run(2):  # shape does not fit this candidate
                    continue
                torch.cuda.synchronize()
                if device_error(clear=True):
                    continue
                times[cid] = graph_time(torch, run, copies, reps)
            assert times, f"no Q6_K candidate ran for {(N, K, ncols)}"
            winner = pick_winner(times)
            nbytes = per + ncols * (K // 32) * 36 + ncols * N * 4
            e = {"N": N, "K": K, "ncols": ncols, "candidate": winner, "us": round(times[winner], 3),
                 "GBps": round(nbytes / (times[winner] * 1e-6) / 1e9, 1), "copies": copies,
                 "all_us": {str(c): round(t, 3) for c, t in sorted(times.items())}}
            entries.append(e)
            print(json.dumps({k: e[k] for k in ("N", "K", "ncols", "candidate", "us", "GBps")}), flush=True)
        del bufs
        torch.cuda.empty_cache()
    data = json.loads(out.read_text()) if out.exists() else {"arch": 100, "entries": []}
    keys = {(e["N"], e["K"], e["ncols"]) for e in entries}
    data["q6k_entries"] = [e for e in data.get("q6k_entries", [])
                           if (e["N"], e["K"], e["ncols"]) not in keys] + entries
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(data, indent=1) + "\n")
    return data


def tune(shapes, ncols_list, out: Path, quick: bool = False, ids=None, merge: bool = False) -> dict:
    import torch

    import abra_b200 as A

    dev = torch.device("cuda:0")
    ids = ids or get_all_candidate_ids()
    entries = []
    failures = []
    for shape in shapes:
        N, K, nmat = shape[:3]
        kshard = tuple(shape[3:6]) if len(shape) >= 6 else (0, 0, 8)
        per = q4k_bytes(N, K) * nmat
        copies = max(4, -(-4 * L2_BYTES // per))
        if quick:
            copies = max(2, copies // 4)
        nb = N * K // 256
        bufs = []
        for i in range(copies * nmat):
            t = torch.empty(nb * 144, dtype=torch.uint8, device=dev)
            A.gen_q4k(t, nb, 0, 7000 + i)
            bufs.append(t)
        for ncols in ncols_list:
            x = torch.from_numpy(np.random.default_rng(K).standard_normal(ncols * K, dtype=np.float32)).to(dev)
            xq = torch.empty(ncols * (K // 32) * 36, dtype=torch.uint8, device=dev)
            A.launch_quantize_f32_to_q8_1(x, xq, K, ncols=ncols)
            y = torch.empty(ncols * N, dtype=torch.float32, device=dev)
            plan = []
            for i in range(copies):
                w = bufs[i * nmat].data_ptr()
                w2 = bufs[i * nmat + 1].data_ptr() if nmat == 2 else 0
                plan.append((w, w2, xq.data_ptr(), y.data_ptr(), N, K))
            times = {}
            for cid in ids:
                nf = len(failures)
                us = time_candidate(torch, plan, ncols, nmat, cid, failures=failures, kshard=kshard)
                if len(failures) > nf:
                    failures[-1].update({"N": N, "K": K, "ncols": ncols, "nmat": nmat})
                    print(json.dumps({"failure": failures[-1]}), flush=True)
                if us is not None:
                    times[cid] = us
            assert times, f"no candidate ran for {(N, K, ncols, nmat)}"
            winner = pick_winner(times)
            nbytes = per + ncols * (K // 32) * 36 + ncols * N * 4
            e = {"N": N, "K": K, "ncols": ncols, "nmat": nmat, "candidate": winner,
                 **({"K_full": kshard[0], "sl_base": kshard[1], "sl_cnt": kshard[2]}
                    if kshard[0] else {}),
                 "name": get_candidate_spec(winner).name, "us": round(times[winner], 3),
                 "GBps": round(nbytes / (times[winner] * 1e-6) / 1e9, 1), "copies": copies,
                 "all_us": {str(c): round(t, 3) for c, t in sorted(times.items())}}
            entries.append(e)
            print(json.dumps({k: e[k] for k in ("N", "K", "ncols", "nmat", "name", "us", "GBps")}),
                  flush=True)
        del bufs
        torch.cuda.empty_cache()
    old = json.loads(out.read_text()) if merge and out.exists() else {}
    if old:
        keys = {(e["N"], e["K"], e["ncols"], e["nmat"]) for e in entries}
        entries = [e for e in old.get("entries", [])
                   if (e["N"], e["K"], e["ncols"], e["nmat"]) not in keys] + entries
        failures = old.get("failures", []) + failures
    data = dict(old)  # other sections (decode_in_situ, q6k_entries) are kept
    data.update({"arch": 100, "device": torch.cuda.get_device_name(0),
                 "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
                 "method": "CUDA graph of back-to-back launches over >= 4 x L2 of weight copies, "
                           "PDL on, best of 3 replays; ties within 0.5% to the lower id",
                 "entries": entries, "failures": failures})
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(data, indent=1) + "\n")
    return data


def decode_slots():
    """The MMVQ launch slots of one decode token (batch 1, one GPU):
    (name, N, K, nmat)."""
    return [("qkv", 6144, 2560, 1), ("o", 2560, 4096, 1), ("gate_up", 9728, 2560, 2),
            ("down", 2560, 9728, 1), ("output", 151936, 2560, 1)]


def tune_decode(out: Path, passes: int = 2, tokens: int = 48, ids=None) -> dict:
    """In-situ tuning: the candidate of each MMVQ slot of the decode step is
    chosen by the time of whole decode tokens (one CUDA graph per token, the
    same graph the runtime replays), one slot at a time, ``passes`` rounds
    of coordinate descent.  Kernel-alone timing misses how a kernel's
    prologue and tail overlap its neighbours under programmatic dependent
    launch; this measures exactly that."""
    import torch

    from .model import DecodeModel

    ids = ids or get_all_candidate_ids()
    m = DecodeModel(max_ctx=tokens + 64)
    prompt = np.random.default_rng(0).integers(0, m.cfg.vocab, 16).astype(np.int32)
    st = torch.cuda.ExternalStream(m.stream)

    def token_ms() -> float:  # every measurement at the same positions
        m.invalidate()
        m.reset(prompt)
        m.step(4)
        m.sync()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(st)
        m.step(tokens)
        e.record(st)
        e.synchronize()
        return s.elapsed_time(e) / tokens

    current = {name: _lib.lib.abra_tune_get(N, K, 1, nmat) for name, N, K, nmat in decode_slots()}
    log = []
    base = token_ms()
    for p in range(passes):
        for name, N, K, nmat in decode_slots():
            times = {}
            for cid in ids:
                if _lib.lib.abra_tune_set(N, K, 1, nmat, cid) != 0:
                    continue
                try:
                    times[cid] = token_ms()
                except _lib.AbraError as exc:  # e.g. staging that does not fit
                    log.append({"slot": name, "candidate": cid, "error": str(exc)})
            best = min(times, key=times.get)
            if times[best] > times.get(current[name], float("inf")) * 0.995:
                best = current[name]  # keep the incumbent unless clearly beaten
            current[name] = best
            _lib.lib.abra_tune_set(N, K, 1, nmat, best)
            log.append({"pass": p, "slot": name, "candidate": best, "ms_per_token": round(times[best], 4),
                        "all_ms": {str(c): round(t, 4) for c, t in sorted(times.items())}})
            print(json.dumps({k: log[-1][k] for k in ("pass", "slot", "candidate", "ms_per_token")}), flush=True)
    final = token_ms()
    m.close()
    entries = [{"N": N, "K": K, "ncols": 1, "nmat": nmat, "candidate": current[name],
                "name": get_candidate_spec(current[name]).name, "slot": name, "in_situ": True}
               for name, N, K, nmat in decode_slots()]
    data = json.loads(out.read_text()) if out.exists() else {"arch": 100, "entries": []}
    keys = {(e["N"], e["K"], e["ncols"], e["nmat"]) for e in entries}
    data["entries"] = [e for e in data.get("entries", [])
                       if (e["N"], e["K"], e["ncols"], e["nmat"]) not in keys] + entries
    data["decode_in_situ"] = {"when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
                              "ms_per_token_before": round(base, 4),
                              "ms_per_token_after": round(final, 4), "tokens": tokens,
                              "passes": passes, "log": log}
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(data, indent=1) + "\n")
    print(json.dumps({"before_ms": round(base, 4), "after_ms": round(final, 4)}), flush=True)
    return data


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ncols", type=int, nargs="+", default=[1, 8])
    ap.add_argument("--out", default=str(TUNING_FILE))
    ap.add_argument("--quick", action="store_true", help="fewer weight copies")
    ap.add_argument("--shape", type=int, nargs=3, action="append", metavar=("N", "K", "NMAT"),
                    help="tune only these shapes (repeatable)")
    ap.add_argument("--ids", type=int, nargs="+", help="only these candidate ids")
    ap.add_argument("--tp", action="store_true",
                    help="the per-rank shapes of the 2/4/8-GPU tensor-parallel decode (batch 1)")
    ap.add_argument("--merge", action="store_true", help="keep the other entries of --out")
    ap.add_argument("--q6k", action="store_true",
                    help="tune the Q6_K MMVQ on the real Qwen3-4B-Q4_K_M Q6_K shapes (q6k_entries)")
    ap.add_argument("--decode", action="store_true",
                    help="in-situ: pick each decode slot's candidate by whole-token time")
    a = ap.parse_args(argv)
    if a.decode:
        tune_decode(Path(a.out), ids=a.ids)
        return 0
    if a.q6k:
        shapes = [tuple(s[:2]) for s in a.shape] if a.shape else Q6K_SHAPES
        tune_q6k(shapes, a.ncols, Path(a.out))
        return 0
    shapes = [tuple(s) for s in a.shape] if a.shape else (tp_shapes() if a.tp else DECODE_SHAPES)
    tune(shapes, a.ncols, Path(a.out), a.quick, a.ids, a.merge)
    return 0


if __name__ == "__main__":
    sys.exit(main())
