"""The reference arm of bench.py (the CPU restatement on the host cores) runs
without a GPU: one short invocation, its JSON line checked for the fields
the measurement contract asks for."""
from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_line():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"]


def test_bench_cli_parses():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True,
                         text=True, timeout=300, cwd=ROOT)
    assert res.returncode == 0 and "--impl" in res.stdout and "--case" in res.stdout


class _Checked:
    """Stand-in for the abra_b200 entry points the quantize-once block calls:
    instead of launching, it checks that every byte range each kernel would
    touch (from the call's N, K and column count) lies inside one of the
    block's tensors, and that the alignments the C ABI demands hold."""

    def __init__(self, tensors):
        import abra_b200 as A

        self.spans = [(t.data_ptr(), t.data_ptr() + t.numel() * t.element_size()) for t in tensors]
        self.q4k_nbytes = A.q4k_nbytes
        self.calls = 0

    def _in(self, p, nbytes, align=4):
        assert isinstance(p, int) and p % align == 0, (p, align)
        assert any(lo <= p and p + nbytes <= hi for lo, hi in self.spans), (p, nbytes)

    def rmsnorm_quantize_q8_1(self, x, w, eps, xq, K, ncols=1, d_xn_out=None, stream=None):
        self.calls += 1
        self._in(x, ncols * K * 4)
        self._in(w, K * 4)
        self._in(xq, ncols * K // 32 * 36)
        if d_xn_out is not None:
            self._in(d_xn_out, ncols * K * 4)

    def launch_quantize_f32_to_q8_1(self, x, xq, K, stream=None, ncols=1):
        self.calls += 1
        self._in(x, ncols * K * 4)
        self._in(xq, ncols * K // 32 * 36)

    def mmvq(self, w, x, y, N, K, ncols=1, ldy=None, candidate=0, pdl=False, stream=None):
        self.calls += 1
        self._in(w, self.q4k_nbytes(N, K), 16)
        self._in(x, ncols * K // 32 * 36, 16)
        self._in(y, ncols * (ldy or N) * 4)

    def mmvq_swiglu(self, wg, wu, x, y, N, K, ncols=1, ldy=None, candidate=0, pdl=False,
                    stream=None):
        self.calls += 1
        self._in(wu, self.q4k_nbytes(N, K), 16)
        self.calls -= 1
        self.mmvq(wg, x, y, N, K, ncols, ldy)

    def mmvq_rmsnorm(self, w, x, g, eps, y, N, K, d_w_up=None, d_x_q8_out=None, candidate=0,
                     pdl=False, stream=None):
        self.calls += 1
        self._in(w, self.q4k_nbytes(N, K), 16)
        if d_w_up is not None:
            self._in(d_w_up, self.q4k_nbytes(N, K), 16)
        self._in(x, K * 4)
        self._in(g, K * 4, 16)
        self._in(y, N * 4)
        if d_x_q8_out is not None:
            self._in(d_x_q8_out, K // 32 * 36)


def test_quantize_once_block_addresses_stay_in_their_buffers():
    """bench.py's quantize-once block (three forms of RMSNorm -> Q8_1 -> five
    consumers) run against checked stand-ins on CPU tensors: every pointer
    and size it passes fits its buffer, and each form makes the launches it
    reports."""
    import torch

    sys.path.insert(0, str(ROOT))
    import bench

    b = bench.fused_block_buffers(torch, torch.device("cpu"), copies=2)
    tensors = b["wqkv"] + b["wg"] + b["wu"] + [b[k] for k in
                                                ("x", "g", "xn", "xq", "y_sep", "y_once", "y_fused")]
    fake = _Checked(tensors)
    forms = bench.fused_block_forms(fake, b)
    assert set(forms) == {"per_consumer", "quantize_once", "fused_prologue"}
    for name, (fn, launches, qw, qr, _) in forms.items():
        for r in range(2):
            fake.calls = 0
            fn(r)
            assert fake.calls == launches, (name, fake.calls)
    assert forms["per_consumer"][2] + forms["per_consumer"][3] == 11 * 2880
    assert forms["fused_prologue"][2] == forms["fused_prologue"][3] == 0
