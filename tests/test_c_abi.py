"""The C ABI from plain C: tests/c_abi_host.c, compiled with gcc against
include/abra_b200.h and linked with libabra_b200.so, makes the calls that
need no GPU (tables, tuning, launch plans, the lookup draft, the
tensor-parallel split, argument checks) and exits 0 when they all hold."""
from __future__ import annotations

import shutil
import subprocess

import pytest

from conftest import ROOT


def test_c_caller_builds_links_and_runs(tmp_path):
    import abra_b200

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    lib = abra_b200.LIB_PATH
    exe = tmp_path / "c_abi_host"
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "c_abi_host.c"), "-o", str(exe), str(lib),
           f"-Wl,-rpath,{lib.parent}"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr + run.stdout
    assert "ok" in run.stdout
