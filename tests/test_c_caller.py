"""The C ABI from a C caller: tests/c_abi_caller.c, compiled with gcc as C99 (-Wall -Wextra
-Werror) against include/qms_cuda.h and linked to the in-tree libqms_cuda.so, runs its host-side
checks (block layout, argument validation before any device call, init without a GPU). CPU only:
the program makes no compute call."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "large_model_b200"


def test_c_caller_compiles_against_the_header_and_validates(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no gcc")
    assert (LIBDIR / "libqms_cuda.so").exists(), "build the library first (__graft_entry__.build())"
    exe = tmp_path / "c_abi_caller"
    cmd = [gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "c_abi_caller.c"), "-L", str(LIBDIR), "-lqms_cuda",
           f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    import torch
    args = [] if torch.cuda.is_available() else ["nogpu"]
    r = subprocess.run([str(exe)] + args, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr
