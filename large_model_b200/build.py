"""Build libqms_cuda.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed), and, where the
reference's source tree is present, the device build of its CLI (`bin/qms`): the reference's own
main.c, gguf.c, quant.c, kernels.c, tok.c and chat.c compiled unchanged, with host/qms_dev_model.c
in place of model.c (it compiles model.c inside itself and routes qms_forward to the device).

    python -m large_model_b200.build            # incremental
    python -m large_model_b200.build --clean
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libqms_cuda.so"
CLI = PKG / "bin" / "qms"
HOST = PKG / "host"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-Xptxas", "-O3",
                "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(obj: Path, deps: list[Path]) -> bool:
    return not obj.exists() or any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if _stale(obj, _deps(src)):
        cmd = [NVCC] + FLAGS + ["-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)
    return obj


def reference_root() -> Path | None:
    """The reference source tree (QMS_REFERENCE, else BASELINE.json's reference_path), if present."""
    p = os.environ.get("QMS_REFERENCE")
    if not p:
        try:
            p = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            p = None
    if p and (Path(p) / "src" / "model.c").exists():
        return Path(p)
    return None


def build_cli(verbose: bool = False) -> Path | None:
    """gcc: the reference CLI with the device model layer (needs the reference's sources)."""
    ref = reference_root()
    if ref is None:
        return None
    src = ref / "src"
    srcs = [src / f for f in ("main.c", "gguf.c", "quant.c", "kernels.c", "tok.c", "chat.c")]
    srcs.append(HOST / "qms_dev_model.c")
    deps = srcs + [LIB] + sorted(src.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))
    if CLI.exists() and all(d.stat().st_mtime <= CLI.stat().st_mtime for d in deps):
        return CLI
    CLI.parent.mkdir(exist_ok=True)
    cmd = ["gcc", "-O2", "-std=gnu11", "-D_GNU_SOURCE", "-march=x86-64-v3", "-fopenmp", "-Wall",
           f"-I{src}", f"-I{ROOT / 'include'}", "-o", str(CLI)] + [str(x) for x in srcs] + \
          [f"-L{PKG}", "-lqms_cuda", "-Wl,-rpath,$ORIGIN/..", "-lm"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"device CLI build failed:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return CLI


def build(verbose: bool = False, clean: bool = False) -> Path:
    if clean and OBJ.exists():
        shutil.rmtree(OBJ)
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + ["-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_cli(verbose)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, clean=a.clean))
