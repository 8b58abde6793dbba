"""Build libcta_stencil.so (sm_100a) in-tree with nvcc.

The shared library is the only native artefact of the package: the CUDA
kernels (``csrc/*.cu``) and the C ABI declared in ``include/cta_stencil.h``.
It links the CUDA runtime statically, so it has no dependency on the CUDA
runtime that PyTorch ships; both share the device's primary context.

Usage: ``python -m cta_b200.build [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_ROOT = PKG_DIR.parent                     # continuous-time-attention_b200/
CSRC = SRC_ROOT / "csrc"
REPO_ROOT = SRC_ROOT.parent
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = SRC_ROOT / "_build"
LIB_NAME = "libcta_stencil.so"
LIB_PATH = PKG_DIR / LIB_NAME

# the kernel units (one per dtype and arithmetic, so that they compile in
# parallel) first, then the host-side units
SOURCES = [
    "bld_fwd_bf16_fm.cu", "bld_fwd_f16_fm.cu", "bld_fwd_bf16.cu", "bld_fwd_f16.cu", "bld_fwd_f32.cu",
    "bld_dalpha_bf16_fm.cu", "bld_dalpha_f16_fm.cu", "bld_dalpha_bf16.cu", "bld_dalpha_f16.cu",
    "bld_dalpha_f32.cu", "stencil_bdl.cu", "capi.cu", "bld_fwd.cu", "bld_dalpha.cu", "noalloc.cu",
]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    # no contraction: every fused multiply-add in the kernels is written explicitly
    "-fmad=false",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-Wall",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs())


# A march kernel keeps its whole state in registers; a stack frame above a few
# bytes means a helper was not inlined (its state went to local memory) or
# large spills, either of which costs an order of magnitude.
MAX_STACK_BYTES = 64


def stack_frames(ptxas_log: str) -> list:
    """(kernel, bytes) for every entry function of a ptxas -v report whose
    stack frame exceeds MAX_STACK_BYTES."""
    out = []
    name = None
    for line in ptxas_log.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            name = m.group(1)
            continue
        m = re.search(r"(\d+) bytes stack frame", line)
        if m and name is not None:
            if int(m.group(1)) > MAX_STACK_BYTES:
                out.append((name, int(m.group(1))))
            name = None
    return out


def build(force: bool = False, verbose: bool = False, jobs: int | None = None, defines: tuple = (),
          out: Path | None = None) -> Path:
    """Compile every kernel translation unit for sm_100a and link the library.

    `defines` (e.g. ("CTA_FWD_STAGES=4",)) and `out` build a tuning variant into
    another file; the default build is the in-tree libcta_stencil.so.
    """
    target = Path(out) if out is not None else LIB_PATH
    if not force and not defines and out is None and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    build_dir = BUILD_DIR if not defines else BUILD_DIR / ("var_" + "_".join(d.replace("=", "") for d in defines))
    build_dir.mkdir(parents=True, exist_ok=True)
    incs = ["-I", str(INCLUDE), "-I", str(CSRC)] + [f"-D{d}" for d in defines]

    headers = [f for f in _inputs() if f.suffix != ".cu"]
    newest_header = max((f.stat().st_mtime for f in headers), default=0.0)

    def compile_one(name: str) -> Path:
        obj = build_dir / (Path(name).stem + ".o")
        # ptxas -v always: its per-kernel report is checked for stack frames
        cmd = [nvcc, *ARCH_FLAGS, "-Xptxas=-v", *CFLAGS, *incs, "-c", str(CSRC / name), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        # an object is reused when it is newer than its source and every header
        # and was built by the same command
        stamp = obj.with_suffix(".cmd")
        if (not force and not verbose and obj.exists() and stamp.exists() and stamp.read_text() == " ".join(cmd)
                and obj.stat().st_mtime > max((CSRC / name).stat().st_mtime, newest_header)):
            return obj
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {name}:\n{res.stdout}\n{res.stderr}")
        if verbose and (res.stdout or res.stderr):
            print(res.stdout + res.stderr, flush=True)
        big = stack_frames(res.stderr)
        if big:
            raise RuntimeError(f"{name}: kernels with a stack frame above {MAX_STACK_BYTES} bytes (a call that was "
                               f"not inlined, or spills): " + "; ".join(f"{k} {v} B" for k, v in big[:8]))
        stamp.write_text(" ".join(cmd))
        return obj

    with ThreadPoolExecutor(max_workers=jobs or min(len(SOURCES), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, SOURCES))

    tmp = target.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-Xlinker", f"-soname={LIB_NAME}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, target)
    return target


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
