"""Builds liblucciola_b200.so (the C-ABI library) in place for sm_100a.

Every .cu/.cpp under csrc/ is compiled by nvcc into _build/ and linked into
liblucciola_b200.so next to this file, with the CUDA runtime linked
statically. Only rebuilt when a source or header is newer than the library.

    python lucciola-rs_b200/build.py [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "liblucciola_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(p for p in CSRC.rglob("*") if p.suffix in (".cu", ".cpp"))


def headers() -> list[Path]:
    hs = [p for p in CSRC.rglob("*") if p.suffix in (".h", ".cuh")]
    return hs + [ROOT / "include" / "lucciola_attn.h"]


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    cmd = [nvcc(), *ARCH, *COMMON, *extra, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *COMMON, *extra, "-x", "c++", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers() + [Path(__file__)])


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None) -> Path:
    if not force and not extra and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    extra = extra or []
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j))
    return 0


if __name__ == "__main__":
    sys.exit(main())
