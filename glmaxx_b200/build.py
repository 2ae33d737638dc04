"""In-tree build of libglmaxx_sm100.so (nvcc, sm_100a) -- the product library.

    python -m glmaxx_b200.build [--force]

Compiles every csrc/*.cu for `-gencode arch=compute_100a,code=sm_100a` and
every host-only csrc/*.cpp with g++, in parallel, and links them into
glmaxx_b200/libglmaxx_sm100.so next to this file, so the built library travels
with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "glmaxx_sm100"
LIB = PKG / "libglmaxx_sm100.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _deps():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")) + list(CSRC.glob("*.cuh")) +
                  list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h")) + [Path(__file__)])


def _cuda_include() -> str:
    return str(Path(_nvcc()).resolve().parent.parent / "include")


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    nvcc = _nvcc()
    BUILD.mkdir(parents=True, exist_ok=True)
    env = dict(os.environ)
    # nvcc's host compiler: the system gcc (an environment CC wrapper may lack runtime specs)
    host_cc = ["-ccbin", "/usr/bin/g++"] if Path("/usr/bin/g++").exists() else []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if src.suffix == ".cpp":
            cxx = host_cc[1] if host_cc else (shutil.which("g++") or "g++")
            cmd = [cxx, "-O3", "-std=c++17", "-fPIC", "-Wall", "-Wextra", f"-I{ROOT / 'include'}",
                   f"-I{CSRC}", f"-I{_cuda_include()}", "-c", str(src), "-o", str(obj)]
        else:
            cmd = [nvcc, *host_cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True, env=env)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed on {src.name}:\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *host_cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart",
           "-Xlinker", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
