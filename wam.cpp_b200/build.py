"""Builds libwam_b200.so (the engine + C ABI) for sm_100a with nvcc.

Usage: python wam.cpp_b200/build.py [--force] [--jobs N]

Objects go to wam.cpp_b200/_build/, the library to wam.cpp_b200/lib/. Each
translation unit is rebuilt only when it or a header in csrc/ or include/
changed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB_DIR = HERE / "lib"
LIB = LIB_DIR / "libwam_b200.so"
ADAPTER_SRC = HERE / "adapter" / "b200_engine.cpp"
ADAPTER_LIB = LIB_DIR / "libwam_b200_adapter.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I", str(CSRC), "-I", str(REPO / "include"), "--expt-relaxed-constexpr"]


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def headers_mtime() -> float:
    files = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def compile_one(src: Path, force: bool, hdr_time: float) -> Path:
    obj = BUILD / (src.name + ".o")
    if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
            and obj.stat().st_mtime >= hdr_time):
        return obj
    cmd = [NVCC, *COMMON, *ARCH, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, *COMMON, *ARCH, "-x", "cu", "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise SystemExit(f"nvcc failed on {src.name}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    hdr_time = headers_mtime()
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(lambda s: compile_one(s, force, hdr_time), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise SystemExit("link failed")
    return LIB


def build_adapter(reference_root: str | os.PathLike, force: bool = False) -> Path:
    """Compiles the B200Engine adapter (adapter/b200_engine.cpp) against the
    reference's own engine.h (reference_root/src, reference_root/include: the
    headers only, no reference source is compiled) into lib/libwam_b200_adapter.so,
    linked to libwam_b200.so."""
    ref = Path(reference_root)
    if not (ref / "src" / "models" / "gwp05" / "engine" / "engine.h").exists():
        raise SystemExit(f"{ref} does not hold the reference's engine.h")
    deps = [ADAPTER_SRC, HERE / "adapter" / "b200_engine.h", REPO / "include" / "wam_b200.h", LIB]
    if (not force and ADAPTER_LIB.exists()
            and ADAPTER_LIB.stat().st_mtime >= max(d.stat().st_mtime for d in deps)):
        return ADAPTER_LIB
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden",
           "-I", str(ref / "src"), "-I", str(ref / "include"), "-I", str(REPO / "include"),
           "-I", str(HERE / "adapter"), str(ADAPTER_SRC), "-L", str(LIB_DIR), "-lwam_b200",
           "-Wl,-rpath,$ORIGIN", "-o", str(ADAPTER_LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise SystemExit("adapter build failed")
    return ADAPTER_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--reference", default=os.environ.get("WAM_REFERENCE_ROOT"),
                    help="reference source tree: also build the B200Engine adapter against it")
    a = ap.parse_args()
    print(build(a.force, a.jobs))
    if a.reference:
        print(build_adapter(a.reference, a.force))
