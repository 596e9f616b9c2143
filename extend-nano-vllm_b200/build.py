"""Build libb200moe.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: python extend-nano-vllm_b200/build.py [--force] [--jobs N]

Each csrc/*.cu is compiled with nvcc as relocatable device code (the status
word is shared across translation units) and the objects are device-linked
into one shared library next to this file.  The CUDA runtime is linked
statically and the driver entry point used for TMA descriptors is fetched at
run time, so the library loads on machines without a GPU driver.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB_NAME = "libb200moe.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-rdc=true", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build b200moe")
    return path


def sources() -> list[str]:
    return sorted(
        os.path.join(CSRC, name) for name in os.listdir(CSRC) if name.endswith(".cu")
    )


def _newest_input_mtime() -> float:
    paths = sources() + [os.path.join(CSRC, n) for n in os.listdir(CSRC)]
    paths += [os.path.join(INCLUDE, n) for n in os.listdir(INCLUDE)]
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def up_to_date() -> bool:
    return os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= _newest_input_mtime()


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", src, "-o", obj]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{result.stdout}\n{result.stderr}")
    if result.stderr.strip():
        sys.stderr.write(result.stderr)
    return obj


def _object_is_fresh(src: str) -> bool:
    """An object is reused when newer than its source, the shared headers and this script."""
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    if not os.path.exists(obj):
        return False
    deps = [src, os.path.abspath(__file__)]
    deps += [os.path.join(CSRC, n) for n in os.listdir(CSRC) if n.endswith(".cuh")]
    deps += [os.path.join(INCLUDE, n) for n in os.listdir(INCLUDE)]
    return os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps)


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None,
          verbose: bool = False) -> str:
    """Compile the kernel sources that changed and link LIB_PATH; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    extra = list(extra or [])
    if verbose:
        extra += ["-Xptxas", "-v"]
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)

    def obj_for(src: str) -> str:
        if not force and not verbose and not extra and _object_is_fresh(src):
            return os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        return _compile(src, extra)

    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(obj_for, srcs))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-rdc=true", "-cudart", "static", "-o", tmp, *objs]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.ptxas_verbose))


if __name__ == "__main__":
    main()
