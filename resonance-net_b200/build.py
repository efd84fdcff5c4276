"""Build recipe for librnet_b200.so (sm_100a) — plain nvcc, no CMake.

Every CUDA source under csrc/ and every C++ source under host/ is compiled to
an object in _build/ and linked into one shared library next to this file.
Objects are rebuilt when their source or any header in the tree is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "librnet_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "-I", os.path.join(ROOT, "include"), "-I", os.path.join(HERE, "csrc"),
          "-DRNET_BUILD_LIB=1"]


def _headers() -> list[str]:
    pats = ["csrc/*.cuh", "csrc/*.h", "host/*.h"]
    out = [p for pat in pats for p in glob.glob(os.path.join(HERE, pat))]
    out += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return out


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) +
                  glob.glob(os.path.join(HERE, "host", "*.cpp")))


def _obj(src: str) -> str:
    rel = os.path.relpath(src, HERE).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src: str) -> tuple[str, int, str]:
    obj = _obj(src)
    cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, *COMMON, "-x", "cu", *ARCH, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r.returncode, r.stdout + r.stderr


def build(verbose: bool = False, jobs: int | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr_mtime = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    srcs = _sources()
    todo = []
    for s in srcs:
        o = _obj(s)
        if not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_mtime):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for src, rc, log in ex.map(_compile, todo):
                if verbose or rc != 0:
                    sys.stderr.write(f"[nvcc] {os.path.relpath(src, ROOT)}\n{log}")
                if rc != 0:
                    raise RuntimeError(f"nvcc failed for {src}")
    objs = [_obj(s) for s in srcs]
    if (not os.path.exists(LIB) or todo or
            os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
