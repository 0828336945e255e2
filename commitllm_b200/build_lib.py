"""Build libvcommit.so in-tree with nvcc for sm_100a.

    python -m commitllm_b200.build_lib          # or via __graft_entry__.build()

Each .cu file is compiled to an object (in parallel) and linked into
``commitllm_b200/libvcommit.so`` next to this file.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvcommit.so")
SOURCES = ["merkle.cu", "trace.cu", "kv_transcript.cu", "kvt_commit.cu", "int_peak.cu", "api.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if not f.endswith(".cu")]
    return hs + [os.path.join(HERE, "..", "include", "vcommit.h"), os.path.abspath(__file__)]


def _obj_stale(src: str, obj: str) -> bool:
    """An object is rebuilt when its source or any header (all of csrc/ but the
    .cu files, the C header, this script) is newer than it."""
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [os.path.join(CSRC, src)] + _headers() if os.path.exists(p))


def _compile(src: str, verbose: bool, force: bool = True) -> str:
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    if not force and not verbose and not _obj_stale(src, obj):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(HERE, "..", "include", "vcommit.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, force), SOURCES))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
