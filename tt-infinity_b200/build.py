"""Build the B200 KV block store library (libkvs_b200.so) in-tree for sm_100a.

    python tt-infinity_b200/build.py [--debug]

Compiles csrc/*.cu and csrc/*.cpp with nvcc into kvcache_manager/libkvs_b200.so (the C ABI of
include/kvs.h). nvcc cross-compiles for sm_100a without a GPU.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "kvcache_manager" / "libkvs_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def needs_build(out: Path) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + [ROOT / "include" / "kvs.h"]
    return any(p.stat().st_mtime > t for p in deps)


FAST_SRC = CSRC / "pyext" / "kvs_fastcall.c"


def fastcall_path() -> Path:
    import sysconfig

    return PKG / "kvcache_manager" / ("_fastcall" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_fastcall(force: bool = False) -> Path:
    """The CPython module of the block calls' hot path (gcc; it calls the library through
    function pointers, so it does not link against it)."""
    import sysconfig

    import numpy as np

    out = fastcall_path()
    if not force and out.exists() and out.stat().st_mtime > FAST_SRC.stat().st_mtime:
        return out
    cc = os.environ.get("CC", "gcc")
    cmd = [cc, "-O2", "-shared", "-fPIC", "-Wall", "-I", sysconfig.get_paths()["include"], "-I", np.get_include(),
           str(FAST_SRC), "-o", str(out) + ".tmp"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("gcc failed building the _fastcall module")
    os.replace(str(out) + ".tmp", out)
    return out


def build(debug: bool = False, verbose: bool = False, force: bool = False) -> Path:
    build_fastcall(force)
    if not force and not needs_build(OUT):
        return OUT
    flags = ARCH + [
        "-std=c++17",
        "-lineinfo",
        "-O0" if debug else "-O3",
        "-Xcompiler", "-fPIC,-Wall,-Wno-unused-function",
        "-shared",
        "-I", str(ROOT / "include"),
        "-I", str(CSRC),
        "-o", str(OUT) + ".tmp",
    ]
    if verbose:
        flags += ["-Xptxas", "-v"]
    cmd = [NVCC, *flags, *map(str, sources())]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libkvs_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    build(debug="--debug" in sys.argv, verbose="-v" in sys.argv, force=True)
    print(OUT)
