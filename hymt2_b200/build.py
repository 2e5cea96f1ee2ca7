"""In-tree build of the native libraries (nvcc / gcc, no JIT cache).

  hymt2_b200/libhymt2_cuda.so  standalone backend (ctypes: tests, bench)
  hymt2_b200/libhymt2_cuda.a   the same objects for linking into the hymt2
                               host library in place of its src/cuda.c
  hymt2_b200/libhysynth.so     synthetic GGUF writer
Run `python -m hymt2_b200.build` or call build_all().
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

from . import _paths

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-Xcompiler", "-Wall"]
CSRC = os.path.join(_paths.PKG, "csrc")
SOURCES = ["hy_backend.cu"]
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith(".cuh"))  # every header the sources include


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(home, "bin", "nvcc")
    return p if os.path.exists(p) else (shutil.which("nvcc") or "nvcc")


def _cc() -> str:
    for c in ("/usr/bin/gcc", shutil.which("gcc") or "", shutil.which("cc") or ""):
        if c and os.path.exists(c):
            return c
    return "gcc"


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str], cwd: str | None = None) -> None:
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout[-4000:], r.stderr[-4000:]))


def build_backend(force: bool = False, trace: bool = False) -> None:
    """The product backend (.so and .a); with trace=True instead the
    measurement variant libhymt2_cuda_trace.so (-DHYK_TRACE: per-kernel and
    persistent-kernel %globaltimer timelines)."""
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps += [os.path.join(_paths.ROOT, "include", h) for h in ("hy_device_abi.h", "hymt2_cuda.h")]
    deps.append(os.path.abspath(__file__))
    so, ar = (_paths.TRACE_LIB, None) if trace else (_paths.BACKEND_LIB, _paths.BACKEND_ARCHIVE)
    if not force and not _stale(so, deps) and (ar is None or not _stale(ar, deps)):
        return
    objdir = os.path.join(_paths.PKG, "_build", "trace" if trace else "product")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        _run([_nvcc(), *ARCH, *NVCC_FLAGS, *(["-DHYK_TRACE"] if trace else []), "-c", os.path.join(CSRC, src),
              "-o", obj])
        objs.append(obj)
    tmp = so + ".tmp"
    _run([_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lrt", "-ldl", "-lpthread"])
    os.replace(tmp, so)
    if ar:
        if os.path.exists(ar):
            os.remove(ar)
        _run(["ar", "rcs", ar, *objs])


def build_synth(force: bool = False) -> None:
    src = os.path.join(_paths.PKG, "synth", "hysynth.c")
    hdr = os.path.join(_paths.PKG, "synth", "hysynth.h")
    out = _paths.SYNTH_LIB
    if not force and not _stale(out, [src, hdr]):
        return
    _run([_cc(), "-O2", "-fPIC", "-shared", "-Wall", "-o", out + ".tmp", src, "-lm"])
    os.replace(out + ".tmp", out)


def build_oracle(reference: str | None = None) -> None:
    """Test-only checkers under oracle/ (see oracle/Makefile): always the C
    restatement; the reference's own CPU library and the drop-in link only
    when `reference` names a checkout of the reference (its src/)."""
    odir = os.path.join(_paths.ROOT, "oracle")
    env_cc = "CC=" + _cc()
    _run(["make", "-s", env_cc, "orc"], cwd=odir)
    if reference and os.path.isdir(os.path.join(reference, "src")):
        _run(["make", "-s", env_cc, "REF=" + reference, "ref"], cwd=odir)
        if os.path.exists(_paths.BACKEND_ARCHIVE):
            _run(["make", "-s", env_cc, "REF=" + reference, "dropin"], cwd=odir)


def build_all(force: bool = False, reference: str | None = None) -> None:
    build_synth(force)
    build_backend(force)
    build_oracle(reference)


if __name__ == "__main__":
    if "--trace" in sys.argv:
        build_backend(force="--force" in sys.argv, trace=True)
        print("built:", _paths.TRACE_LIB)
        sys.exit(0)
    build_all(force="--force" in sys.argv, reference=os.environ.get("HYMT2_REFERENCE"))
    print("built:", _paths.BACKEND_LIB, _paths.BACKEND_ARCHIVE, _paths.SYNTH_LIB)
