"""Build the native library ``libmtc_b200.so`` in-tree with nvcc for sm_100a.

    python -m tensorpack_b200.build [--force]

Objects go to ``tensorpack_b200/_build/``; the shared library is written next
to this file so it travels with the package.  The library carries a SHA-256
of its sources, headers and compiler flags (a marker string in its read-only
data); a rebuild happens when that hash differs from the sources on disk, so
a stale prebuilt library shipped next to newer sources is never used.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmtc_b200.so")
# CPU model of the strip-stream decode kernel used by the format tests (host
# code only; never loaded by the package).
MODEL_SRC = os.path.join(ROOT, "tests", "native", "strip_model.cu")
MODEL_LIB = os.path.join(ROOT, "tests", "native", "libstrip_model.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    out = list(sources())
    for d in (CSRC, INCLUDE):
        out += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh"))]
    return out


HASH_MARKER = b"MTC_SOURCE_HASH="


def source_hash() -> str:
    """SHA-256 over the compiler flags and every source and header (by name
    and content), in a fixed order."""
    h = hashlib.sha256()
    h.update(" ".join(ARCH + FLAGS[:-1]).encode())
    for p in sorted(_deps(), key=os.path.basename):
        h.update(os.path.basename(p).encode() + b"\0")
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def library_hash(path: str = LIB):
    """The source hash recorded in a built library, or None."""
    try:
        with open(path, "rb") as f:
            data = f.read()
    except OSError:
        return None
    i = data.find(HASH_MARKER)
    if i < 0:
        return None
    return data[i + len(HASH_MARKER):i + len(HASH_MARKER) + 64].decode("ascii", errors="replace")


def needs_build() -> bool:
    return library_hash(LIB) != source_hash()


def build(force: bool = False, verbose: bool = False, defines=(), out: str = LIB, build_dir: str = BUILD) -> str:
    """Compile every csrc/*.cu and link ``out``; ``defines`` are extra -D flags."""
    if out == LIB and not defines and not force and not needs_build():
        return LIB
    os.makedirs(build_dir, exist_ok=True)
    cc = nvcc()
    digest = source_hash()

    def compile_one(src):
        obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
        cmd = [cc, *ARCH, *FLAGS, *("-D" + d for d in defines), "-c", src, "-o", obj]
        if os.path.basename(src) == "mtc_abi.cu":
            cmd.insert(-4, f"-DMTC_SOURCE_HASH=\"{digest}\"")
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
        if verbose and r.stderr:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = out + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, out)
    return out


def build_strip_model(force: bool = False) -> str:
    """Compile the tests' CPU model of the strip kernel (host code, nvcc as
    the C++ front end so that it shares mtc_strip.cuh with the kernel)."""
    deps = [MODEL_SRC, os.path.join(CSRC, "mtc_strip.cuh")]
    if (not force and os.path.exists(MODEL_LIB)
            and all(os.path.getmtime(d) <= os.path.getmtime(MODEL_LIB) for d in deps)):
        return MODEL_LIB
    tmp = MODEL_LIB + ".tmp"
    cmd = [nvcc(), "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-shared",
           MODEL_SRC, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {MODEL_SRC}:\n{r.stderr}")
    os.replace(tmp, MODEL_LIB)
    return MODEL_LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    print(build_strip_model(force=a.force))


if __name__ == "__main__":
    main()
