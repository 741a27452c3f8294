"""Build recipe for libspk.so (sm_100a), in-tree.

Each ``csrc/*.cu`` file is compiled to an object with nvcc in parallel, then
linked into ``spikingtransformer_b200/libspk.so``.  The CUDA runtime is linked
statically; the driver API entry point used for TMA descriptors is resolved at
run time (``cudaGetDriverEntryPoint``), so the library needs no ``-lcuda``.

    python -m spikingtransformer_b200.build [--force] [-j N]
"""

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libspk.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I" + INCLUDE]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _compile(src, extra):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc()] + ARCH + FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, " ".join(cmd), r.stderr[-8000:]))
    return obj, r.stderr


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in _sources() + _headers() + [__file__])


def build(force=False, jobs=None, verbose=False, ptxas_info=False):
    """Compile every CUDA source for sm_100a and link libspk.so (no-op if fresh)."""
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    srcs = _sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, extra), srcs))
    objs = [o for o, _ in results]
    if verbose or ptxas_info:
        for (o, err), s in zip(results, srcs):
            if err.strip():
                sys.stderr.write("== %s\n%s\n" % (os.path.basename(s), err))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr[-8000:]))
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=True, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
