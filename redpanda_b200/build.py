"""Build the sm_100a scan library ``libm3scan.so`` in-tree with nvcc.

    python -m redpanda_b200.build [--force] [--jobs N] [--ptxas-verbose]

Every ``csrc/*.cu`` file compiles to an object under ``redpanda_b200/_build``
(in parallel) and the objects link into ``redpanda_b200/libm3scan.so``.  The
library exports only the ``extern "C"`` entry points of ``include/m3scan.h``.
"""

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(PKG, "libm3scan.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the m3 scan library needs the CUDA toolkit to build")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)
            if f.endswith((".cuh", ".h"))] + [os.path.join(INCLUDE, "m3scan.h")]


def _compile(src, verbose, build_dir, extra):
    obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
    cmd = [_nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build_library(force=False, jobs=None, verbose=False, out=LIB, extra_flags=(),
                  build_dir=BUILD):
    """Compile the library if any source is newer than it; return its path.

    ``out``/``extra_flags``/``build_dir`` build a variant (e.g. ``-D`` tuning
    macros) next to the default library without touching it.
    """
    srcs = _sources()
    if (not force and os.path.exists(out)
            and os.path.getmtime(out) >= max(os.path.getmtime(f) for f in srcs + _deps())):
        return out
    os.makedirs(build_dir, exist_ok=True)
    jobs = jobs or min(len(srcs), os.cpu_count() or 1)
    logs = []
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = []
        for obj, log in ex.map(lambda s: _compile(s, verbose, build_dir, list(extra_flags)), srcs):
            objs.append(obj)
            logs.append(log)
    tmp = out + ".tmp"
    cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    if verbose:
        sys.stderr.write("\n".join(logs))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build_library(force=a.force, jobs=a.jobs, verbose=a.ptxas_verbose))


if __name__ == "__main__":
    main()
