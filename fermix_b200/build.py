"""Build libfermix_b200.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

Each csrc/*.cu is compiled to an object of its own, in parallel, then linked into one
shared library:

    python -m fermix_b200.build [--force] [-j N]
"""

import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
OBJ_DIR = os.path.join(OUT_DIR, "obj")
OUT = os.path.join(OUT_DIR, "libfermix_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC"]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def units():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.inl")) +
                  glob.glob(os.path.join(INCLUDE, "*.h")))


def sources():
    return units() + headers()


def _obj(cu):
    return os.path.join(OBJ_DIR, os.path.basename(cu)[:-3] + ".o")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def up_to_date():
    return not _stale(OUT, sources() + [os.path.abspath(__file__)])


def _compile(cu, verbose):
    obj = _obj(cu)
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-c", "-o", obj + ".tmp", cu]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(cu)}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout + r.stderr, flush=True)
    os.replace(obj + ".tmp", obj)
    return obj


def build(force=False, verbose=False, jobs=None):
    if not force and up_to_date():
        return OUT
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdr = headers() + [os.path.abspath(__file__)]
    todo = [cu for cu in units() if force or _stale(_obj(cu), [cu] + hdr)]
    jobs = jobs or max(1, min(len(todo), os.cpu_count() or 1))
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as ex:
            for f in [ex.submit(_compile, cu, verbose) for cu in todo]:
                f.result()
    objs = [_obj(cu) for cu in units()]
    cmd = [_nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", OUT + ".tmp", *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    j = None
    if "-j" in sys.argv:
        j = int(sys.argv[sys.argv.index("-j") + 1])
    print(build(force="--force" in sys.argv, verbose=True, jobs=j))
