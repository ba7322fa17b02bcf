"""Builds the package's CUDA library (reworld_b200/_lib/libreworld_b200.so) for sm_100a.

Each .cu file under csrc/ is compiled with nvcc for `-gencode
arch=compute_100a,code=sm_100a` and the objects are linked into one shared
library that the package loads with ctypes.  Run `python reworld_b200/build.py`
(by path: importing the package requires the library to exist) or call build().
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB_NAME = "libreworld_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newest_input_mtime():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(HERE, "..", "include", "reworld_b200.h"))
    files.append(os.path.abspath(__file__))
    return max(os.path.getmtime(f) for f in files if os.path.exists(f))


def lib_path():
    return os.path.join(OUT_DIR, LIB_NAME)


def build(force=False, verbose=False):
    """Compiles csrc/*.cu into _lib/libreworld_b200.so (skipped when up to date)."""
    os.makedirs(OUT_DIR, exist_ok=True)
    out = lib_path()
    if not force and os.path.exists(out) and os.path.getmtime(out) >= _newest_input_mtime():
        return out
    objs = []

    def compile_one(src):
        obj = os.path.join(OUT_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stdout.write(r.stdout + r.stderr)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = out + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-cudart=static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    for o in objs:
        os.remove(o)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
