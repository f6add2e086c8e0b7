"""Build libpolykern.so (the sm_100a kernels) in-tree with nvcc.

``python -m polytensors_b200._build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` file for ``sm_100a`` and links them into ``polytensors_b200/lib/libpolykern.so``.
Objects go to ``poly-tensors_b200/_build/``; a source is recompiled only when it or any
header is newer than its object.  nvcc cross-compiles, so no GPU is needed.
"""

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

PACKAGE_DIR = pathlib.Path(__file__).resolve().parent
PROJECT_DIR = PACKAGE_DIR.parent
CSRC = PROJECT_DIR / "csrc"
INCLUDE = PROJECT_DIR.parent / "include"
BUILD_DIR = PROJECT_DIR / "_build"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_PATH = LIB_DIR / "libpolykern.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc():
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and pathlib.Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(obj, src, headers):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def _compile(nvcc, src, obj, verbose):
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stderr}")
    return proc.stderr


def build(verbose=False, jobs=None):
    """Compile stale sources and (re)link libpolykern.so; returns the library path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    objects = [BUILD_DIR / (s.stem + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objects) if verbose or _stale(o, s, headers)]
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
            for (src, _), log in zip(todo, pool.map(lambda so: _compile(nvcc, so[0], so[1], verbose), todo)):
                if verbose and log:
                    print(f"--- {src.name}\n{log}", file=sys.stderr)
    if todo or not LIB_PATH.exists() or any(o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart_static", "-ldl",
               "-lpthread", "-lrt"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link of libpolykern.so failed:\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
