"""Build librlenv.so in place from csrc/*.cu for sm_100a.

Each translation unit is compiled by nvcc in parallel; the objects are linked
into librlenv.so next to this file, where rlenv_lib.py loads it. The build is
incremental: a unit is recompiled only when it or a header it may include is
newer than its object.

Run as a script (`python rlenv_build.py [-v]`) or call build().
"""

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJ = HERE / "_build"
LIB = HERE / "librlenv.so"
# the check build: the same sources with -DRLENV_CHECKS (kernels record bad actions and
# non-finite outputs in a device word that rlenv_checks_status reads)
OBJ_CHECKS = HERE / "_build_checks"
LIB_CHECKS = HERE / "librlenv_checks.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build librlenv.so")
    return exe


def _includes(path, seen=None):
    """Every local header a source reaches through #include "..." (recursively)."""
    import re

    seen = set() if seen is None else seen
    for name in re.findall(r'^#include "([^"]+)"', path.read_text(), flags=re.M):
        for d in (CSRC, INCLUDE):
            h = d / name
            if h.exists() and h not in seen:
                seen.add(h)
                _includes(h, seen)
    return seen


def _stale(src, obj):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in _includes(src))


def _compile(src, obj, extra, verbose):
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(verbose=False, ptxas_verbose=False, jobs=None, checks=False):
    """Compile every csrc/*.cu for sm_100a and link librlenv.so (librlenv_checks.so with
    checks=True). Returns its path."""
    obj_dir, lib = (OBJ_CHECKS, LIB_CHECKS) if checks else (OBJ, LIB)
    obj_dir.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    extra = (["-Xptxas", "-v"] if ptxas_verbose else []) + (["-DRLENV_CHECKS"] if checks else [])
    todo = [s for s in sources if ptxas_verbose or _stale(s, obj_dir / (s.stem + ".o"))]
    logs = {}
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, obj_dir / (s.stem + ".o"), extra, verbose): s for s in todo}
            for f in concurrent.futures.as_completed(futs):
                logs[futs[f].name] = f.result()
    objs = [obj_dir / (s.stem + ".o") for s in sources]
    if todo or not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)
    if ptxas_verbose:
        for name in sorted(logs):
            print(f"==== {name}\n{logs[name]}")
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv, checks="--checks" in sys.argv))
