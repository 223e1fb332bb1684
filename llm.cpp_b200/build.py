"""Builds libllmk.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

    python llm.cpp_b200/build.py [--force] [-j N]

Each csrc/*.cu / *.cpp is compiled to _build/*.o with nvcc (-gencode
arch=compute_100a,code=sm_100a -lineinfo) and linked into
llm.cpp_b200/libllmk.so. Objects are rebuilt when a source or any header in
csrc/ or include/ is newer. NCCL is linked from the PyTorch-bundled
nvidia-nccl wheel (same library torch.distributed loads), with an rpath to it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INC = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libllmk.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                     "-I" + INC, "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def nccl_paths() -> tuple[str | None, str | None]:
    """(include dir, lib dir) of the NCCL that torch.distributed uses."""
    try:
        import nvidia.nccl  # type: ignore
        base = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
            return inc, lib
    except Exception:
        pass
    if os.path.exists("/usr/include/nccl.h"):
        return "/usr/include", None
    return None, None


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(
        os.path.join(INC, "*.h")) + glob.glob(os.path.join(INC, "*.hpp"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    inc_nccl, lib_nccl = nccl_paths()
    extra = ["-I" + inc_nccl] if inc_nccl else []
    hdr_t = _newest_header()
    cc = nvcc()

    def obj_of(s: str) -> str:
        return os.path.join(BUILD, os.path.basename(s) + ".o")

    def needs(s: str) -> bool:
        o = obj_of(s)
        if force or not os.path.exists(o):
            return True
        return os.path.getmtime(o) < max(os.path.getmtime(s), hdr_t)

    def compile_one(s: str) -> str:
        cmd = [cc] + NVCC_FLAGS + extra + ["-c", s, "-o", obj_of(s)]
        if s.endswith(".cpp"):
            cmd = [cc] + NVCC_FLAGS + extra + ["-x", "cu", "-c", s, "-o", obj_of(s)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {os.path.basename(s)}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, file=sys.stderr)
        return s

    todo = [s for s in srcs if needs(s)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for f in cf.as_completed([ex.submit(compile_one, s) for s in todo]):
                f.result()
    objs = [obj_of(s) for s in srcs]
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        link = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        if lib_nccl:
            link += ["-L" + lib_nccl, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + lib_nccl]
        else:
            link += ["-lnccl"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def ensure_built() -> str:
    """Returns the library path, building only when it does not exist yet
    (a prebuilt library shipped next to the sources is used as-is)."""
    if os.path.exists(LIB):
        return LIB
    return build()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
