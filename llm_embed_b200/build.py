"""Build libllmembed_cuda.so in-tree for sm_100a with nvcc.

    python -m llm_embed_b200.build [--verbose]

Objects go to llm_embed_b200/_build/, the library to
llm_embed_b200/libllmembed_cuda.so (the file the Python binding and any
dlopen-based host load).  Sources compile in parallel; an object is rebuilt
when its .cu or any header in csrc/ is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libllmembed_cuda.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
                  "-Xptxas", "-warn-spills", "-I", os.path.join(HERE, "..", "include")]
# Extra nvcc flags (e.g. -DLE_TC_S_B=3 to build a pipeline-depth variant).
NVFLAGS += os.environ.get("LLMEMBED_NVCC_FLAGS", "").split()


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _host_compiler() -> list[str]:
    # Use the system g++ explicitly: some images export CC/CXX pointing at
    # wrappers that nvcc's host pass cannot drive.
    return ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(HERE, "..", "include", "*.h"))
    newest_hdr = max((os.path.getmtime(h) for h in headers), default=0)
    nvcc = _nvcc()
    hc = _host_compiler()

    def compile_one(src: str) -> str:
        obj = os.path.join(OBJ, os.path.splitext(os.path.basename(src))[0] + ".o")
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_hdr):
            return obj
        cmd = [nvcc, *hc, *NVFLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc, *hc, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
