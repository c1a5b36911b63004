"""Build libb200ep.so (CUDA kernels for sm_100a + the C++ EP core) in-tree.

    python onnxruntime-mlx_b200/build.py [--force] [-j N] [--verbose-ptxas]

Objects go to onnxruntime-mlx_b200/_build/; the shared library lands next to the Python
locator package (onnxruntime-mlx_b200/onnxruntime_ep_b200/libb200ep.so) so that it travels
with the source tree.  nvcc cross-compiles for sm_100a without a GPU.
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
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "onnxruntime_ep_b200", "libb200ep.so")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
HOST_CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else (shutil.which("g++") or "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    """NCCL headers/library from the nvidia-nccl wheel that ships with torch."""
    try:
        import nvidia.nccl  # type: ignore

        base = list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:  # noqa: BLE001
        pass
    return None, None


def sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    cpp = sorted(glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))
    return cu + cpp


def headers():
    hs = glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
    hs += glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def obj_path(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "__")
    return os.path.join(BUILD, rel + ".o")


def compile_one(src, force, ptxas_v):
    obj = obj_path(src)
    newest_header = max((os.path.getmtime(h) for h in headers()), default=0)
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
        return obj, ""
    inc = ["-I", CSRC, "-I", os.path.join(ROOT, "include")]
    nccl_inc, _ = nccl_dirs()
    if nccl_inc:
        inc += ["-I", nccl_inc, "-DB200EP_HAVE_NCCL=1"]
    cmd = [NVCC, "-ccbin", HOST_CXX, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", "-c", src, "-o", obj, *inc]
    if src.endswith(".cpp"):
        cmd += ["-x", "cu"]  # host code shares the CUDA headers of the kernels
    if ptxas_v and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int = 0, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    jobs = jobs or min(8, os.cpu_count() or 4)
    logs = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(compile_one, s, force, ptxas_v) for s in srcs]
        objs = []
        for f in futs:
            o, log = f.result()
            objs.append(o)
            if log:
                logs.append(log)
    if ptxas_v:
        for log in logs:
            sys.stderr.write(log)
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(OUT) or os.path.getmtime(OUT) < newest:
        _, nccl_lib = nccl_dirs()
        link = [NVCC, "-ccbin", HOST_CXX, *ARCH, "-shared", "-o", OUT, *objs]
        if nccl_lib:
            link += ["-L", nccl_lib, "-l:libnccl.so.2", "-Xlinker", f"-rpath={nccl_lib}"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(link)}\n{r.stdout}\n{r.stderr}")
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.verbose_ptxas))


if __name__ == "__main__":
    main()
