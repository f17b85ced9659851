"""In-tree build of the two native libraries of dvattn_b200.

* ``libdvattn_b200.so`` -- the CUDA kernels behind the C ABI of ``include/dvattn_b200.h``,
  compiled by nvcc for sm_100a only (static cudart, no torch dependency).
* ``dvatt.abi3.so``    -- the ``torch.ops.libdvatt`` registration (same file name as the
  reference extension), a thin C++ layer over the C ABI linked against torch.

Run ``python dvattn_b200/_build.py`` (or ``__graft_entry__.build()``).  Outputs land next to
this file; sources are rebuilt only when newer than their outputs.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(ROOT, "_build")
CAPI_SO = os.path.join(HERE, "libdvattn_b200.so")
TORCH_SO = os.path.join(HERE, "dvatt.abi3.so")

CU_SOURCES = ["decode.cu", "rope.cu", "merge.cu", "capi.cu", "noalloc.cu", "peer.cu", "prefill.cu", "append.cu", "views.cu",
              "rope_tables.cu"]
HEADERS = ["common.cuh", "schedule.cuh", "decode.cuh", "tma_host.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return os.path.join(home, "bin", "nvcc")


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def build_capi(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "dvattn_b200.h")]
    objs = []
    jobs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if _newer(o, [s] + hdrs):
            jobs.append([_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                         "-Xptxas", "-v" if verbose else "-O3", "-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        list(ex.map(_run, jobs))
    if _newer(CAPI_SO, objs):
        _run([_nvcc(), *ARCH, "-shared", "-cudart", "static", *objs, "-o", CAPI_SO])
    return CAPI_SO


def build_torch_ops() -> str:
    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, os.path.join(ROOT, "include", "dvattn_b200.h"), CAPI_SO]
    if not _newer(TORCH_SO, deps):
        return TORCH_SO
    inc = ce.include_paths(device_type="cuda")
    libs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", src, "-o", TORCH_SO]
    for i in inc:
        cmd += ["-isystem", i]
    for d in libs:
        cmd += ["-L", d]
    cmd += ["-L", HERE, "-ldvattn_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
            "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    return TORCH_SO


def build(verbose: bool = False) -> None:
    build_capi(verbose)
    build_torch_ops()


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", CAPI_SO, TORCH_SO)
