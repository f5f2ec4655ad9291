"""In-tree build of the native libraries.

  librbln_attn.so        the C-ABI (include/rbln_attn.h): every *.cu under
                         csrc/, compiled by nvcc for sm_100a only, static cudart
  librbln_attn_torch.so  the PyTorch operator layer (csrc/torch_ops.cpp),
                         linked against librbln_attn.so (rpath $ORIGIN)

Both land in torch_rbln_b200/_lib/. Objects go to <repo>/_build/. nvcc
cross-compiles without a GPU, so this runs on a CPU-only host too.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
PROJ = os.path.dirname(PKG)                  # torch-rbln_b200/
REPO = os.path.dirname(PROJ)
CSRC = os.path.join(PROJ, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIBDIR = os.path.join(PKG, "_lib")
OBJDIR = os.path.join(REPO, "_build")
CABI_SO = os.path.join(LIBDIR, "librbln_attn.so")
TORCH_SO = os.path.join(LIBDIR, "librbln_attn_torch.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _cuda_include() -> str:
    return os.path.join(os.path.dirname(os.path.dirname(_nvcc())), "include")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)


def build(verbose: bool = False, force: bool = False) -> list[str]:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    cus = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    nvcc = _nvcc()
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
                    "-diag-suppress", "177", "--expt-relaxed-constexpr"]

    def compile_cu(src: str) -> str:
        obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
        if force or _stale(obj, [src] + headers):
            _run([nvcc] + flags + ["-c", src, "-o", obj], verbose)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(cus)))) as ex:
        objs = list(ex.map(compile_cu, cus))
    if force or _stale(CABI_SO, objs):
        _run([nvcc] + ARCH + ["-shared", "-o", CABI_SO] + objs, verbose)

    import torch.utils.cpp_extension as ce
    import torch

    src = os.path.join(CSRC, "torch_ops.cpp")
    if force or _stale(TORCH_SO, [src, CABI_SO] + headers):
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        inc = []
        for p in ce.include_paths() + [_cuda_include(), INCLUDE]:
            inc += ["-I", p]
        libs = []
        for p in ce.library_paths():
            libs += ["-L", p, f"-Wl,-rpath,{p}"]
        cmd = (["g++", "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
                "-DTORCH_API_INCLUDE_EXTENSION_H", src, "-o", TORCH_SO] + inc + libs +
               ["-L", LIBDIR, "-lrbln_attn", "-Wl,-rpath,$ORIGIN", "-lc10", "-lc10_cuda", "-ltorch",
                "-ltorch_cpu", "-ltorch_cuda"])
        _run(cmd, verbose)
    return [CABI_SO, TORCH_SO]


if __name__ == "__main__":
    for p in build(verbose="-v" in sys.argv, force="-f" in sys.argv):
        print(p)
