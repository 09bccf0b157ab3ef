"""Build the sm_100a libraries in-tree.

Outputs:
  esimd_learning_b200/libcek_b200.so
      the C-ABI kernel library (include/cek.h), nvcc
  python/custom_esimd_kernels_vllm/custom_esimd_kernels.so
      torch.library registration of the GEMV / add+RMSNorm / decode-helper ops (g++)
  python/custom_esimd_kernels_vllm/custom_esimd_kernels_gemm.so
      torch.library registration of the GEMM ops

The two extension modules keep the reference's module names and PyInit
symbols (csrc/xpu/torch_extension.cc:21-24, torch_extension_gemm.cc:16-20) and
sit in the reference's wrapper package, so
`from custom_esimd_kernels_vllm import custom_esimd_kernels, custom_esimd_kernels_gemm`
works as in python/custom_esimd_kernels_vllm/__init__.py:3-4.  They find
libcek_b200.so through a relative rpath.

Run: python esimd_learning_b200/build.py [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
WRAPPER = PKG.parent / "python" / "custom_esimd_kernels_vllm"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["abi.cu", "gemv_fp8.cu", "gemv_fp8_bulk.cu", "rmsnorm.cu", "elementwise.cu", "tp_allreduce.cu", "gemm_fp8_tcgen05.cu"]
EXT_MODULES = {
    "custom_esimd_kernels": "torch_extension.cc",
    "custom_esimd_kernels_gemm": "torch_extension_gemm.cc",
}
LIB_NAME = "libcek_b200.so"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} -> exit {r.returncode}")


def _nvcc_obj(src: Path, force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, [src] + _headers()):
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)])
    return obj


def build_lib(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = [CSRC / s for s in CU_SOURCES if (CSRC / s).exists()]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _nvcc_obj(s, force), srcs))
    lib = PKG / LIB_NAME
    if force or _stale(lib, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(lib), *map(str, objs)])
    return lib


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension as ce

    inc = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    cflags = [f"-I{p}" for p in inc] + [f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}",
                                      f"-I{CUDA_HOME / 'include'}",
                                      f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
                                      "-DTORCH_API_INCLUDE_EXTENSION_H"]
    ldflags = [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs] + [
        "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch"]
    return cflags, ldflags


def build_ext(force: bool = False) -> list[Path]:
    lib = PKG / LIB_NAME
    cflags, ldflags = _torch_flags()
    outs = []
    jobs = []
    for mod, src in EXT_MODULES.items():
        s = CSRC / src
        out = WRAPPER / f"{mod}.so"
        outs.append(out)
        if force or _stale(out, [s, lib] + _headers()):
            jobs.append(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", *cflags, str(s), "-o", str(out),
                         f"-L{PKG}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN/../../esimd_learning_b200", *ldflags])
    with cf.ThreadPoolExecutor(max_workers=2) as ex:
        list(ex.map(_run, jobs))
    return outs


def build(force: bool = False) -> None:
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print("built:", LIB_NAME, ", ".join(f"{m}.so" for m in EXT_MODULES))
