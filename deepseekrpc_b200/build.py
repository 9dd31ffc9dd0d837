"""In-tree build of the sm_100a kernels and their bindings.

Produces, next to this file:
  libdsr_b200.so               C ABI (include/dsr_b200.h); CUDA runtime linked statically
  deepseekrpc_cuda<ext>.so      thin PyTorch extension with the reference module's
                               op names (native/bindings.cpp:20-26), layered on the C ABI

Usage: python -m deepseekrpc_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libdsr_b200.so"
EXT_NAME = "deepseekrpc_cuda"

CUDA_SOURCES = ["legacy_ops.cu", "topk.cu", "topk_noalloc.cu", "indexer_decode.cu", "indexer_prefill.cu",
                "candidates.cu", "mla_decode.cu", "append.cu", "decode_step.cu", "p2p.cu", "pool.cu"]
HOST_SOURCES = ["host_common.cpp"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> Path:
    for candidate in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if candidate and (Path(candidate) / "bin" / "nvcc").exists():
            return Path(candidate)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found; the sm_100a kernels cannot be built")


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(Path(d).stat().st_mtime <= t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    proc = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(map(str, cmd))}\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout, proc.stderr, sep="", flush=True)
    return proc


def build_library(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    home = cuda_home()
    nvcc = home / "bin" / "nvcc"
    BUILD.mkdir(exist_ok=True)
    # every source includes some of the headers: any header change rebuilds everything
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "dsr_b200.h"]
    common = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-I", str(ROOT / "include")]
    jobs = []
    objects = []
    for src in CUDA_SOURCES:
        obj = BUILD / (src + ".o")
        objects.append(obj)
        if force or not _newer(obj, [CSRC / src, *headers]):
            cmd = [nvcc, *ARCH, *common, "-c", CSRC / src, "-o", obj]
            if ptxas_verbose:
                cmd[1:1] = ["-Xptxas", "-v"]
            jobs.append(cmd)
    for src in HOST_SOURCES:
        obj = BUILD / (src + ".o")
        objects.append(obj)
        if force or not _newer(obj, [CSRC / src, *headers]):
            jobs.append(["g++", "-O3", "-std=c++17", "-fPIC", "-I", home / "include", "-I", ROOT / "include",
                         "-c", CSRC / src, "-o", obj])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as pool:
            results = list(pool.map(lambda c: _run(c, verbose or ptxas_verbose), jobs))
        if ptxas_verbose:
            for r in results:
                sys.stdout.write(r.stderr)
    if force or jobs or not _newer(LIB, objects):
        _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objects], verbose)
    return LIB


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    target = PKG / (EXT_NAME + suffix)
    src = CSRC / "torch_ext.cpp"
    deps = [src, ROOT / "include" / "dsr_b200.h", LIB]
    if not force and _newer(target, deps):
        return target
    home = cuda_home()
    includes = []
    for p in cpp_extension.include_paths(device_type="cuda"):
        includes += ["-I", p]
    includes += ["-I", str(home / "include"), "-I", str(ROOT / "include"),
                 "-I", sysconfig.get_paths()["include"]]
    libdirs = []
    for p in cpp_extension.library_paths(device_type="cuda"):
        libdirs += ["-L", p, f"-Wl,-rpath,{p}"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-DTORCH_EXTENSION_NAME={EXT_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *includes, str(src), "-o", str(target), *libdirs,
           "-L", str(PKG), "-ldsr_b200", "-Wl,-rpath,$ORIGIN",
           "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda"]
    _run(cmd, verbose)
    return target


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False):
    lib = build_library(force=force, verbose=verbose, ptxas_verbose=ptxas_verbose)
    ext = build_extension(force=force, verbose=verbose)
    return lib, ext


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas", action="store_true", help="print register / spill / smem usage")
    parser.add_argument("--lib-only", action="store_true")
    args = parser.parse_args(argv)
    if args.lib_only:
        print(build_library(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas))
    else:
        print(*build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas), sep="\n")


if __name__ == "__main__":
    main()
