"""Build recipe for the in-tree native libraries of the Q8_0 hot path.

    libb200q8.so       the CUDA kernels + C ABI (include/b200q8.h), sm_100a only
    libb200q8_host.so  host C++: seeded input streams, thread policy, the
                       ggml-seam shim and the package decoder driver
                       (include/b200q8_host.h) over that ABI (host/*.cpp)
    synth_b200_frames  the command-line frame driver (host/cli/), over
                       libb200q8_host.so
    libb200q8_peaks.so measured int8 ceilings (peaks/): tcgen05 kind::i8,
                       mma.sync s8 and the per-block fp32 rescale (bench.py
                       --workload int8-peaks); not on the product path

Both are written next to this file so they travel with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
LIB = os.path.join(PKG, "libb200q8.so")
HOST_LIB = os.path.join(PKG, "libb200q8_host.so")
CLI = os.path.join(PKG, "synth_b200_frames")
PEAKS_LIB = os.path.join(PKG, "libb200q8_peaks.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the B200 library cannot be built")


def _cuda_home() -> str:
    nvcc = _nvcc()
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))


def _sources(d: str, exts: tuple[str, ...]) -> list[str]:
    return sorted(os.path.join(d, f) for f in os.listdir(d) if f.endswith(exts))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> list[str]:
    """Compile what is out of date; returns the built library paths."""
    include = os.path.join(ROOT, "include")
    deps = _sources(CSRC, (".cu", ".cuh", ".h")) + _sources(include, (".h",))
    if force or _stale(LIB, deps):
        cmd = [_nvcc(), *NVCC_FLAGS, "-o", LIB, os.path.join(CSRC, "libb200q8.cu")]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
    out = [LIB]
    peaks_src = os.path.join(PKG, "peaks", "int8_peaks.cu")
    if os.path.exists(peaks_src):
        if force or _stale(PEAKS_LIB, [peaks_src] + _sources(CSRC, (".cuh",)) + _sources(include, (".h",))):
            subprocess.run([_nvcc(), *NVCC_FLAGS, "-o", PEAKS_LIB, peaks_src], check=True)
        out.append(PEAKS_LIB)
    host_srcs = _sources(HOST, (".cpp",))
    cuda = _cuda_home()
    cuda_flags = [f"-I{os.path.join(cuda, 'include')}"]
    cuda_libs = [f"-L{os.path.join(cuda, 'lib64')}", "-lcudart", f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}"]
    if host_srcs:
        host_deps = host_srcs + _sources(HOST, (".h",)) + _sources(include, (".h",)) + [LIB]
        if force or _stale(HOST_LIB, host_deps):
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", f"-I{include}", *cuda_flags, "-o",
                   HOST_LIB, *host_srcs, f"-L{PKG}", "-lb200q8", *cuda_libs, "-Wl,-rpath,$ORIGIN"]
            subprocess.run(cmd, check=True)
        out.append(HOST_LIB)
    cli_srcs = _sources(os.path.join(HOST, "cli"), (".cpp",))
    if cli_srcs:
        if force or _stale(CLI, cli_srcs + _sources(include, (".h",)) + [HOST_LIB]):
            cmd = ["g++", "-O2", "-std=c++17", f"-I{include}", "-o", CLI, *cli_srcs, f"-L{PKG}", "-lb200q8_host",
                   "-lb200q8", "-Wl,-rpath,$ORIGIN"]
            subprocess.run(cmd, check=True)
        out.append(CLI)
    return out


if __name__ == "__main__":
    for p in build(force=True, verbose=True):
        print(p)
