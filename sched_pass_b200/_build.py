"""Ahead-of-time build of the native parts, in-tree.

* ``sched_b200_C`` -- the sm_100a kernels and their torch bindings (nvcc,
  ``-gencode arch=compute_100a,code=sm_100a``), built with
  ``torch.utils.cpp_extension`` into ``sched_pass_b200/_build/``;
* ``sched-weave`` -- the LLVM-IR weaver (plain C++, g++), same directory;
* ``libsched_rt_host.so`` -- the host runtime library (named-global ABI,
  native KV block allocator and batch planner), g++ only.

The build output lives inside the package so that it travels with a copy of
the repository; nothing is written under the user's home directory.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)
BUILD_DIR = os.path.join(PKG_DIR, "_build")
CSRC = os.path.join(REPO, "csrc")
INCLUDE = os.path.join(REPO, "include")

EXT_NAME = "sched_b200_C"
ARCH_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]

KERNEL_SOURCES = [
    "kernels/gemm.cu",
    "kernels/attention_decode.cu",
    "kernels/attention_prefill.cu",
    "kernels/elementwise.cu",
    "kernels/moe.cu",
    "kernels/kv_tier.cu",
    "kernels/microbench.cu",
]
HOST_SOURCES = ["bindings.cpp", "comm/symm.cpp"]


def ext_sources() -> list[str]:
    srcs = []
    for rel in HOST_SOURCES + KERNEL_SOURCES:
        p = os.path.join(CSRC, rel)
        if os.path.exists(p):
            srcs.append(p)
    return srcs


def ext_path() -> str:
    return os.path.join(BUILD_DIR, EXT_NAME + ".so")


def build_extension(verbose: bool = False):
    """Compile (or confirm up to date) the kernel extension; returns the module."""
    import torch.utils.cpp_extension as ce

    os.makedirs(BUILD_DIR, exist_ok=True)
    jobs = str(max(1, min(16, os.cpu_count() or 4)))
    os.environ.setdefault("MAX_JOBS", jobs)
    return ce.load(
        name=EXT_NAME,
        sources=ext_sources(),
        extra_include_paths=[INCLUDE, os.path.join(CSRC, "kernels"), os.path.join(CSRC, "comm")],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=NVCC_FLAGS,
        extra_ldflags=["-lcuda"],
        build_directory=BUILD_DIR,
        verbose=verbose,
        with_cuda=True,
    )


WEAVE_SOURCES = ["weave/ir.cpp", "weave/cfg.cpp", "weave/passes.cpp", "weave/weave_pass.cpp", "weave/workqueue_pass.cpp",
                 "weave/main.cpp"]


def weave_binary() -> str:
    return os.path.join(BUILD_DIR, "sched-weave")


def build_weaver(verbose: bool = False) -> str:
    """g++ build of the IR weaver CLI (no LLVM libraries needed)."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in WEAVE_SOURCES if os.path.exists(os.path.join(CSRC, s))]
    if not srcs:
        return None
    out = weave_binary()
    newest = max(os.path.getmtime(s) for s in srcs + glob.glob(os.path.join(CSRC, "weave", "*.h"))
                 + [os.path.join(INCLUDE, "sched", "manifest.h"), os.path.join(INCLUDE, "sched", "abi.h")])
    if os.path.exists(out) and os.path.getmtime(out) >= newest:
        return out
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-I" + INCLUDE, "-I" + os.path.join(CSRC, "weave"), *srcs, "-o", out]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


HOSTLIB_SOURCES = ["runtime/host_runtime.cpp"]


def hostlib_path() -> str:
    return os.path.join(BUILD_DIR, "libsched_rt_host.so")


def build_hostlib(verbose: bool = False) -> str:
    """g++ build of the CPU-only host runtime library (ctypes-loadable)."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in HOSTLIB_SOURCES]
    out = hostlib_path()
    newest = max(os.path.getmtime(s) for s in srcs + [os.path.join(INCLUDE, "sched", "abi.h")])
    if os.path.exists(out) and os.path.getmtime(out) >= newest:
        return out
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-I" + INCLUDE, *srcs, "-o", out]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def build_all(verbose: bool = False) -> None:
    build_weaver(verbose)
    build_hostlib(verbose)
    build_extension(verbose)


def clean() -> None:
    shutil.rmtree(BUILD_DIR, ignore_errors=True)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built:", ext_path(), weave_binary(), hostlib_path())
