"""Build recipe for the native parts: the product library, its CLI and the
CPU oracle used by the tests.

    python maxim-rs_b200/build.py            # incremental
    python maxim-rs_b200/build.py --clean    # from scratch

Outputs (in-tree, git-ignored, shipped with the repository snapshot):
    maxim-rs_b200/libmaxim_b200.so   host contract + GPU executor + sm_100a kernels
    maxim-rs_b200/maxim              the PNG-in / PNG-out CLI
    oracle/_build/libmaxim_oracle.so the CPU restatement of the reference
                                     executor with its own copy of the host
                                     contract (test infrastructure only)

CUDA code is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`);
nvcc cross-compiles it without a GPU. The CUDA runtime is linked statically and
the driver API is reached through cudaGetDriverEntryPoint, so the library needs
nothing from the system at run time beyond libcuda.so (loaded by the runtime)
and zlib.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INC = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
ORACLE = os.path.join(ROOT, "oracle")
ORACLE_BUILD = os.path.join(ORACLE, "_build")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_INC = os.path.join(os.path.dirname(os.path.dirname(NVCC)), "include")
CXXFLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter", "-I" + INC, "-I" + CSRC,
            "-I" + CUDA_INC]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + INC, "-I" + CSRC,
                  "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]

LIB = os.path.join(PKG, "libmaxim_b200.so")
CLI = os.path.join(PKG, "maxim")
ORACLE_LIB = os.path.join(ORACLE_BUILD, "libmaxim_oracle.so")
# The host-contract sources the oracle library carries its own copy of.
ORACLE_HOST_SOURCES = ["capi_host.cpp", "config.cpp", "image.cpp", "model.cpp", "safetensors.cpp", "weights.cpp"]


def _newer(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers(d):
    return [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh"))] + \
        [os.path.join(INC, f) for f in os.listdir(INC)]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n%s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return r.stdout + r.stderr


def build(verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(ORACLE_BUILD, exist_ok=True)
    hdrs = _headers(CSRC)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith((".cpp", ".cu")) and f != "cli.cpp")
    jobs, objs = [], []
    for f in srcs:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if _newer(obj, [src] + hdrs):
            if f.endswith(".cu"):
                jobs.append([NVCC] + NVFLAGS + ["-c", src, "-o", obj])
            else:
                jobs.append(["g++"] + CXXFLAGS + ["-c", src, "-o", obj])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for out in ex.map(_run, jobs):
            logs.append(out)
    if jobs or not os.path.exists(LIB):
        logs.append(_run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lz", "-lpthread", "-ldl", "-lrt"]))
    cli_src = os.path.join(CSRC, "cli.cpp")
    if os.path.exists(cli_src) and _newer(CLI, [cli_src, LIB] + hdrs):
        logs.append(_run(["g++"] + CXXFLAGS + [cli_src, "-o", CLI, "-L" + PKG, "-lmaxim_b200",
                                               "-Wl,-rpath,$ORIGIN"]))
    # The oracle library: the CPU executor plus its own copy of the host
    # contract (plan builder, safetensors, image pipeline), compiled with
    # hidden visibility and re-exported under mxo_ names, so a CPU-only run
    # needs nothing from the product library.
    osrcs = [os.path.join(ORACLE, "exec_cpu.cpp"), os.path.join(ORACLE, "host_api.cpp")] + \
        [os.path.join(CSRC, f) for f in ORACLE_HOST_SOURCES]
    if _newer(ORACLE_LIB, osrcs + hdrs):
        # No FMA contraction: the reference's accumulations are separate
        # multiplies and adds, and contracting them changes every rounding.
        logs.append(_run(["g++", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-std=c++17", "-fPIC", "-shared",
                          "-fvisibility=hidden", "-fvisibility-inlines-hidden", "-I" + INC, "-I" + CSRC] + osrcs +
                         ["-o", ORACLE_LIB, "-lz", "-lpthread"]))
    if verbose:
        for l in logs:
            if l.strip():
                print(l)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    if a.clean:
        for p in (BUILD, ORACLE_BUILD):
            shutil.rmtree(p, ignore_errors=True)
        for p in (LIB, CLI):
            if os.path.exists(p):
                os.remove(p)
    build(verbose=a.verbose)
    print("built", LIB)


if __name__ == "__main__":
    sys.exit(main())
