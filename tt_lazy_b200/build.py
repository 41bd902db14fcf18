"""Build recipe for the tt_lazy B200 backend (in-tree, no JIT cache).

Produces, under ``tt_lazy_b200/lib/``:

* ``libtt_cuda.so``  -- the C-ABI backend (``include/tt_cuda.h``): every CUDA
  kernel, compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``),
  CUDA runtime linked statically.
* ``libtt_lazy.so``  -- the C++ front end (Tensor / operations / tape /
  passes / handlers) linked against ``libtt_cuda.so``.
* ``_tt_lazy*.so``   -- the pybind11 module over the front end (tests, bench).

Run ``python tt_lazy_b200/build.py`` (or ``__graft_entry__.build()``).
Objects are rebuilt only when a source or header is newer than the output.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
LIB = os.path.join(PKG, "lib")
OBJ = os.path.join(LIB, "obj")
INCLUDE = os.path.join(ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: no multiply-add contraction anywhere, so every element-wise step
# is one IEEE op (bit-exact against the reference's separate passes); the GEMM
# main loops use explicit fused multiply-adds where they want them.
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC, "-I" + OBJ]

CUDA_SOURCES = ["runtime.cu", "chain.cu", "chain_tma.cu", "chain_jit.cu", "transpose.cu", "gemm_ffma.cu", "gemm_tc.cu"]
CPP_SOURCES = ["comm.cpp"]


def _nccl_dirs():
    purelib = sysconfig.get_paths()["purelib"]
    inc = os.path.join(purelib, "nvidia", "nccl", "include")
    lib = os.path.join(purelib, "nvidia", "nccl", "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return None, None


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def _headers(*dirs):
    out = []
    for d in dirs:
        out += glob.glob(os.path.join(d, "*.h")) + glob.glob(os.path.join(d, "*.cuh")) + glob.glob(
            os.path.join(d, "*.hpp"))
    return out


def _embed_jit_source():
    """expf_ref.cuh + chain_jit_device.cuh as a C++ raw string (the NVRTC
    source prefix; NVRTC gets no include path)."""
    srcs = [os.path.join(CSRC, "expf_ref.cuh"), os.path.join(CSRC, "chain_jit_device.cuh")]
    out = os.path.join(OBJ, "chain_jit_src.inc")
    if _stale(out, srcs):
        text = "\n".join(line for s in srcs for line in open(s).read().splitlines()
                         if line.strip() != "#pragma once") + "\n"
        assert ")TTJSRC" not in text
        with open(out + ".tmp", "w") as f:
            f.write('static const char kJitDeviceSrc[] = R"TTJSRC(' + text + ')TTJSRC";\n')
        os.replace(out + ".tmp", out)
    return out


def build_cuda(verbose=False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers(CSRC, INCLUDE) + [_embed_jit_source()]
    nccl_inc, nccl_lib = _nccl_dirs()
    objs = []
    for src in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src + ".o")
        if _stale(o, [s] + hdrs):
            _run([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o + ".tmp"], verbose)
            os.replace(o + ".tmp", o)
        objs.append(o)
    for src in CPP_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src + ".o")
        if _stale(o, [s] + hdrs):
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-I" + INCLUDE, "-I" + CSRC,
                   "-I" + os.path.join(CUDA_HOME, "include"), "-c", s, "-o", o + ".tmp"]
            if nccl_inc:
                cmd.insert(1, "-DTTC_HAVE_NCCL=1")
                cmd.insert(1, "-I" + nccl_inc)
            _run(cmd, verbose)
            os.replace(o + ".tmp", o)
        objs.append(o)
    out = os.path.join(LIB, "libtt_cuda.so")
    if _stale(out, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", out + ".tmp"] + objs + [
            "-Xlinker", "-soname,libtt_cuda.so", "-ldl"]
        if nccl_lib:
            cmd += ["-L" + nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath," + nccl_lib]
        _run(cmd, verbose)
        os.replace(out + ".tmp", out)
    return out


def build_host(verbose=False) -> str | None:
    """C++ front end + pybind11 module (skipped while host/ has no sources)."""
    srcs = sorted(glob.glob(os.path.join(HOST, "*.cpp")))
    srcs = [s for s in srcs if not s.endswith("pybind_module.cpp")]
    if not srcs:
        return None
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers(HOST, INCLUDE)
    objs = []
    for s in srcs:
        o = os.path.join(OBJ, "host_" + os.path.basename(s) + ".o")
        if _stale(o, [s] + hdrs):
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-I" + INCLUDE, "-I" + HOST, "-c", s, "-o", o + ".tmp"],
                 verbose)
            os.replace(o + ".tmp", o)
        objs.append(o)
    lib = os.path.join(LIB, "libtt_lazy.so")
    if _stale(lib, objs + [os.path.join(LIB, "libtt_cuda.so")]):
        _run(["g++", "-shared", "-o", lib + ".tmp"] + objs + ["-L" + LIB, "-l:libtt_cuda.so",
             "-Wl,-rpath,$ORIGIN", "-Wl,-soname,libtt_lazy.so"], verbose)
        os.replace(lib + ".tmp", lib)
    mod_src = os.path.join(HOST, "pybind_module.cpp")
    if not os.path.exists(mod_src):
        return lib
    import pybind11

    ext = sysconfig.get_config_var("EXT_SUFFIX")
    mod = os.path.join(PKG, "_tt_lazy" + ext)
    if _stale(mod, [mod_src, lib] + hdrs):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I" + INCLUDE, "-I" + HOST,
              "-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"], mod_src,
              "-o", mod + ".tmp", "-L" + LIB, "-l:libtt_lazy.so", "-l:libtt_cuda.so",
              "-Wl,-rpath,$ORIGIN/lib"], verbose)
        os.replace(mod + ".tmp", mod)
    return lib


def build(verbose=False):
    cuda = build_cuda(verbose)
    host = build_host(verbose)
    return cuda, host


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", LIB)
