"""Builds the CUDA library of the denoiser path in-tree.

    python sana.cpp_b200/build.py [--force] [--verbose-ptxas]

Compiles ``csrc/*.cu`` for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) and
links ``lib/libsana_cuda.so`` (CUDA runtime linked statically, C ABI of
``include/sana_cuda.h``), then the C++17 host layer ``host/*.cpp`` (the reference's
transformer.h / transformer_ops.h / scheduler.h entry points over that C ABI) into
``lib/libsana_shim.so``; ``host/tensor.cpp`` is left out of it (a sana.cpp build brings its own
Tensor). ``host/frontend/*.cpp`` (weights_io.h, torch_rng.h and the text-encoder stand-in of
gemma_encoder.h, which a sana.cpp build without ggml / llama.cpp lacks) become
``lib/libsana_frontend.so``. Objects go to ``build/`` (git-ignored); the ``.so`` files stay in
the tree so they travel with the repository snapshot.

``build_reference_frontends(ref_root)`` compiles the reference's own front ends, unmodified
(``tests/bench_full_pipeline.cpp`` and ``src/infer_main.cpp``), against these libraries into
``lib/bench_full_pipeline`` and ``lib/sana_infer``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "build")
LIB = os.path.join(HERE, "lib")
SO = os.path.join(LIB, "libsana_cuda.so")
SHIM_SO = os.path.join(LIB, "libsana_shim.so")
FRONTEND_SO = os.path.join(LIB, "libsana_frontend.so")
INCLUDE = os.path.join(ROOT, "include")
HOST = os.path.join(HERE, "host")
CXX = os.environ.get("CXX_HOST", "g++")
HOST_FLAGS = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-I", INCLUDE, "-I", os.path.join(HOST, "include"),
              "-I", HOST]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
                "--diag-suppress", "177"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool, ptxas_v: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    if force or _stale(obj, [src] + _headers()):
        cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if ptxas_v else []) + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if ptxas_v:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, ptxas_v), sources))
    if force or _stale(SO, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", SO] + objs + ["-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_shim(force)
    build_frontend(force)
    return SO


def _host_headers():
    return glob.glob(os.path.join(HOST, "*.h")) + glob.glob(os.path.join(HOST, "include", "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _host_objects(srcs, tag: str, force: bool):
    objs = []
    for src in srcs:
        obj = os.path.join(OBJ, tag + os.path.basename(src)[:-4] + ".o")
        if force or _stale(obj, [src] + _host_headers()):
            r = subprocess.run([CXX] + HOST_FLAGS + ["-c", src, "-o", obj], capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"{CXX} failed for {src}:\n{r.stdout}\n{r.stderr}")
        objs.append(obj)
    return objs


def _link_shared(target: str, objs, force: bool) -> str:
    if force or _stale(target, objs + [SO]):
        cmd = [CXX, "-shared", "-o", target] + objs + ["-L", LIB, "-lsana_cuda", "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link of {target} failed:\n{r.stdout}\n{r.stderr}")
    return target


def build_shim(force: bool = False) -> str:
    """lib/libsana_shim.so from host/*.cpp except tensor.cpp, linked against libsana_cuda.so."""
    srcs = sorted(s for s in glob.glob(os.path.join(HOST, "*.cpp")) if os.path.basename(s) != "tensor.cpp")
    return _link_shared(SHIM_SO, _host_objects(srcs, "host_", force), force)


def build_frontend(force: bool = False) -> str:
    """lib/libsana_frontend.so from host/frontend/*.cpp, linked against libsana_cuda.so."""
    srcs = sorted(glob.glob(os.path.join(HOST, "frontend", "*.cpp")))
    return _link_shared(FRONTEND_SO, _host_objects(srcs, "frontend_", force), force)


# The reference's front ends (path inside its tree -> executable under lib/).
REFERENCE_FRONTENDS = {"tests/bench_full_pipeline.cpp": "bench_full_pipeline", "src/infer_main.cpp": "sana_infer"}


def build_reference_frontends(ref_root: str, force: bool = False) -> dict:
    """Compiles the reference's front ends from its tree, unmodified, against this repository's
    headers (host/include, include) and libraries: Tensor from host/tensor.cpp, the hot path from
    libsana_shim.so, weights_io / torch_rng / the encoder stand-in from libsana_frontend.so.
    Each source is fed to the compiler on standard input from build/ (which holds no headers),
    so that its quoted includes resolve to host/include rather than to the reference headers
    beside it. Returns {source: executable}."""
    tensor_obj = _host_objects([os.path.join(HOST, "tensor.cpp")], "frontend_", force)[0]
    out = {}
    for rel, name in REFERENCE_FRONTENDS.items():
        src = os.path.join(ref_root, rel)
        exe = os.path.join(LIB, name)
        if force or _stale(exe, [src, tensor_obj, SHIM_SO, FRONTEND_SO] + _host_headers()):
            cmd = [CXX, "-std=c++17", "-O2", "-iquote", os.path.join(HOST, "include"), "-iquote", INCLUDE,
                   "-x", "c++", "-", "-x", "none", tensor_obj, "-o", exe, "-L", LIB, "-lsana_shim",
                   "-lsana_frontend", "-lsana_cuda", "-Wl,-rpath,$ORIGIN"]
            with open(src, "rb") as f:
                r = subprocess.run(cmd, stdin=f, capture_output=True, cwd=OBJ)
            r.stdout, r.stderr = r.stdout.decode(errors="replace"), r.stderr.decode(errors="replace")
            if r.returncode != 0:
                raise RuntimeError(f"build of {rel} failed:\n{r.stdout}\n{r.stderr}")
        out[rel] = exe
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--reference-root", help="also build the reference's front ends from this tree")
    a = ap.parse_args()
    print(build(a.force, a.verbose_ptxas))
    if a.reference_root:
        for exe in build_reference_frontends(a.reference_root, a.force).values():
            print(exe)
