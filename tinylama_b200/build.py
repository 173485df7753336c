"""Build libtlattn.so (the CUDA path, sm_100a) in-tree with nvcc.

Objects go to tinylama_b200/_build/, the library to tinylama_b200/libtlattn.so.  Sources are
compiled in parallel; a source is rebuilt when it or any header is newer than its object.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtlattn.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]
SOURCES = ["tl_attn_api.cu", "rope_append.cu", "decode_attn.cu", "prefill_simt.cu",
           "prefill_tc.cu", "dist.cu", "decode_noalloc.cu", "decode_mma.cu", "model_gpu.cu"]


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "tl_attn.h"))
    hs.append(os.path.join(ROOT, "include", "tl_model.h"))
    return hs


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    newest = max([os.path.getmtime(path)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest and not verbose_ptxas:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


HOST_SRC = os.path.join(HERE, "host", "tl_host.cpp")
HOST_LIB = os.path.join(HERE, "libtlhost.so")
CXX = os.environ.get("CXX", "g++")


def build_host() -> str:
    """libtlhost.so: the C++ host forward pass (CPU linears) over libtlattn.so's attention.
    -ffp-contract=off keeps the reference's float32 rounding (no fused multiply-adds)."""
    deps = [HOST_SRC, os.path.join(ROOT, "include", "tl_host.h"), os.path.join(ROOT, "include", "tl_attn.h"),
            os.path.join(ROOT, "include", "tl_model.h"), LIB]
    if os.path.exists(HOST_LIB) and os.path.getmtime(HOST_LIB) >= max(os.path.getmtime(d) for d in deps):
        return HOST_LIB
    cmd = [CXX, "-O2", "-ffp-contract=off", "-fno-fast-math", "-std=c++17", "-fPIC", "-shared", "-pthread",
           "-fvisibility=hidden", HOST_SRC, "-o", HOST_LIB, "-L" + HERE, "-ltlattn", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host build failed:\n{r.stdout}\n{r.stderr}")
    return HOST_LIB


def build(verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), SOURCES))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_host()
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
