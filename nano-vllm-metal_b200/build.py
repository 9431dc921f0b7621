"""Build libnvm_attn.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python nano-vllm-metal_b200/build.py [--force] [--jobs N]

Each .cu under csrc/ is compiled to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and the objects are
linked into nano_vllm_b200/libnvm_attn.so (static CUDA runtime, no -lcuda: the
driver's tensor-map encoder is fetched through cudaGetDriverEntryPoint).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "nano_vllm_b200", "libnvm_attn.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "nvm_attn.h"))
    return hs


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sources()
    extra = extra or []
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_verbose else []
    print(build(force=args.force or args.ptxas_verbose, jobs=args.jobs, extra=extra))
