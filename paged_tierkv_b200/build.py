"""Build the sm_100a C-ABI library ``lib/libtierkv_b200.so`` in-tree with nvcc.

    python -m paged_tierkv_b200.build [--verbose-ptxas]

The library has no PyTorch dependency: plain CUDA runtime (linked statically)
plus the driver entry point ``cuTensorMapEncodeTiled`` looked up at run time.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIBNAME = "libtierkv_b200.so"
SOURCES = ["tkv_api.cu", "tkv_decode.cu", "tkv_quant.cu", "tkv_prefill.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return os.path.join(cuda, "bin", "nvcc")


def lib_path() -> str:
    return os.path.join(LIBDIR, LIBNAME)


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False, defines: tuple[str, ...] = (),
          out: str | None = None, objdir: str | None = None) -> str:
    """Compile and link; `defines` (e.g. "TKV_STAGES_8K=12") select a variant,
    `out` / `objdir` place it elsewhere than the in-tree library."""
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = objdir or os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "tierkv_b200.h"))
    nvcc = nvcc_path()
    common = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "-I", os.path.join(ROOT, "include"), "-I", CSRC, *ARCH]
    if verbose_ptxas:
        common += ["-Xptxas", "-v"]
    common += [f"-D{d}" for d in defines]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or verbose_ptxas or _stale(o, [s] + headers):
            cmd = [nvcc, *common, "-c", s, "-o", o]
            subprocess.run(cmd, check=True)
    out = out or lib_path()
    if force or _stale(out, objs):
        tmp = out + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", *objs, "-o", tmp]
        subprocess.run(cmd, check=True)
        os.replace(tmp, out)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(verbose_ptxas=args.verbose_ptxas, force=args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
