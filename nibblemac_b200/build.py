"""Build the native parts in-tree.

    python -m nibblemac_b200.build          # libpinfer.so, libnbpq.so, oracle (and oracle/_ref)

Outputs:
  nibblemac_b200/lib/libpinfer.so   the B200 engine (CUDA sm_100a kernels + C++ host code),
                                     SONAME libpinfer.so.0.3, exports pinfer_* / nb_* only
  nibblemac_b200/lib/libnbpq.so     host Q4K quantiser for writing .pq files
  oracle/liboracle.so               CPU checker (tests only)
  oracle/_ref/                      the reference engine built from its own sources, when a
                                     reference checkout is available (tests only)
nvcc cross-compiles for sm_100a without a GPU, so this runs on any host with CUDA 12.9.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
BUILD = PKG / "_build"
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# Bit-exactness: no fast math; float ops that must round separately use IEEE intrinsics, and
# --fmad=false keeps every other expression unfused as well.
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-prec-div=true",
                     "-prec-sqrt=true", "-ftz=false", "-Xcompiler", "-fPIC,-ffp-contract=off",
                     "-I", str(ROOT / "include"), "-I", str(CSRC)]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-I", str(ROOT / "include"),
             "-I", str(CSRC), "-I", "/usr/local/cuda/include"]


def run(cmd: list[str], cwd: Path | None = None) -> None:
    print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True, cwd=cwd)


def newer(out: Path, deps: list[Path]) -> bool:
    return out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps)


def build_quant() -> Path:
    out = LIB / "libnbpq.so"
    src = CSRC / "pq_quant.c"
    if not newer(out, [src]):
        run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
             src, "-o", out, "-lm"])
    return out


def build_engine() -> Path:
    out = LIB / "libpinfer.so"
    cu = ["nb_kernels.cu", "nb_gemm.cu", "nb_engine.cu", "nb_prefill.cu", "nb_batch.cu", "nb_capi.cu"]
    cpp = ["nb_model.cpp", "nb_libm.cpp", "nb_nccl.cpp"]
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    BUILD.mkdir(exist_ok=True)
    objs = []
    for f in cu:
        o = BUILD / (f + ".o")
        if not newer(o, [CSRC / f] + headers):
            run([NVCC, *NVCC_FLAGS, "-c", CSRC / f, "-o", o])
        objs.append(o)
    for f in cpp:
        o = BUILD / (f + ".o")
        if not newer(o, [CSRC / f] + headers):
            run(["g++", *CXX_FLAGS, "-c", CSRC / f, "-o", o])
        objs.append(o)
    if not newer(out, objs + [CSRC / "pinfer.map"]):
        run([NVCC, *ARCH, "-shared", "-o", out, *objs,
             "-Xlinker", "-soname=libpinfer.so.0.3",
             "-Xlinker", f"--version-script={CSRC / 'pinfer.map'}", "-lpthread", "-ldl"])
    return out


def reference_checkout() -> Path | None:
    """The reference's source checkout: $NB_REFERENCE, else a `reference` directory beside this
    repository; None when neither holds the engine sources."""
    env = os.environ.get("NB_REFERENCE")
    for cand in ([Path(env)] if env else []) + [ROOT.parent / "reference"]:
        if (cand / "engine" / "src" / "forward.c").exists():
            return cand
    return None


def build_oracle() -> None:
    run(["make", "-s", "-C", ROOT / "oracle", "all"])
    ref = reference_checkout()
    if ref is not None:
        run(["make", "-s", "-C", ROOT / "oracle", "ref", f"REF={ref}"])


def main() -> None:
    LIB.mkdir(exist_ok=True)
    build_quant()
    build_engine()
    if "--no-oracle" not in sys.argv:
        build_oracle()


if __name__ == "__main__":
    main()
