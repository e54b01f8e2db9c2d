"""Build recipe for the in-tree CUDA library ``final_b200/lib/libb2moe.so``.

The library is compiled for sm_100a only (tcgen05 / TMA / TMEM code) with an
explicit ``-gencode arch=compute_100a,code=sm_100a`` and links the CUDA
runtime statically, so the .so that travels with the repository needs no
runtime lookup beyond the NVIDIA driver.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libb2moe.so"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]

SOURCES = ["b2moe_api.cu", "ep.cu", "noalloc.cu", "mlp.cu", "lfm2.cu", "loader.cpp"]


def _needs_rebuild(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _deps():
    out = []
    for p in (list(CSRC.rglob("*.cu")) + list(CSRC.rglob("*.cuh")) + list(CSRC.rglob("*.h")) +
              list(CSRC.rglob("*.cpp"))):
        out.append(p)
    out += list((ROOT / "include").glob("*.h"))
    return out


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu of the library into one shared object (in-tree)."""
    LIBDIR.mkdir(exist_ok=True)
    if not force and not _needs_rebuild(LIB, _deps()):
        return LIB
    objs = []
    for src in SOURCES:
        obj = LIBDIR / (Path(src).stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *objs, "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    for o in objs:
        os.remove(o)
    return LIB


CPPDIR = PKG / "cpp"
LAYERS_LIB = LIBDIR / "libb2layers.so"
LAYERS_RUN = LIBDIR / "b2_layers_run"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def build_cpp(force: bool = False, verbose: bool = False) -> None:
    """The C++ drop-in layer classes (cpp/b2_layers.*) as libb2layers.so over
    libb2moe.so, and the b2_layers_run driver the parity tests use."""
    deps = list(CPPDIR.glob("*")) + [LIB] + list((ROOT / "include").glob("*.h"))
    if not force and not _needs_rebuild(LAYERS_LIB, deps) and not _needs_rebuild(LAYERS_RUN, deps):
        return
    inc = ["-I", str(CUDA_HOME / "include")]
    rpath = ["-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"]
    cmds = [
        ["g++", "-std=c++17", "-O2", "-Wall", "-fPIC", "-shared", *inc,
         str(CPPDIR / "b2_layers.cpp"), "-o", str(LAYERS_LIB), "-L", str(LIBDIR), "-lb2moe",
         *rpath],
        ["g++", "-std=c++17", "-O2", "-Wall", *inc, str(CPPDIR / "b2_layers_run.cpp"),
         "-o", str(LAYERS_RUN), "-L", str(LIBDIR), "-lb2layers", "-lb2moe",
         "-L", str(CUDA_HOME / "lib64"), "-lcudart", *rpath],
    ]
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)


def reference_dir():
    """The reference checkout whose kernels oracle/_ref is compiled from: the
    B2_REFERENCE_DIR environment variable, else a directory named
    ``reference`` beside this repository; None when neither holds
    src/layer.cu (e.g. on a GPU box, which uses the prebuilt oracle/_ref)."""
    for cand in (os.environ.get("B2_REFERENCE_DIR"), ROOT.parent / "reference"):
        if cand and (Path(cand) / "src" / "layer.cu").is_file():
            return Path(cand)
    return None


def build_oracle(verbose: bool = False) -> None:
    """Build the CPU oracle (and oracle/_ref when the reference tree exists)."""
    cmd = ["make", "-C", str(ROOT / "oracle")]
    ref = reference_dir()
    if ref is not None:
        cmd.append(f"REF={ref}")
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, stdout=None if verbose else subprocess.DEVNULL)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    build_cpp(force="--force" in sys.argv, verbose=True)
    build_oracle(verbose=True)
