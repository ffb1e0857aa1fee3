"""Build libfbgpu.so in-tree: hand-written CUDA for sm_100a plus the C++ host
engine, one shared library with the C ABI of include/fbgpu.h and
include/fb_engine.h.

    python -m ferrisboost_b200.build            # or build() from Python

nvcc cross-compiles for sm_100a without a GPU.  -fmad=false keeps every
device float operation unfused (the split, leaf, quantizer and SHAP
arithmetic restate the reference engine bit for bit) and the host compiler
gets -ffp-contract=off for the same reason.
"""
import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libfbgpu.so"
SOURCES = ["train_kernels.cu", "explain_kernels.cu", "ctx.cu", "engine.cu", "noalloc.cu"]
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"]
    for c in cand:
        if c and (pathlib.Path(c).exists() or c == "nvcc"):
            return c
    return "nvcc"


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((HERE.parent / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and not _stale():
        return LIB
    objs = []
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    common = [_nvcc(), ARCH, "-lineinfo", "-O3", "-std=c++17", "-fmad=false", "-ccbin", "/usr/bin/g++",
              "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off,-O3", "-I", str(HERE.parent / "include")]
    procs = []
    for src in SOURCES:
        obj = obj_dir / (pathlib.Path(src).stem + ".o")
        objs.append(str(obj))
        cmd = common + ["-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode:
            failed.append(f"{src}:\n{out.decode()}")
        elif verbose and out:
            print(out.decode())
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIB.with_suffix(".so.tmp")
    link = [_nvcc(), ARCH, "-shared", "-ccbin", "/usr/bin/g++", "-o", str(tmp)] + objs + ["-lgomp"]
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
