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
SOURCES = ["train_kernels.cu", "explain_kernels.cu", "ctx.cu", "engine.cu", "noalloc.cu", "nccl_loader.cu", "lossguide.cu",
           "sketch.cu", "shap_paths.cu", "hist_ceiling.cu", "qscale.cu", "devmem.cu"]
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"]
    for c in cand:
        if c and (pathlib.Path(c).exists() or c == "nvcc"):
            return c
    return "nvcc"


def _nccl_include() -> str:
    """Directory of nccl.h: the one of the NCCL wheel PyTorch loads at run time
    (the library binds NCCL with dlopen, so only the header is needed here),
    else the system's."""
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
        if spec and spec.submodule_search_locations:
            for loc in spec.submodule_search_locations:
                inc = pathlib.Path(loc) / "include"
                if (inc / "nccl.h").exists():
                    return str(inc)
    except (ImportError, ValueError):
        pass
    for inc in (os.environ.get("NCCL_INCLUDE"), "/usr/include", "/usr/local/include"):
        if inc and (pathlib.Path(inc) / "nccl.h").exists():
            return inc
    raise RuntimeError("nccl.h not found (set NCCL_INCLUDE)")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((HERE.parent / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


EXP_TABLE = HERE / "expf_exceptions.bin"


def build_exp_table(force: bool = False) -> pathlib.Path:
    """Generate expf_exceptions.bin: every f32 input on which the host libm's
    expf differs from the library's f64 exp (csrc/fexp.h), by evaluating both
    on all 2^32 inputs (csrc/gen_expf_table.cpp; a few seconds on 8 cores)."""
    gen_src = CSRC / "gen_expf_table.cpp"
    if not force and EXP_TABLE.exists() and EXP_TABLE.stat().st_mtime >= max(
            gen_src.stat().st_mtime, (CSRC / "fexp.h").stat().st_mtime):
        return EXP_TABLE
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    exe = obj_dir / "gen_expf_table"
    subprocess.run(["/usr/bin/g++", "-O2", "-std=c++17", "-fopenmp", "-ffp-contract=off", "-march=x86-64-v2",
                    "-I", str(CSRC), str(gen_src), "-o", str(exe)], check=True)
    tmp = EXP_TABLE.with_suffix(".bin.tmp")
    subprocess.run([str(exe), str(tmp)], check=True, stdout=subprocess.DEVNULL)
    os.replace(tmp, EXP_TABLE)
    return EXP_TABLE


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    build_exp_table()
    if not force and not _stale():
        return LIB
    objs = []
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    common = [_nvcc(), ARCH, "-lineinfo", "-O3", "-std=c++17", "-fmad=false", "-ccbin", "/usr/bin/g++",
              "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off,-O3", "-I", str(HERE.parent / "include"),
              "-I", _nccl_include()]
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
    link = [_nvcc(), ARCH, "-shared", "-ccbin", "/usr/bin/g++", "-o", str(tmp)] + objs + ["-lgomp", "-ldl"]
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
