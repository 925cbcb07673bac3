"""Build recipe for the native libraries (sm_100a only).

    libdsa_topk_indexer.so        C ABI of include/dsa_topk_indexer.h (CUDA)
    libdsa_topk_indexer_tvmffi.so TVM-FFI export `launch_topk_c` over the C ABI

Both are written next to this file (in-tree), so they travel with the
repository snapshot to the GPU machine. nvcc cross-compiles without a GPU.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libdsa_topk_indexer.so")
TVM_LIB = os.path.join(HERE, "libdsa_topk_indexer_tvmffi.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc():
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
            if f.endswith((".cu", ".cuh", ".h"))] + [os.path.join(INCLUDE, "dsa_topk_indexer.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_cuda(force=False, verbose=False):
    deps = _sources()
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-o", LIB + ".tmp",
           os.path.join(CSRC, "dsa_indexer.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_tvm_ffi(force=False):
    """Optional: needs the tvm_ffi headers/library (present in this image)."""
    src = os.path.join(CSRC, "tvm_ffi_binding.cc")
    if not os.path.exists(src):
        return None
    try:
        import tvm_ffi.libinfo as li
    except Exception:
        return None
    deps = [src, os.path.join(INCLUDE, "dsa_topk_indexer.h"), LIB]
    if not force and not _stale(TVM_LIB, deps):
        return TVM_LIB
    inc = li.find_include_path()
    libdir = os.path.dirname(li.find_libtvm_ffi())
    dlpack = li.find_dlpack_include_path()
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-I", INCLUDE, "-I", inc, "-I", dlpack,
           "-I", "/usr/local/cuda/include", "-o", TVM_LIB + ".tmp", src,
           "-L", HERE, "-l:libdsa_topk_indexer.so", "-L", libdir, "-ltvm_ffi",
           "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + libdir]
    subprocess.run(cmd, check=True)
    os.replace(TVM_LIB + ".tmp", TVM_LIB)
    return TVM_LIB


def build(force=False, verbose=False):
    lib = build_cuda(force=force, verbose=verbose)
    tvm = build_tvm_ffi(force=force)
    return lib, tvm


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
