"""Compiles the REFERENCE's own CUDA path (solution/cuda/kernel.cu of the
reference repository, read where it lies) into oracle/_ref/.

TEST INFRASTRUCTURE ONLY. The resulting extension exposes the reference's
`launch_topk_c` (kernel.cu:818-891). It is used (a) to pin the oracle and the
golden vectors against outputs of the reference itself, run on a B200, and
(b) to time the reference's GPU kernel beside ours on the shapes it supports
(N_max <= 8192). Nothing in the shipped library links it. The reference
sources are not copied into this repository; only the build output is written
(into oracle/_ref/, which git ignores but which travels to the GPU machine).

Run on the development machine (needs the reference checkout and nvcc, no
GPU):
    python oracle/build_ref.py [/path/to/reference]
The checkout is found from the argument, else the DSA_REFERENCE_ROOT
environment variable, else a directory named "reference" beside this
repository.
"""
import glob
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "dsa_ref_kernel"


def default_root():
    """The reference checkout: $DSA_REFERENCE_ROOT, else ../reference next to
    this repository."""
    env = os.environ.get("DSA_REFERENCE_ROOT")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def source(ref_root=None):
    """Path of the reference's kernel.cu (it may not exist)."""
    return os.path.join(ref_root or default_root(), "solution", "cuda", "kernel.cu")


def build(ref_root=None):
    src = source(ref_root)
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"  # as the reference's binding.py:13 sets it
    from torch.utils.cpp_extension import load
    os.makedirs(OUT, exist_ok=True)
    load(name=NAME, sources=[src], build_directory=OUT, verbose=False,
         extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"], is_python_module=True)
    return lib_path()


def lib_path():
    c = glob.glob(os.path.join(OUT, NAME + "*.so"))
    return c[0] if c else None


def load_ref():
    """Imports the prebuilt reference extension (raises if absent)."""
    p = lib_path()
    if p is None:
        raise FileNotFoundError("reference extension not built (oracle/build_ref.py)")
    import torch  # noqa: F401  (the extension links libtorch)
    spec = importlib.util.spec_from_file_location(NAME, p)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(*sys.argv[1:]))
