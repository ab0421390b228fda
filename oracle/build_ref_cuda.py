"""Builds the reference's own CUDA extension (``_duck_cuda``: extension.cu +
solver.cpp) for sm_100a from the reference checkout named by DUCK_REFERENCE,
into oracle/_ref/cuda/.  It is test infrastructure: bench.py times the
reference's CUDA step on the same B200 as a context number beside its own
(kernel against kernel); nothing in the product loads it.

The flags are the reference's (scripts/build_cuda.py:26-37: -O3, -std=c++17,
--expt-relaxed-constexpr, --fmad=false, float math and unrolling off) plus
the sm_100a target.

    DUCK_REFERENCE=<reference checkout> python oracle/build_ref_cuda.py
"""

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "cuda"


def build(reference):
    ref = Path(reference)
    if not (ref / "src" / "cuda" / "extension.cu").exists():
        print(f"reference sources not found under {ref}; skipping the CUDA reference build", file=sys.stderr)
        return None
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", "4")
    # The system compiler links libstdc++ dynamically; a compiler that links
    # a static copy into the module crashes it once numpy has loaded the
    # shared one.
    os.environ["CXX"] = "/usr/bin/g++"
    os.environ["CC"] = "/usr/bin/gcc"
    from torch.utils.cpp_extension import load

    OUT.mkdir(parents=True, exist_ok=True)
    defines = ["-DDUCK_NATIVE_FLOAT_MATH=0", "-DDUCK_UNROLL_SMALL_MATRICES=0"]
    module = load(
        name="_duck_cuda",
        sources=[str(ref / "src/cuda/extension.cu"), str(ref / "src/solver.cpp")],
        extra_include_paths=[str(ref / "include")],
        build_directory=str(OUT),
        extra_cflags=["-O3", "-std=c++17"] + defines,
        extra_cuda_cflags=["-O3", "-std=c++17", "--expt-relaxed-constexpr", "--fmad=false",
                           "-gencode", "arch=compute_100a,code=sm_100a"] + defines,
        verbose=False,
    )
    # Keep only the module: the objects and ninja files are not needed to
    # load it, and everything under oracle/_ref travels to the GPU box.
    for item in OUT.iterdir():
        if item.name != Path(module.__file__).name:
            item.unlink()
    return module.__file__


if __name__ == "__main__":
    if "DUCK_REFERENCE" not in os.environ:
        sys.exit("set DUCK_REFERENCE to the reference checkout")
    print(build(os.environ["DUCK_REFERENCE"]))
