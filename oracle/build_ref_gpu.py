"""Build the reference's own GPU solution (the CUTLASS pipeline behind
``solution/python/kernel.py:95-120``) for sm_100a, for side-by-side timing.

Test and measurement infrastructure only: nothing in the library calls it.
It compiles the reference's three source files where they lie
(``solution/python/{main.cpp,kernel.cu,moe_grouped_gemm_fp8.cu}``) with the
flags of ``kernel.py:75-86`` and the CUTLASS headers bundled with the
installed flashinfer package (the same fallback as ``kernel.py:20-44``), into
``oracle/_ref/gpu_ext/`` (git-ignored, shipped to GPU boxes with the tree).
Runs here, without a GPU (about ten minutes, mostly the CUTLASS unit).

    python oracle/build_ref_gpu.py <path to the reference checkout>
"""

from __future__ import annotations

import os
import pathlib
import sys

OUT = pathlib.Path(__file__).resolve().parent / "_ref" / "gpu_ext"
NAME = "moe_ref_gpu_ext"


def cutlass_include() -> str:
    import flashinfer
    p = pathlib.Path(flashinfer.__file__).parent / "data" / "cutlass" / "include"
    if not (p / "cutlass" / "cutlass.h").exists():
        raise RuntimeError(f"CUTLASS headers not found under {p}")
    return str(p)


def build(ref_root: str) -> pathlib.Path:
    src = pathlib.Path(ref_root) / "solution" / "python"
    sources = [str(src / f) for f in ("main.cpp", "kernel.cu", "moe_grouped_gemm_fp8.cu")]
    for s in sources:
        if not pathlib.Path(s).exists():
            raise FileNotFoundError(s)
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"      # sm_100a only (no GPU to detect here)
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    import torch.utils.cpp_extension as cpp_ext
    cpp_ext.load(name=NAME, sources=sources,
                 extra_cuda_cflags=["-std=c++17", "--expt-relaxed-constexpr", "-O2"],
                 extra_include_paths=[str(src), cutlass_include()],
                 build_directory=str(OUT), verbose=True)
    return OUT / f"{NAME}.so"


def load():
    """Import the prebuilt extension (``run(...)`` as in ``main.cpp:268-270``)."""
    import importlib.util
    import torch  # noqa: F401  (the extension links libtorch)
    so = OUT / f"{NAME}.so"
    if not so.exists():
        raise ImportError(f"{so} is missing; run oracle/build_ref_gpu.py where the reference checkout is")
    spec = importlib.util.spec_from_file_location(NAME, so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    print(build(sys.argv[1]))
