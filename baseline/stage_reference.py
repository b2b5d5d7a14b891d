"""Stage the unmodified reference implementation under baseline/_ref for the bench's reference
arms (the reference's own CPU search, its Cython CPU backend, and its CUDA search path).

    python baseline/stage_reference.py --reference <reference source tree>   (or OMQ_REFERENCE)

Runs in the build container (it needs the reference source tree and nvcc; no GPU). Output goes
only to baseline/_ref/, which git ignores and GPU runs carry along:
  * the reference's Python package, installed with
    pip install --no-index --no-build-isolation --no-deps --target baseline/_ref <copy of the tree>
    (--no-deps: its requirements pin torch from an index; the image's torch is used);
  * its C++ game engines (alphazero_py), built from the reference sources by `make -C oracle ref`;
  * its Cython tree (python/mcts/cpu/cython_tree_optimized.pyx), cythonized and compiled without
    OpenMP, next to the installed package's cpu/ modules;
  * its CUDA kernels (python/mcts/gpu/mcts_kernels.cu, the one file build_cuda.py compiles) as the
    torch extension mcts_cuda_kernels for sm_100, in baseline/_ref/build_cuda_shared/, where the
    reference's cuda_manager looks for it (relative to the working directory);
  * a stand-in for GPUtil, a third-party module the reference's profiler imports
    (python/mcts/profiling/gpu_profiler.py:15) and the image lacks. Without it AsyncWaveSearch
    runs with no profiler and fails on its first expansion (`self.profiler.profile(...)` on None,
    async_wave_search.py:784). The stand-in reports no GPUs, so the profiler's monitoring thread
    records CPU samples only (it already ignores GPU query errors).
Nothing staged here is imported by the package or the tests.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
import sysconfig
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")


def run(cmd, **kw):
    print("+", " ".join(cmd) if isinstance(cmd, list) else cmd, flush=True)
    subprocess.run(cmd, check=True, **kw)


def install_package(ref: str) -> None:
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "ref")
        shutil.copytree(ref, src, ignore=shutil.ignore_patterns(".git", "build*", "*.so"))
        run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
             "--find-links", "/opt/wheelhouse", "--target", OUT, "--upgrade", src])


def game_engines(ref: str) -> None:
    run(["make", "-C", os.path.join(REPO, "oracle"), "ref", f"REF={ref}"])
    for so in glob.glob(os.path.join(REPO, "oracle", "_ref", "alphazero_py*.so")):
        shutil.copy2(so, OUT)


def cython_tree(ref: str) -> None:
    from Cython.Build import cythonize
    import numpy as np
    pyx = os.path.join(ref, "python", "mcts", "cpu", "cython_tree_optimized.pyx")
    with tempfile.TemporaryDirectory() as tmp:
        local = os.path.join(tmp, "cython_tree_optimized.pyx")
        shutil.copy2(pyx, local)
        cythonize([local], language_level=3, quiet=True)
        c = os.path.join(tmp, "cython_tree_optimized.c")
        cpp = os.path.join(tmp, "cython_tree_optimized.cpp")
        source = cpp if os.path.exists(cpp) else c
        suffix = sysconfig.get_config_var("EXT_SUFFIX")
        dst = os.path.join(OUT, "mcts", "cpu", "cython_tree_optimized" + suffix)
        run(["g++" if source.endswith(".cpp") else "gcc", "-O3", "-shared", "-fPIC",
             f"-I{sysconfig.get_paths()['include']}", f"-I{np.get_include()}", source, "-o", dst])


def cuda_kernels(ref: str) -> None:
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load
    build = os.path.join(OUT, "build_cuda_shared")
    os.makedirs(build, exist_ok=True)
    src = os.path.join(ref, "python", "mcts", "gpu", "mcts_kernels.cu")
    # the flags of build_cuda.py, for the B200's compute capability
    load(name="mcts_cuda_kernels", sources=[src], build_directory=build, verbose=False,
         extra_cuda_cflags=["-O3", "--use_fast_math", "--expt-relaxed-constexpr", "--expt-extended-lambda",
                            "-diag-suppress=20012", "-diag-suppress=177"])
    built = glob.glob(os.path.join(build, "mcts_cuda_kernels*.so"))
    if not built:
        raise RuntimeError("mcts_cuda_kernels was not built")
    if built[0] != os.path.join(build, "mcts_cuda_kernels.so"):
        shutil.copy2(built[0], os.path.join(build, "mcts_cuda_kernels.so"))


def gputil_stand_in() -> None:
    with open(os.path.join(OUT, "GPUtil.py"), "w") as f:
        f.write('"""Stand-in for the GPUtil package (absent from this image): no GPUs to report."""\n\n\n'
                "def getGPUs():\n    return []\n")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OMQ_REFERENCE"),
                    required="OMQ_REFERENCE" not in os.environ)
    ap.add_argument("--skip-cuda", action="store_true")
    a = ap.parse_args()
    os.makedirs(OUT, exist_ok=True)
    install_package(a.reference)
    game_engines(a.reference)
    cython_tree(a.reference)
    gputil_stand_in()
    if not a.skip_cuda:
        cuda_kernels(a.reference)
    print("staged the reference under", OUT)


if __name__ == "__main__":
    main()
