"""Builds the native parts of mod_b200 in place.

    python setup.py build_ext --inplace

* ``mod_b200/_C``    : sm_100a CUDA kernels (tcgen05/TMA GEMMs, attention, ...)
* ``mod_b200/_cpu``  : C++17/OpenMP CPU backend + safetensors mmap reader

Only ``sm_100a`` code is generated (no PTX fallback, no other architectures).
"""
import glob
import os

from setuptools import find_packages, setup

os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"  # keep torch from adding other -gencode targets

from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
import torch  # noqa: E402

TORCH_LIB = os.path.join(os.path.dirname(torch.__file__), "lib")
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("MB_PTXAS_VERBOSE") else "-DMB_QUIET",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def cuda_ext():
    srcs = sorted(glob.glob(os.path.join("csrc", "cuda", "*.cu"))) + ["csrc/cuda/ops.cpp"]
    return CUDAExtension(
        name="mod_b200._C",
        sources=srcs,
        include_dirs=[os.path.join(ROOT, "csrc", "cuda")],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    )


def cpu_ext():
    srcs = sorted(glob.glob(os.path.join("csrc", "cpu", "*.cc"))) + sorted(glob.glob(os.path.join("csrc", "io", "*.cc")))
    return CppExtension(
        name="mod_b200._cpu",
        sources=srcs,
        include_dirs=[os.path.join(ROOT, "csrc", "cpu"), os.path.join(ROOT, "csrc", "io")],
        extra_compile_args=CXX_FLAGS + ["-fopenmp", "-march=x86-64-v3"],
        # link the OpenMP runtime torch already ships, so one process has one runtime
        extra_link_args=["-L" + TORCH_LIB, "-l:libgomp.so.1", "-Wl,-rpath," + TORCH_LIB],
    )


exts = [cuda_ext()]
if glob.glob(os.path.join("csrc", "cpu", "*.cc")):
    exts.append(cpu_ext())

setup(
    name="mod_b200",
    version="0.1.0",
    packages=find_packages(include=["mod_b200", "mod_b200.*"]),
    package_data={"mod_b200": ["config/baselines/*.yaml", "models/plugins/*/plugin_manifest.json"]},
    entry_points={"console_scripts": ["mod_b200 = mod_b200.cli.main:main"]},
    python_requires=">=3.10",
    ext_modules=exts,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
