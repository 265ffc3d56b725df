"""Build the sm_100a extension in place:  python setup.py build_ext --inplace

Every .cu under csrc/ is compiled for sm_100a only (Blackwell B200); torch's
own arch list is bypassed by passing the -gencode explicitly.  Two modules:
lumenrl_b200._C (every kernel) and lumenrl_b200._C_bounds (the NVLink comm
kernels with every peer access bounds-checked, -DLRL_DEBUG_BOUNDS).
"""

import glob
import os

from setuptools import find_packages, setup

ROOT = os.path.dirname(os.path.abspath(__file__))


def cuda_sources():
    srcs = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True))
    return ["csrc/bindings.cpp"] + [s for s in srcs if os.sep + "debug_bounds" + os.sep not in s]


def bounds_sources():
    """The NVLink comm kernels again, compiled with -DLRL_DEBUG_BOUNDS into
    lumenrl_b200._C_bounds (thin wrappers, so their objects do not collide
    with the ordinary build's)."""
    d = os.path.join("csrc", "debug_bounds")
    return [os.path.join(d, "module.cpp")] + sorted(glob.glob(os.path.join(d, "*.cu")))


def ext_modules():
    from torch.utils.cpp_extension import CUDAExtension

    nvcc = [
        "-O3", "-std=c++17", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
        "--expt-relaxed-constexpr", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    ]
    if os.environ.get("LRL_PTXAS_VERBOSE"):
        nvcc.append("-Xptxas=-v")
    return [
        CUDAExtension(
            name="lumenrl_b200._C",
            sources=cuda_sources(),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
            libraries=["cuda"],
        ),
        CUDAExtension(
            name="lumenrl_b200._C_bounds",
            sources=bounds_sources(),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17", "-DLRL_DEBUG_BOUNDS"],
                                "nvcc": nvcc + ["-DLRL_DEBUG_BOUNDS"]},
            libraries=["cuda"],
        ),
    ]


def cmdclass():
    from torch.utils.cpp_extension import BuildExtension
    return {"build_ext": BuildExtension.with_options(use_ninja=True)}


setup(
    name="lumenrl_b200",
    version="0.1.0",
    packages=find_packages(include=["lumenrl_b200", "lumenrl_b200.*"]),
    ext_modules=ext_modules(),
    cmdclass=cmdclass(),
    python_requires=">=3.10",
    entry_points={"verl.plugins": ["lumenrl_b200 = lumenrl_b200.plugin.verl:register"]},
)
