"""Build of the in-tree extensions: `elysium_wan_b200._C` (sm_100a kernels)
and `elysium_wan_b200._wire` (host codecs and frame I/O of the TCP data plane).

    python setup.py build_ext --inplace

Every CUDA source is compiled for sm_100a only (-gencode arch=compute_100a,
code=sm_100a); passing -gencode makes torch's extension builder skip its own
architecture list.
"""

import os

import pybind11
from setuptools import Extension, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))

# The image's default CC/CXX wrapper links libstdc++ statically into shared
# objects; a static libstdc++ inside a torch extension crashes the first time
# it formats a number (any error message). Use the system compilers, which
# link the process-wide libstdc++.so.6.
for var, path in (("CC", "/usr/bin/gcc"), ("CXX", "/usr/bin/g++")):
    if os.path.exists(path):
        os.environ[var] = path
CSRC = os.path.join("elysium_wan_b200", "csrc")
CU = ["gemm.cu", "norm.cu", "attention.cu", "ce.cu", "embed.cu", "optim.cu", "misc.cu",
      "collectives.cu", "llama.cu", "attention_tc.cu"]

NVCC = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]


def kernels(name: str, defines: list) -> CUDAExtension:
    return CUDAExtension(
        name=name,
        sources=[os.path.join(CSRC, "bindings.cpp")] + [os.path.join(CSRC, f) for f in CU],
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"] + defines, "nvcc": NVCC + defines},
    )


# EWB_KCHECK=1 builds `_C_kcheck` instead: the same kernels with bounds checks
# (-DEWB_KCHECK) that record the failing site in the status record and skip
# the access; `EWB_KCHECK=1` at run time loads it instead of `_C`. Build it in
# its own temporary directory so the two flag sets do not rebuild each other:
#     EWB_KCHECK=1 python setup.py build_ext --inplace --build-temp build/kcheck
KCHECK = os.environ.get("EWB_KCHECK", "0") == "1"

setup(
    name="elysium_wan_b200",
    ext_modules=[kernels("elysium_wan_b200._C_kcheck", ["-DEWB_KCHECK"])] if KCHECK else [
        kernels("elysium_wan_b200._C", []),
        Extension(
            name="elysium_wan_b200._wire",
            sources=[os.path.join(CSRC, "wire", "wire.cpp")],
            include_dirs=[pybind11.get_include()],
            extra_compile_args=["-O3", "-std=c++17", "-fvisibility=hidden"],
            libraries=["z"],
            language="c++",
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
