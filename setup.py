"""Build script for mtorus.

Two in-tree extensions are produced by ``python setup.py build_ext --inplace``:

* ``mtorus._C``    -- host-side C++ runtime (topology, FP8 codec, communicators,
                      pipeline schedule builder).  Pure C++, no CUDA needed.
* ``mtorus._cuda`` -- hand-written sm_100a kernels (tcgen05/TMA GEMM, LayerNorm,
                      cross-entropy, Adam, FP8 quantisation, peer-memory collectives).

Only ``sm_100a`` is targeted: the ``-gencode`` flag below makes torch skip its own
architecture list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))

# Link the shared system libstdc++ explicitly: the toolchain's search path can
# otherwise resolve -lstdc++ to a static archive, and a second, private copy of
# libstdc++ inside the extension breaks iostream/locale state shared with torch.
_LIBSTDCXX = "/usr/lib/x86_64-linux-gnu/libstdc++.so.6"
_LINK = [_LIBSTDCXX] if os.path.exists(_LIBSTDCXX) else []


def _rel(paths):
    return sorted(os.path.relpath(p, ROOT) for p in paths)


host_sources = _rel(
    glob.glob(os.path.join(ROOT, "csrc/core/*.cpp"))
    + glob.glob(os.path.join(ROOT, "csrc/comm/*.cpp"))
    + glob.glob(os.path.join(ROOT, "csrc/pipeline/*.cpp"))
) + ["csrc/bind_host.cpp"]

cuda_sources = _rel(glob.glob(os.path.join(ROOT, "csrc/kernels/*.cu"))) + [
    "csrc/bind_cuda.cpp"
]

common_cxx = ["-O3", "-std=c++17", "-Wno-unused-function"]
nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]

ext_modules = [
    CppExtension(
        name="mtorus._C",
        sources=host_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": common_cxx + ["-pthread"]},
        extra_link_args=["-pthread"] + _LINK,
    ),
    CUDAExtension(
        name="mtorus._cuda",
        sources=cuda_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": common_cxx, "nvcc": nvcc_flags},
        extra_link_args=_LINK,
    ),
]

setup(
    name="mtorus",
    version="0.1.0",
    packages=[
        "mtorus",
        "mtorus.core",
        "mtorus.comm",
        "mtorus.pipeline",
        "mtorus.training",
        "mtorus.torch_ext",
        "mtorus.models",
        "mtorus.ops",
        "mtorus.parallel",
        "mtorus.utils",
    ],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
