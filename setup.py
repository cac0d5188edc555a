"""In-tree build of the native libraries.

``python setup.py build_ext --inplace`` produces

* ``meshy_b200/_C*.so`` — the sm_100a CUDA kernel library (nvcc,
  ``-gencode arch=compute_100a,code=sm_100a``; no other architecture);
* ``meshy_b200/_native*.so`` — host-side C++ runtime pieces (column store,
  page allocator, scheduler core).
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode=arch=compute_100a,code=sm_100a"]

cuda_sources = [
    "csrc/bindings.cpp",
    "csrc/vmm.cpp",
    "csrc/kernels/gemm.cu",
    "csrc/kernels/gemm_small.cu",
    "csrc/kernels/elementwise.cu",
    "csrc/kernels/attention.cu",
    "csrc/kernels/attention_tc.cu",
    "csrc/kernels/decode_attn.cu",
    "csrc/kernels/misc.cu",
    "csrc/kernels/moe.cu",
    "csrc/kernels/ep.cu",
    "csrc/kernels/sampling.cu",
    "csrc/kernels/value_head.cu",
    "csrc/kernels/topk.cu",
    "csrc/kernels/decode_noalloc.cu",
    "csrc/kernels/decode_mega.cu",
]
extra_cuda = [s for s in ("csrc/kernels/symm.cu", "csrc/kernels/fsdp.cu") if os.path.exists(os.path.join(ROOT, s))]

native_sources = [s for s in ("csrc/native/bindings.cpp", "csrc/native/column_store.cpp")
                  if os.path.exists(os.path.join(ROOT, s))]

ext_modules = [
    CUDAExtension(
        name="meshy_b200._C",
        sources=cuda_sources + extra_cuda,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={
            "cxx": ["-O3", "-std=c++17"],
            "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr"] + ARCH,
        },
    ),
]
if native_sources:
    ext_modules.append(
        CppExtension(
            name="meshy_b200._native",
            sources=native_sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
        )
    )

setup(
    name="meshy_b200",
    version="0.1.0",
    packages=["meshy_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
