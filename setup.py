"""Build of kunserve_b200 and its native extension (sm_100a only).

    python setup.py build_ext --inplace     # builds kunserve_b200/_C*.so in-tree

The CUDA sources are compiled for ``sm_100a`` (B200) only; NCCL comes from
the ``nvidia-nccl`` wheel that PyTorch ships with.
"""
import os
import sys

from setuptools import find_packages, setup

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("kunserve_b200", "csrc")


def nccl_paths():
    import nvidia.nccl as n

    base = os.path.dirname(n.__file__) if getattr(n, "__file__", None) else list(n.__path__)[0]
    return os.path.join(base, "include"), os.path.join(base, "lib")


def ext_modules():
    if "build_ext" not in sys.argv and "develop" not in sys.argv and "bdist_wheel" not in sys.argv:
        return [], {}
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    inc, lib = nccl_paths()
    nvcc = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
            "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("KUS_PTXAS_VERBOSE") else "-DKUS_QUIET"]
    ext = CUDAExtension(
        name="kunserve_b200._C",
        sources=[os.path.join(CSRC, "bindings.cpp"), os.path.join(CSRC, "engine", "engine.cpp"),
                 os.path.join(CSRC, "engine", "arena.cpp"), os.path.join(CSRC, "kernels", "all.cu")],
        include_dirs=[os.path.join(ROOT, CSRC), inc],
        library_dirs=[lib],
        libraries=[":libnccl.so.2"],
        extra_link_args=[f"-Wl,-rpath,{lib}"],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
    )
    return [ext], {"build_ext": BuildExtension.with_options(use_ninja=True)}


exts, cmds = ext_modules()
setup(
    name="kunserve_b200",
    version="0.1.0",
    description="B200-native LLM serving with parameter-centric KV overload handling",
    packages=find_packages(include=["kunserve_b200", "kunserve_b200.*"]),
    ext_modules=exts,
    cmdclass=cmds,
    zip_safe=False,
)
