"""Builds tests/support/libmiso_test_support.so (test-only kernels and launchers: combine_variants.cu,
engine_kernels.cu)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

def _product_build():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "miso_build", os.path.join(ROOT, "miso_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_b = _product_build()

LIB = os.path.join(HERE, "libmiso_test_support.so")
SRCS = [os.path.join(HERE, "combine_variants.cu"), os.path.join(HERE, "engine_kernels.cu")]


def build(force: bool = False) -> str:
    deps = SRCS + [os.path.join(_b.CSRC, "kernels", f) for f in os.listdir(
        os.path.join(_b.CSRC, "kernels"))]
    if not force and os.path.exists(LIB) and all(
            os.path.getmtime(d) <= os.path.getmtime(LIB) for d in deps):
        return LIB
    cmd = [os.environ.get("NVCC", "nvcc"), *[f for f in _b.NVCC_FLAGS if f != "-warn-spills"
                                             and f != "-Xptxas"],
           f"-I{_b.CSRC}", "-o", LIB, *SRCS]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
