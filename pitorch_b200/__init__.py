"""pitorch_b200 -- pitorch's C API on a B200.

The product is the shared library ``libpitorch_b200.so`` (C host layer +
sm_100a CUDA kernels), built in-tree by ``pitorch_b200/csrc/Makefile``. This
package only loads it with ctypes and mirrors the C structs of ``include/``
so tests and benchmarks can drive the same entry points a C caller would.

There is no CPU fallback: if the library is missing, importing ``lib()``
raises, and every compute entry point requires a CUDA device.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpitorch_b200.so")
REPO_ROOT = os.path.dirname(_HERE)
INCLUDE_DIR = os.path.join(REPO_ROOT, "include")

_lib = None


def build(jobs=8):
    """Compile libpitorch_b200.so in-tree (nvcc cross-compiles for sm_100a)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", os.path.join(_HERE, "csrc"), f"-j{jobs}"], check=True)


def lib():
    """The loaded product library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run pitorch_b200.build() "
                               "(there is no CPU fallback)")
        from . import api
        _lib = ctypes.CDLL(LIB_PATH)
        api.declare(_lib)
    return _lib
