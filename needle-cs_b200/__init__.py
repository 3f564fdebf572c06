"""needle_cs_b200: B200-native (sm_100a) batched quantized decode path for needle-cs.

The compute lives in libneedle_b200.so (C ABI: include/needle_cuda.h).  This
package is the Python host side used by the tests and the benchmark; the C#
engine binds the same library through P/Invoke.
"""
from ._native import LIB_PATH, NeedleError, call, check, lib  # noqa: F401

__all__ = ["LIB_PATH", "NeedleError", "call", "check", "lib", "version"]


def version():
    return lib().ndl_version().decode()
