"""nebula_b200 -- B200-native (sm_100a) quantized linear layer for the hydrogen engine.

The compute lives in ``libhq.so`` (CUDA kernels + C ABI, include/hq.h); this
package is the Python host side (``hq``) and the in-tree build (``build``).
"""
import importlib

from . import _lib  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    if name in ("hq", "build"):
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
