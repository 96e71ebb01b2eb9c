"""The native extension loader: ``use_prebuilt`` keeps the reference's signature (tfimage/ext.py:34-60).

The reference routed TensorFold's torch-JIT builds to prebuilt modules. Here the native side is one C-ABI library,
``libtfb.so``, built in-tree by ``build.py`` (nvcc, sm_100a). ``use_prebuilt(directory)`` loads it from
``directory``, ``$TFIMAGE_EXT_DIR`` or this package's folder and returns that folder; a missing library is an
error (there is no compiler fallback at run time and no CPU path).
"""

from __future__ import annotations

from pathlib import Path

from . import _lib

DEFAULT_DIR = _lib.DEFAULT_DIR
SUFFIX = ".so"


def use_prebuilt(directory: str | Path | None = None) -> Path:
    path = _lib.lib_path(directory)
    _lib.load(directory)
    return path.parent
