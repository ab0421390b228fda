"""Drop-in for the reference's ``scripts/build_cuda.py``: ``build()`` returns a
module-like object whose ``CudaBatch`` is this library's batch.

The reference JIT-compiles ``_duck_cuda`` with torch.utils.cpp_extension
(scripts/build_cuda.py:8-39); here the library is prebuilt in-tree for sm_100a
and ``build()`` only (re)builds it when a source changed.
"""

import types

from . import build as _build
from .cuda_batch import CudaBatch


def build():
    _build.build_library()
    return types.SimpleNamespace(CudaBatch=CudaBatch, __file__=str(_build.LIB_PATH))
