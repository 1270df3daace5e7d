"""B200-native (sm_100a) NVFP4 hot path: quantizers, tcgen05 block-scaled GEMM
and the NVFP4 SwiGLU MLP training step, behind the reference's
``float4utils`` / ``gn_kernels`` API.

The directory name is not a Python identifier, so the package is imported
under the name ``nvfp4_b200`` (``__graft_entry__.import_package()`` or
``importlib`` with ``submodule_search_locations``).  All compute goes through
the CUDA library ``lib/libnvfp4b200.so``; there is no CPU fallback.
"""
from . import _build, _lib, ops  # noqa: F401
from ._lib import NVFP4Error  # noqa: F401

__version__ = "0.1.0"


def load_library():
    """Load the CUDA library, raising NVFP4Error if it was not built."""
    return _lib.load()
