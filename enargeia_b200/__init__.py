"""B200-native (sm_100a) rebuild of the enargeia decode hot path.

The CUDA kernels and the C ABI live in libenx.so (sources under csrc/, header include/enx.h);
this package is the host-side mirror of the reference's runtime API over that library.
"""

from .checkpoint import QWEN2_0_5B, SMALL, TINY, ModelConfig  # noqa: F401
from .format import EnargeiaError, read_enargeia, write_enargeia  # noqa: F401

__all__ = ["ModelConfig", "QWEN2_0_5B", "SMALL", "TINY", "read_enargeia", "write_enargeia", "EnargeiaError"]
