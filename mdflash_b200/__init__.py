"""mdflash_b200: the DDTree verification hot path on B200 (sm_100a).

Kernels live in libddtree_b200.so (C ABI: include/ddtree_b200.h); this package is the
PyTorch host side: tensor wrappers (kernels), reference-compatible entry points
(ddtree), the transformers attention plug-in (attention), a static-capacity KV cache
(cache), the device-resident verify step (verifier) and multi-GPU helpers (sharding).
"""
from . import kernels  # noqa: F401
from .kernels import DeviceTree, KvTable  # noqa: F401

__all__ = ["kernels", "DeviceTree", "KvTable"]
