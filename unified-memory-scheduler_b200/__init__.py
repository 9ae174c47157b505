"""umsx: B200-native MoE-layer hot path of appatalks/unified-memory-scheduler.

The compute runs in libumsx.so (hand-written sm_100a CUDA behind a C ABI,
include/umsx.h); this package holds the Python bindings and the layer configs.
The directory name is not a Python identifier, so __graft_entry__.load_package()
registers it as `umsx_b200`.
"""
from . import configs, umsx  # noqa: F401
from .umsx import MoeLayer, MoeStack, UmsxError, combine, kernel_launches, lib, load_gguf_experts  # noqa: F401
