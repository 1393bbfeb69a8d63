"""npu_b200 — B200-native (sm_100a) attention engine behind the reference's
NpuAttention call surface.

    from npu_b200 import NpuAttention, prefill, decode
"""
from .api import decode, decode_workspace_bytes, device_error, prefill  # noqa: F401
from .fa import NpuAttention, enable_attention  # noqa: F401
from ._lib import B2AError  # noqa: F401

__all__ = ["NpuAttention", "enable_attention", "prefill", "decode", "decode_workspace_bytes",
           "device_error", "B2AError"]
