"""p2p_b200 -- B200-native (sm_100a) attention for the LFM2.5-VL engine of KingNish24/P2P.

The kernels live in libp2pattn.so (C ABI: include/p2p_attn.h); this package is the Python
host mirror of the reference engine's attention operators.  Importing it loads the library
and fails if it has not been built; there is no CPU fallback.
"""
from ._lib import (  # noqa: F401
    LIB_PATH, MAX_LAYERS, P2P_ERR_INVALID_ARG, P2P_ERR_KV_FULL, P2P_ERR_NCCL, P2P_ERR_OOM,
    P2P_ERR_TIMEOUT, KvFullError, OomError, P2PError, lib,
)
from .attention import Context, KVCache, LfmAttention, Params  # noqa: F401
from .comm import Comm  # noqa: F401

__all__ = ["Comm", "Context", "KVCache", "LfmAttention", "Params", "P2PError", "KvFullError",
           "OomError", "lib", "LIB_PATH", "MAX_LAYERS", "P2P_ERR_INVALID_ARG", "P2P_ERR_KV_FULL",
           "P2P_ERR_NCCL", "P2P_ERR_OOM", "P2P_ERR_TIMEOUT"]
