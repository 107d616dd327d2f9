"""flash_moe_b200 -- the routed-expert MoE hot path of
vin10122/Intel-optimized-MoE-streaming, rebuilt for NVIDIA B200 (sm_100a).

Host side of ``libmoe_b200.so``: drop-ins for the reference's native
bindings (``native_expert``, ``dequant``), an HBM-resident expert store
(``store.ExpertArena``), the expert backend (``backend.B200ExpertBackend``)
and the MoE layer entry points (``moe_layer``).  Importing the package does
not touch the GPU; the library is loaded on first use and there is no CPU
fallback.
"""
from .formats import BLOCK, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0, SUPPORTED_TYPES
from .key import ExpertKey

__all__ = ["BLOCK", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "SUPPORTED_TYPES", "ExpertKey"]
__version__ = "0.1.0"
