"""TriAttention KV-cache compression for vLLM on NVIDIA B200 (sm_100a).

Drop-in replacement of the ``vllm-ascend-kvcompress-hust`` plugin's method
surface: method API v1 and its registry, the per-layer physical-state and
query-observation contracts, calibration-statistics loading and the
``vllm.general_plugins`` entry point keep their names and meaning; the
score -> select -> compact hot path runs in hand-written sm_100a CUDA kernels
(``libkvc_b200.so``) called through a C ABI.
"""

from .config import PROVIDER_NAME
from .methods import available_methods, register_method

__all__ = ["PROVIDER_NAME", "available_methods", "register_method"]
__version__ = "0.10.0+b200"
