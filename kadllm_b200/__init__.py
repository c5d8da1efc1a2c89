"""B200-native GRBeam (shared-prefix wide-beam decoding) for hybrid Qwen3.5 models.

Drop-in names of Kadllm's GRBeam API: ``grbeam_search``, ``GRBeamAdapter``,
``PrefillResult``, ``GRBeamResult``, the ``ops`` operators and
``adapters.Qwen35GRBeamAdapter``.  Compute runs in the sm_100a CUDA library
``libkadllm_b200.so`` (C ABI in ``include/kadllm_b200.h``).
"""

from .grbeam import GRBeamAdapter, GRBeamResult, PrefillResult, grbeam_search
from .ops import causal_conv1d, gated_delta, prefix_attention

__all__ = [
    "GRBeamResult",
    "PrefillResult",
    "GRBeamAdapter",
    "grbeam_search",
    "causal_conv1d",
    "gated_delta",
    "prefix_attention",
]
