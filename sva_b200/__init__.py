"""B200-native (sm_100a) Summon-Verify Attention decode path.

Drop-in for the reference package ``sva``: the same exports, backed by the CUDA kernels of
libsva_b200.so (see include/sva_b200.h for the C ABI).
"""

from .artifacts import SVAArtifactBundle, SVALayerArtifacts, load_sva_artifact_bundle
from .llama import SVALlamaAttention, SVALlamaPatcher, SVALlamaServingConfig, patch_llama_attention
from .stats import SVAStats

__version__ = "0.1.0"

__all__ = [
    "SVAArtifactBundle",
    "SVALayerArtifacts",
    "SVALlamaAttention",
    "SVALlamaPatcher",
    "SVALlamaServingConfig",
    "SVAStats",
    "load_sva_artifact_bundle",
    "patch_llama_attention",
]
