"""FlashMap drafter hot path on NVIDIA B200 (sm_100a).

Drop-in for the reference package ``flashmap`` (al-jshen/flashmap): the same
``FlashMapConfig``, ``FlashMapDraftModel``, ``FlashMapCache`` and
``FlashMapGenerateOutput`` names, with drafting, sampling and acceptance run
by the CUDA library ``libflashmap_b200.so`` (C ABI: include/flashmap_b200.h).
"""

from transformers import AutoConfig, AutoModel

from .configuration_flashmap import DEFAULT_JUMP_GRIDS, FlashMapConfig, jump_times
from .modeling_flashmap import DraftSession, FlashMapCache, FlashMapDraftModel, FlashMapGenerateOutput

# AutoModel loads FlashMap release folders once the package is imported
# (the reference registers the same way, flashmap/__init__.py:9-12).
AutoConfig.register(FlashMapConfig.model_type, FlashMapConfig, exist_ok=True)
AutoModel.register(FlashMapConfig, FlashMapDraftModel, exist_ok=True)

__all__ = [
    "DEFAULT_JUMP_GRIDS",
    "DraftSession",
    "FlashMapCache",
    "FlashMapConfig",
    "FlashMapDraftModel",
    "FlashMapGenerateOutput",
    "jump_times",
]
