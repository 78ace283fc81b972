"""aegaeon_b200 — B200-native (sm_100a) per-token serving path of Aegaeon.

``aegaeon_b200.ops`` mirrors the reference's ``aegaeon.ops`` operator module (``swap``) and adds
the per-layer cache write, paged decode attention and block copy that the reference reaches
through vLLM. ``aegaeon_b200.layout`` holds the block geometry and per-step metadata builders.
"""
from . import layout, ops  # noqa: F401
from .ops import (  # noqa: F401
    DecodePlan,
    copy_blocks,
    flash_attn_decode,
    paged_attention_decode,
    read_device_errors,
    reshape_and_cache,
    reshape_and_cache_flash,
    swap,
    swap_sm,
)

__version__ = "0.1.0"
