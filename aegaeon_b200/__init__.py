"""aegaeon_b200 — B200-native (sm_100a) per-token serving path of Aegaeon.

``aegaeon_b200.ops`` mirrors the reference's ``aegaeon.ops`` operator module (``swap``) and adds
the per-layer cache write, paged decode attention and block copy that the reference reaches
through vLLM. ``aegaeon_b200.layout`` holds the block geometry and per-step metadata builders,
``aegaeon_b200.step`` the CUDA-graph decode-step runner.

Submodules load on first use, so that ``python -m aegaeon_b200.build`` works before the native
library exists (or while it is stale).
"""
import importlib

__version__ = "0.1.0"

_SUBMODULES = ("build", "layout", "ops", "step", "synth")
_OPS_EXPORTS = ("DecodePlan", "copy_blocks", "decode_layer", "decode_layer_flash", "flash_attn_decode",
                "paged_attention_decode", "read_device_errors", "reshape_and_cache", "reshape_and_cache_flash",
                "swap", "swap_sm")

__all__ = list(_SUBMODULES) + list(_OPS_EXPORTS)


def __getattr__(name):
    if name in _SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    if name in _OPS_EXPORTS:
        return getattr(importlib.import_module(".ops", __name__), name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
