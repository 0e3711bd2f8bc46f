"""Exact graph transforms for Qwen3.5/Ornith sparse MoE, B200 edition.

Mirror of Runnel's product transform (src/runnel/mlx.py): the same function
name, the same traversal ``model.language_model.layers[i].mlp.switch_mlp``,
the same validation errors and the same packed layout (routed up||gate rows
concatenated on axis 1).  The packed module's forward runs the B200 kernel.
"""
from __future__ import annotations

import gc
from typing import Any

from .switch_layers import (FusedQuantizedSharedMLP, FusedQuantizedSwitchGLU, SharedExpertMLP,
                            SwitchGLU)

__all__ = ["fuse_routed_gate_up", "fuse_shared_gate_up", "FusedQuantizedSwitchGLU"]


def fuse_routed_gate_up(model: Any) -> int:
    """Replace every layer's routed gate/up pair with one packed module.

    The routed gate and up projections share one affine format; concatenating
    their packed rows (up first, then gate) keeps each row's arithmetic and
    lets one gather kernel produce both halves of the SwiGLU input.  Returns
    the number of layers transformed.
    """
    count = 0
    for layer in model.language_model.layers:
        old = layer.mlp.switch_mlp
        if not hasattr(old.gate_proj, "bits"):
            raise ValueError("routed gate/up are not quantized as expected")
        fused = FusedQuantizedSwitchGLU(old)
        layer.mlp.switch_mlp = fused
        count += 1
        del old, fused
        gc.collect()
    return count


def fuse_shared_gate_up(model: Any) -> int:
    """Pack every layer's shared-expert up||gate on axis 0 (the optional shared
    fusion of bench/mlx_lm_adapter.py:49-94)."""
    count = 0
    for layer in model.language_model.layers:
        old = layer.mlp.shared_expert
        if isinstance(old, SharedExpertMLP):
            layer.mlp.shared_expert = FusedQuantizedSharedMLP(old)
            count += 1
    return count


def is_packed(switch_mlp) -> bool:
    return isinstance(switch_mlp, FusedQuantizedSwitchGLU) and not isinstance(switch_mlp, SwitchGLU)
