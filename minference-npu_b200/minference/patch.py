"""HF transformers patch: route attention modules through the sm_100a ops.

Same entry points as the reference (MInference-NPU minference/patch.py:90-159):
``minference_patch(model, config)`` rebinds ``forward``,
``init_minference_parameters`` and ``gather_last_q_sparse_topk`` on every
attention module of the model's attention class, and writes
``starting_layer`` / ``config_path`` / ``minference_attn_type`` into
``model.config``.  ``patch_hf`` builds the config from keyword arguments.

The reference also swaps HF's O(S^2) 4D-mask helper for a skip-if-no-padding
version (:39-87).  With transformers 5.x the same effect comes from the SDPA
mask path, which returns no mask for unpadded causal inputs, so the patch
selects ``sdpa`` as the model's attention implementation (the patched
forward never reads the mask).
"""

from __future__ import annotations

from typing import Any

import torch

from .modules.minference_forward import (
    gather_last_q_sparse_topk,
    init_minference_parameters,
    load_pattern_config,
    minference_forward,
)

__all__ = [
    "minference_patch",
    "patch_hf",
    "minference_patch_kv_cache_cpu",
    "minference_patch_with_kvcompress",
    "minference_patch_vllm",
    "new_patch",
]


def minference_patch(model: torch.nn.Module, config: Any) -> torch.nn.Module:
    try:
        attention_module = model.model.layers[0].self_attn
    except AttributeError as e:
        raise RuntimeError(
            "model.model.layers[0].self_attn not found; only Llama-family / Phi-style models "
            "are supported"
        ) from e
    AttentionClass = attention_module.__class__
    forward_closure = minference_forward()

    model.config.starting_layer = config.starting_layer
    model.config.config_path = config.config_path
    model.config.minference_attn_type = config.attn_type
    best = getattr(config, "attn_kwargs", {}).get("best_pattern")
    if best is not None:
        # validated once here; each layer keeps its own entry
        model.config.minference_best_pattern = load_pattern_config(
            best, num_layers=len(model.model.layers), num_heads=model.config.num_attention_heads
        )
    if hasattr(model.config, "_attn_implementation"):
        try:
            model.config._attn_implementation = "sdpa"
        except Exception:  # noqa: BLE001
            pass

    def update_module(m: torch.nn.Module) -> None:
        if isinstance(m, AttentionClass):
            m._minference_initialized = False
            m.init_minference_parameters = init_minference_parameters.__get__(m, AttentionClass)
            m.gather_last_q_sparse_topk = gather_last_q_sparse_topk.__get__(m, AttentionClass)
            m.forward = forward_closure.__get__(m, AttentionClass)

    model.apply(update_module)
    print(
        f"[MInference-B200] Patched {AttentionClass.__name__}.forward "
        f"(starting_layer={config.starting_layer}, attn_type={config.attn_type})"
    )
    return model


def patch_hf(model: torch.nn.Module, attn_type: str = "minference",
             attn_kwargs: dict | None = None, **kwargs: Any) -> torch.nn.Module:
    """Compatibility entry matching upstream ``patch_hf``."""
    attn_kwargs = dict(attn_kwargs or {})
    attn_kwargs.update(kwargs)
    if attn_type not in ("minference", "dense"):
        raise NotImplementedError(
            f"patch_hf attn_type={attn_type!r} is not supported; use 'minference' or 'dense'"
        )
    from .minference_configuration import MInferenceConfig

    config = MInferenceConfig(
        attn_type=attn_type,
        attn_kwargs=attn_kwargs,
        starting_layer=attn_kwargs.get("starting_layer", -1),
        config_path=attn_kwargs.get("config_path"),
        model_name=attn_kwargs.get("model_name"),
    )
    return minference_patch(model, config)


def minference_patch_kv_cache_cpu(model):
    raise NotImplementedError("KV cache CPU offload is not part of this build")


def minference_patch_with_kvcompress(model, config):
    raise NotImplementedError("KV compression integrations are not part of this build")


def minference_patch_vllm(*args, **kwargs):
    raise NotImplementedError("vLLM integration is not part of this build")


def new_patch(model, config):
    raise NotImplementedError(
        f"new_patch (attn_type={config.attn_type!r}, kv_type={config.kv_type!r}) is not part "
        "of this build"
    )
