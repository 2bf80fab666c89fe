"""Top-level patch entry: ``MInference(attn_type, model_name|config_path, ...)(model)``.

Same constructor and behaviour as the reference
(MInference-NPU minference/models_patch.py:26-94): ``attn_type`` is one of
``minference`` (per-head sparse patterns from the config), ``dense`` (every
head dense causal on the B200 kernel) or ``hf`` (model returned unpatched).
"""

from __future__ import annotations

import json

from .minference_configuration import MInferenceConfig

_SUPPORTED_ATTN = ("minference", "dense", "hf")
_SUPPORTED_KV = ("dense",)


class MInference:
    def __init__(self, attn_type: str = "minference", model_name: str | None = None,
                 config_path: str | None = None, starting_layer: int = -1,
                 kv_type: str = "dense", is_search: bool = False,
                 attn_kwargs: dict | None = None, **kwargs):
        if attn_type not in _SUPPORTED_ATTN:
            raise ValueError(f"attn_type={attn_type!r} is not supported; use one of {_SUPPORTED_ATTN}")
        if kv_type not in _SUPPORTED_KV:
            raise ValueError(f"kv_type={kv_type!r} is not supported; use one of {_SUPPORTED_KV}")
        self.config = MInferenceConfig(
            attn_type=attn_type, model_name=model_name, config_path=config_path,
            starting_layer=starting_layer, kv_cache_cpu=False, kv_type=kv_type,
            is_search=is_search, attn_kwargs=attn_kwargs or {}, **kwargs,
        )

    def __call__(self, model):
        return self.patch_model(model)

    def patch_model(self, model):
        if self.config.attn_type == "hf":
            return model
        if self.config.attn_type == "minference" and not self.config.is_search:
            if not self.config.config_path:
                raise ValueError(
                    "attn_type='minference' needs model_name (registered) or config_path "
                    "(per-head pattern JSON)"
                )
            with open(self.config.config_path) as f:
                self.config.attn_kwargs.setdefault("best_pattern", json.load(f))
        from .patch import minference_patch

        return minference_patch(model, self.config)
