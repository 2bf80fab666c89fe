"""``MInferenceConfig``: which attention path a patched model takes and where
its per-head patterns come from.

The constructor keywords, attribute names, class-level type lists and
``attn_kwargs`` keys are the drop-in API of the reference class
(MInference-NPU minference/minference_configuration.py:7-75); callers build it
the same way and read the same fields.  Validation raises ``AssertionError``
for unsupported types and unregistered model names, as the reference does.
"""

from __future__ import annotations

from .configs.model2path import MODEL2PATH

# attn_type aliases accepted on input and the name each maps to
_ATTN_ALIASES = {"minference_with_dense": "dense"}


class MInferenceConfig:
    MINFERENCE_ATTENTION_TYPES = ["minference"]
    OTHER_ATTENTION_TYPES = ["hf", "dense"]
    KV_TYPES = ["dense"]

    def __init__(self, attn_type: str = "minference", model_name: str | None = None,
                 config_path: str | None = None, starting_layer: int = -1,
                 kv_cache_cpu: bool = False, kv_cache_cpu_device: str = "cpu",
                 kv_type: str = "dense", is_search: bool = False,
                 attn_kwargs: dict | None = None, **kwargs):
        attn_type, kv_type = self.update_config_type(attn_type, kv_type)
        known = self.get_available_attn_types()
        assert attn_type in known, f"attn_type {attn_type!r} is not supported (one of {known})"
        assert kv_type in self.KV_TYPES, f"kv_type {kv_type!r} is not supported ({self.KV_TYPES})"
        self.attn_type = attn_type
        self.kv_type = kv_type
        self.model_name = model_name
        self.starting_layer = starting_layer
        self.is_search = is_search
        self.kv_cache_cpu = kv_cache_cpu
        self.kv_cache_cpu_device = kv_cache_cpu_device
        self.config_path = self.update_config_path(config_path, model_name)
        # per-layer options handed to the patched attention modules; explicit
        # attn_kwargs entries win over the derived ones
        self.attn_kwargs = dict(is_search=is_search, starting_layer=starting_layer,
                                config_path=self.config_path)
        self.attn_kwargs.update(attn_kwargs or {})

    def update_config_path(self, config_path: str | None = None,
                           model_name: str | None = None) -> str:
        """Pattern JSON for sparse attention types; "" for hf / dense."""
        if self.attn_type not in self.MINFERENCE_ATTENTION_TYPES:
            return ""
        if config_path is not None:
            return config_path
        assert model_name in MODEL2PATH, (
            f"model {model_name!r} has no registered pattern config; pass config_path= "
            f"(registered: {sorted(MODEL2PATH)})"
        )
        return MODEL2PATH[model_name]

    def get(self, attr, default=None):
        return getattr(self, attr, default)

    @staticmethod
    def update_config_type(attn_type: str, kv_type: str) -> tuple[str, str]:
        """Normalise aliases: an empty kv_type means "dense"."""
        return _ATTN_ALIASES.get(attn_type, attn_type), (kv_type or "dense")

    @classmethod
    def get_available_attn_types(cls) -> list[str]:
        return [*cls.MINFERENCE_ATTENTION_TYPES, *cls.OTHER_ATTENTION_TYPES]

    @classmethod
    def get_available_kv_types(cls) -> list[str]:
        return list(cls.KV_TYPES)
