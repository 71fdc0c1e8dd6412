"""Idempotent vLLM general plugin routing FULL decoder attention to OSCAR on CUDA.

Same behaviour as the reference's ``oscar_ascend/plugin.py:13-130``, retargeted from
``NPUPlatform`` to vLLM's ``CudaPlatform.get_attn_backend_cls(selected_backend,
attn_selector_config, num_heads)``: decoder / non-MLA / non-sparse / causal layers get
``oscar_new_b200.backend.OscarAttentionBackend``; MTP draft layers keep the native
backend; after weight loading each OSCAR layer loads its calibrated rotations.
Enabled by ``OSCAR_ENABLED=1`` (``OSCAR_ASCEND_ENABLED=1`` is accepted as well).
Registered through ``[project.entry-points."vllm.general_plugins"]``.
"""

from __future__ import annotations

import functools
import inspect
import logging
import sys

from .backend import enabled

LOG = logging.getLogger(__name__)
BACKEND_PATH = "oscar_new_b200.backend.OscarAttentionBackend"
_registered = False


def should_route(selector) -> bool:
    """Keep vision/encoder, MLA, sparse and non-causal attention native."""
    return (
        str(getattr(selector, "attn_type", "decoder")).split(".")[-1].lower() == "decoder"
        and not getattr(selector, "use_mla", False)
        and not getattr(selector, "use_sparse", False)
        and not getattr(selector, "use_non_causal", False)
    )


def is_draft_layer(prefix: str) -> bool:
    return "mtp" in prefix.split(".")


def install_selector(platform_cls):
    """Wrap ``platform_cls.get_attn_backend_cls`` (idempotent per class)."""
    if platform_cls.__dict__.get("_oscar_selector_installed", False):
        return
    original = platform_cls.get_attn_backend_cls.__func__

    @classmethod
    @functools.wraps(original)
    def select(cls, selected_backend, attn_selector_config, num_heads=None):
        _install_loaded_attention_hooks()
        if should_route(attn_selector_config):
            for name in ("has_sink", "use_mm_prefix", "use_per_head_quant_scales"):
                if getattr(attn_selector_config, name, False):
                    raise ValueError(f"OSCAR does not support selector option {name}")
            # Runners may probe with a sentinel head_size of 0 before model construction;
            # real layers validate D=256 in the implementation's constructor.
            if attn_selector_config.head_size not in (0, 256):
                return original(cls, selected_backend, attn_selector_config, num_heads)
            return BACKEND_PATH
        return original(cls, selected_backend, attn_selector_config, num_heads)

    platform_cls.get_attn_backend_cls = select
    platform_cls._oscar_selector_installed = True


def register(platform_cls=None):
    """vLLM general-plugin entry point."""
    global _registered
    if _registered or not enabled():
        return
    if platform_cls is None:
        from vllm.platforms.cuda import CudaPlatform as platform_cls  # noqa: N813
    install_selector(platform_cls)
    _install_loaded_attention_hooks()
    _registered = True
    LOG.warning("OSCAR INT2 KV attention enabled for FULL decoder layers; prefix sharing disabled, "
                "MTP draft layers native.")


def _install_loaded_attention_hooks(attention_cls=None):
    """Wrap a fully imported ``Attention`` class: draft layers native, rotations after load."""
    if attention_cls is None:
        module = sys.modules.get("vllm.model_executor.layers.attention.attention") or sys.modules.get(
            "vllm.attention.layer")
        if module is None or getattr(getattr(module, "__spec__", None), "_initializing", False):
            return False
        attention_cls = getattr(module, "Attention", None)
        if attention_cls is None:
            return False
    if getattr(attention_cls, "_oscar_hooks_installed", False):
        return True
    original_init = attention_cls.__init__
    signature = inspect.signature(original_init)

    @functools.wraps(original_init)
    def initialize(layer, *args, **kwargs):
        bound = signature.bind(layer, *args, **kwargs)
        prefix = bound.arguments.get("prefix", "")
        if is_draft_layer(prefix) and bound.arguments.get("attn_backend") is None and "attn_backend" in signature.parameters:
            # MTP draft layers have their own weights and no calibrated rotations.
            from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend

            bound.arguments["attn_backend"] = FlashAttentionBackend
        return original_init(*bound.args, **bound.kwargs)

    attention_cls.__init__ = initialize
    original_process = getattr(attention_cls, "process_weights_after_loading", None)
    if original_process is not None:

        @functools.wraps(original_process)
        def process(layer, act_dtype):
            result = original_process(layer, act_dtype)
            from .backend import OscarAttentionImpl

            if isinstance(getattr(layer, "impl", None), OscarAttentionImpl):
                layer.impl.initialize_layer(layer)
            return result

        attention_cls.process_weights_after_loading = process
    attention_cls._oscar_hooks_installed = True
    return True
