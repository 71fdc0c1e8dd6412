"""vLLM attention backend running OSCAR's INT2 KV cache on B200.

Same surface as the reference's ``oscar_ascend/backend.py:13-227`` on vLLM's CUDA
worker: ``OscarAttentionBackend`` (the Ascend parent supplied the cache shape; here it is
``(2, num_blocks, block_size, H, D)`` so ``kv_cache[0]`` / ``kv_cache[1]`` are the
contiguous K / V stripes ``CacheLayout.tensor_views`` reinterprets) and
``OscarAttentionImpl.forward``.  One forward launches: fused K/V rotation + INT2 store +
Q rotation, then INT2 history + BF16 sink/recent/current attention, split merge,
inverse V rotation, path merge and the window store (the reference's 9-10 launches,
order preserved: store before attention, window store last).
"""

from __future__ import annotations

import os

import torch
from vllm.v1.attention.backend import AttentionBackend, AttentionImpl

from .config import OscarConfig, decode_split_cap


class OscarAttentionBackend(AttentionBackend):
    forward_includes_kv_cache_update = True
    supported_dtypes = [torch.bfloat16]
    supported_kv_cache_dtypes = ["auto", "bfloat16"]

    @staticmethod
    def get_name():
        return "CUSTOM"

    @staticmethod
    def get_impl_cls():
        return OscarAttentionImpl

    @staticmethod
    def get_builder_cls():
        from .metadata import OscarMetadataBuilder

        return OscarMetadataBuilder

    @staticmethod
    def get_supported_kernel_block_sizes():
        return [128]

    @staticmethod
    def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str="auto"):
        return (2, num_blocks, block_size, num_kv_heads, head_size)

    @staticmethod
    def copy_blocks(*args, **kwargs):
        raise NotImplementedError("OSCAR ring ownership does not support shared/copied request pages")

    @staticmethod
    def swap_blocks(*args, **kwargs):
        raise NotImplementedError("OSCAR supports native recompute preemption, not KV swapping")


def validate_vllm_config(config):
    """Engine options the OSCAR layout cannot honour (reference backend.py:41-64)."""
    if config.cache_config.enable_prefix_caching:
        raise ValueError("OSCAR requires --no-enable-prefix-caching (BF16 ring owner isolation)")
    if config.cache_config.cache_dtype not in ("auto", "bfloat16"):
        raise ValueError("Use --kv-cache-dtype auto with OSCAR")
    if config.model_config.dtype != torch.bfloat16:
        raise ValueError("OSCAR target model must use BF16 activations/cache")
    if getattr(config, "kv_transfer_config", None) is not None:
        raise ValueError("KV transfer is not supported by this OSCAR layout")
    pc = config.parallel_config
    if getattr(pc, "decode_context_parallel_size", 1) != 1 or getattr(pc, "prefill_context_parallel_size", 1) != 1:
        raise ValueError("OSCAR currently requires PCP=DCP=1")
    if getattr(pc, "enable_dbo", False):
        raise ValueError("DBO requires separate metadata buffer sets and is not supported")
    hf = config.model_config.hf_text_config
    if getattr(hf, "head_dim", 256) != 256:
        raise ValueError("OSCAR INT2 is implemented for head_dim 256")


class OscarAttentionImpl(AttentionImpl):
    def __init__(self, num_heads, head_size, scale, num_kv_heads=None, alibi_slopes=None, sliding_window=None,
                 kv_cache_dtype="auto", logits_soft_cap=None, attn_type="decoder", kv_sharing_target_layer_name=None,
                 **kwargs):
        vllm_config = kwargs.pop("vllm_config", None)
        if vllm_config is None:
            from vllm.config import get_current_vllm_config

            vllm_config = get_current_vllm_config()
        self.vllm_config = vllm_config
        validate_vllm_config(vllm_config)
        num_kv_heads = num_heads if num_kv_heads is None else num_kv_heads
        if alibi_slopes is not None or sliding_window is not None or logits_soft_cap:
            raise ValueError("OSCAR does not implement ALiBi, SWA or logits soft cap")
        if kv_sharing_target_layer_name is not None or kwargs.get("sinks") is not None:
            raise ValueError("OSCAR does not support cross-layer KV sharing or learnable attention sinks")
        if str(attn_type).split(".")[-1].lower() != "decoder" or head_size != 256:
            raise ValueError("OSCAR requires FULL decoder attention with D256")
        if num_kv_heads <= 0 or num_heads % num_kv_heads:
            raise ValueError("query heads must be a positive multiple of KV heads")
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_size = head_size
        self.scale = float(scale)
        self.kv_cache_dtype = kv_cache_dtype
        self.attn_type = attn_type
        spec = getattr(vllm_config, "speculative_config", None)
        self.cfg = OscarConfig.from_env(spec.num_speculative_tokens if spec else 0)
        self.rk = self.rv = None
        self.history = self.window = None
        self.cache_identity = None

    def initialize_layer(self, layer):
        from .rotations import get_rotation

        device = torch.device("cuda", torch.cuda.current_device())
        self.rk = get_rotation(self.cfg.k_rotation_path, layer.layer_name, device)
        self.rv = get_rotation(self.cfg.v_rotation_path, layer.layer_name, device)

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        if output is None:
            raise ValueError("OSCAR needs a preallocated attention output buffer")
        if output_scale is not None or output_block_scale is not None:
            raise ValueError("Fused output quantization is unsupported")
        if attn_metadata is None:
            return output.zero_()
        if self.rk is None or self.rv is None:
            raise RuntimeError("OSCAR rotations were not initialized after model weight loading")
        if key is None or value is None:
            raise ValueError("OSCAR requires the current K/V to maintain exact BF16 windows")
        if not query.is_cuda:
            raise RuntimeError("OSCAR serving kernels run on a CUDA device")
        from . import kernels

        meta = attn_metadata
        n = query.shape[0]
        query = query.view(n, self.num_heads, self.head_size)
        key = key.view(key.shape[0], self.num_kv_heads, self.head_size)
        value = value.view(value.shape[0], self.num_kv_heads, self.head_size)
        if key.shape[0] != n or value.shape[0] != n:
            raise ValueError("Q/K/V must have matching current-token dimensions")
        identity = (kv_cache.data_ptr(), meta.layout)
        if self.cache_identity != identity:
            self.history, self.window = meta.layout.tensor_views(kv_cache)
            self.cache_identity = identity
        if not output.is_contiguous():
            raise ValueError("Attention output must be contiguous")
        if n == 0:
            return output
        if getattr(meta, "prefill_only", False):
            return self._first_prefill(query, key, value, meta, output)
        qrot = kernels.rotate_store(key, value, self.rk, self.rv, self.history, meta.slot_mapping, meta.counts,
                                    meta.layout, query=query)
        splits = decode_split_cap(meta.num_reqs, self.num_kv_heads, meta.max_query_len, n, self.num_heads)
        out = output.view(n, self.num_heads * self.head_size)
        kernels.decode_attention(qrot, query, key, value, self.history, self.window, meta, meta.layout,
                                 self.scale, splits, self.rv, out)
        return output


    def _first_prefill(self, query, key, value, meta, output):
        """Requests that start at position 0: the cache gets the same INT2 history and
        BF16 window writes as on the general path; attention is causal over the current
        bf16 K/V only, computed by this library's tcgen05 prefill kernel (the reference
        hands this case to the vendor's fused attention, backend.py:175-193)."""
        from . import kernels

        kernels.rotate_store(key, value, self.rk, self.rv, self.history, meta.slot_mapping, meta.counts,
                             meta.layout)
        out = output.view(-1, self.num_heads, self.head_size)
        end = int(meta.query_start_loc_cpu[meta.num_reqs])
        kernels.prefill_attention(query, key, value, meta.query_start_loc, meta.num_reqs, meta.max_query_len,
                                  self.scale, out[:end])
        # rows past the step's last request are padding (graph-sized batches): zero, as
        # the reference does after its fused prefill attention
        out[end:].zero_()
        kernels.store_windows(key, value, self.window, meta, meta.layout)
        return output


def enabled() -> bool:
    return os.getenv("OSCAR_ENABLED", os.getenv("OSCAR_ASCEND_ENABLED", "0")) == "1"
