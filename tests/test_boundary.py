"""Host-side boundary: config, layout, rotations, backend/impl surface, plugin routing,
metadata builder checks.  Cases follow the reference's own CPU tests
(tests/test_layout.py, tests/test_rotations.py, tests/test_graph_startup.py)."""

from dataclasses import replace
from types import SimpleNamespace

import pytest
import torch

from oscar_new_b200.config import OscarConfig, choose_splits, percentile_selection
from oscar_new_b200.layout import CacheLayout
from oscar_new_b200.rotations import get_rotation, layer_index, load_checkpoint

# ----------------------------------------------------------------------------
# config / layout (reference tests/test_layout.py)
# ----------------------------------------------------------------------------


@pytest.mark.parametrize("bad", [0, 128, 256, 384, 512, 640, 769])
def test_reject_small_or_nondivisible_page(bad):
    with pytest.raises(ValueError):
        CacheLayout(bad)


def test_pages_resolve_and_do_not_touch_foreign_pages():
    layout = CacheLayout(768)
    pages = 9
    stripe = layout.stripe_page_bytes * pages
    raw = torch.full((2 * stripe,), 0x5A, dtype=torch.uint8)
    cache = raw.view(torch.bfloat16).view(2, -1, 128, 1, 256)
    hist, ring = layout.tensor_views(cache)
    assert hist.data_ptr() == cache[0].data_ptr() and ring.data_ptr() == cache[1].data_ptr()
    table = [p * 6 + j for p in (5, 2, 7) for j in range(6)]
    for t in range(2304):
        begin = layout.slot_offset(layout.logical_slot(table, t))
        hist[begin : begin + 136] = 7
        off = layout.window_offset(table[0], t)
        raw[stripe + off : stripe + off + 512] = 3
    for p in (0, 1, 3, 4, 6, 8):
        assert (hist[p * layout.stripe_page_bytes : (p + 1) * layout.stripe_page_bytes] == 0x5A).all()
    vbytes = raw[stripe:]
    for p in range(pages):
        if p != 5:
            assert (vbytes[p * layout.stripe_page_bytes : (p + 1) * layout.stripe_page_bytes] == 0x5A).all()


def test_ring_preserves_rejection_rollback_and_sink():
    cfg = OscarConfig()
    layout = CacheLayout(768, config=cfg)
    memory, end = {}, 0
    for chunk, rejected in ((1024, 0), (4, 3), (4, 2), (4, 0), (300, 0), (4, 3)):
        prefix = end
        for t in range(max(cfg.sink_tokens, prefix - cfg.recent_tokens), prefix):
            assert memory[layout.window_offset(12, t)] == t
        for t in range(min(prefix, cfg.sink_tokens)):
            assert memory[layout.window_offset(12, t)] == t
        for t in range(prefix, prefix + chunk):
            memory[layout.window_offset(12, t)] = t
        end = prefix + chunk - rejected


def test_window_owner_must_start_a_page():
    layout = CacheLayout(768)
    with pytest.raises(ValueError):
        layout.window_offset(13, 0)


def test_split_policy_and_bad_config():
    assert [choose_splits(b, 1, 4) for b in (1, 16, 128)] == [32, 16, 8]
    assert choose_splits(1, 1, 16384) == 1
    assert percentile_selection(0.96) == (11, 10, pytest.approx(0.8))
    for kwargs in ({"group_size": 128}, {"head_dim": 128}, {"k_clip_ratio": 0.5},
                   {"k_clip_factor": float("nan")}, {"sink_tokens": -1}, {"speculative_tokens": 16},
                   {"clip_mode": "none"}, {"block_n": 8}, {"queries_per_tile": 3}):
        with pytest.raises(ValueError):
            replace(OscarConfig(), **kwargs)


def test_decode_split_cap_bounds_the_scratch():
    from oscar_new_b200.config import decode_split_cap

    assert decode_split_cap(32, 4, 4, 128, 24) == 64  # 200 MB of split scratch
    assert decode_split_cap(256, 4, 4, 1024, 24) == 9  # capped by the 256 MiB budget
    assert decode_split_cap(2048, 4, 4, 8192, 24) == 8  # never below the reference policy
    assert decode_split_cap(1, 1, 900, 900, 6) == 1  # prefill keeps one split


def test_config_reads_reference_environment_names(monkeypatch):
    monkeypatch.setenv("VLLM_OSCAR_SINK_TOKENS", "4")
    monkeypatch.setenv("VLLM_OSCAR_RECENT_TOKENS", "128")
    monkeypatch.setenv("VLLM_OSCAR_K_CLIP_RATIO", "0.92")
    monkeypatch.setenv("OSCAR_ASCEND_CLIP_MODE", "factor")
    cfg = OscarConfig.from_env(speculative_tokens=3)
    assert (cfg.sink_tokens, cfg.recent_tokens, cfg.k_clip_ratio, cfg.clip_mode) == (4, 128, 0.92, "factor")
    assert cfg.ring_tokens == 132 and cfg.window_tokens == 136


# ----------------------------------------------------------------------------
# rotations (reference tests/test_rotations.py)
# ----------------------------------------------------------------------------


@pytest.mark.parametrize("name,expected", [("model.layers.3.self_attn.attn", 3),
                                           ("model.language_model.layers.63.self_attn.attn", 63)])
def test_layer_name(name, expected):
    assert layer_index(name) == expected


def test_missing_layer_or_wrong_dimension_is_not_identity(tmp_path):
    path = tmp_path / "rot.pt"
    torch.save({"layers": {3: {"rotation": torch.eye(256)}}}, path)
    torch.testing.assert_close(get_rotation(str(path), "model.layers.3.attn", "cpu"), torch.eye(256).bfloat16())
    with pytest.raises(ValueError, match="Missing"):
        get_rotation(str(path), "model.layers.7.attn", "cpu")
    with pytest.raises(ValueError, match="D128"):
        get_rotation(str(path), "model.layers.3.attn", "cpu", 128)
    with pytest.raises(ValueError):
        load_checkpoint("")


def test_nonorthogonal_rotation_rejected_also_under_bf16_default(tmp_path):
    path = tmp_path / "bad.pt"
    torch.save({3: torch.ones(256, 256)}, path)
    with pytest.raises(ValueError, match="orthogonal"):
        get_rotation(str(path), "model.layers.3.attn", "cpu")
    prev = torch.get_default_dtype()
    try:
        torch.set_default_dtype(torch.bfloat16)
        with pytest.raises(ValueError, match="orthogonal"):
            get_rotation(str(path), "model.layers.3.attn", "cpu")
    finally:
        torch.set_default_dtype(prev)


def test_three_dimensional_checkpoint(tmp_path):
    q, _ = torch.linalg.qr(torch.randn(256, 256, generator=torch.Generator().manual_seed(2)))
    path = tmp_path / "stack.pt"
    torch.save(torch.stack([torch.eye(256), q]), path)
    torch.testing.assert_close(get_rotation(str(path), "model.layers.1.attn", "cpu"), q.bfloat16())


def test_rotation_file_is_checked_once_for_every_layer(tmp_path):
    """All layers are audited when the file loads; a bad layer does not hide good ones."""
    q, _ = torch.linalg.qr(torch.randn(256, 256, generator=torch.Generator().manual_seed(4)))
    bad = q.clone()
    bad[0, 0] = float("nan")
    path = tmp_path / "mixed.pt"
    torch.save({"layers": {0: {"rotation": q}, 1: bad, 2: torch.eye(128), 5: 2 * torch.eye(256)}}, path)
    f = load_checkpoint(str(path))
    assert sorted(f) == [0, 1, 2, 5] and set(f.problems) == {1, 5}
    assert "non-finite" in f.problems[1] and "orthogonal" in f.problems[5]
    torch.testing.assert_close(get_rotation(str(path), "model.layers.0.attn", "cpu"), q.bfloat16())
    with pytest.raises(ValueError, match="non-finite"):
        get_rotation(str(path), "model.layers.1.attn", "cpu")
    torch.testing.assert_close(get_rotation(str(path), "model.layers.2.attn", "cpu", 128), torch.eye(128).bfloat16())
    with pytest.raises(ValueError, match="D256"):
        get_rotation(str(path), "model.layers.2.attn", "cpu")
    with pytest.raises(ValueError, match="orthogonal"):
        get_rotation(str(path), "model.layers.5.attn", "cpu")
    with pytest.raises(ValueError, match="no decoder layer"):
        get_rotation(str(path), "model.norm", "cpu")
    torch.save({3: "not a matrix"}, tmp_path / "junk.pt")
    with pytest.raises(ValueError, match="no rotation matrix"):
        load_checkpoint(str(tmp_path / "junk.pt"))


def test_step_arena_layout_segments_are_aligned_and_disjoint():
    from oscar_new_b200.kernels import step_arena_layout

    for reqs, cols, cap in ((5, 39, 19), (257, 262, 4096), (1, 1, 1)):
        off = step_arena_layout(reqs, cols, cap)
        assert off["qstarts"] == 4
        ends = [off["qstarts"] + reqs + 1, off["seq_lens"] + reqs, off["table"] + reqs * cols,
                off["tasks"] + 2 * cap]
        starts = [off["qstarts"], off["seq_lens"], off["table"], off["tasks"]]
        assert all(v % 4 == 0 for v in starts + [off["words"]])
        assert all(e <= s for e, s in zip(ends, starts[1:] + [off["words"]]))


# ----------------------------------------------------------------------------
# backend / impl / plugin / builder
# ----------------------------------------------------------------------------


def fake_vllm_config(**over):
    cfg = SimpleNamespace(
        cache_config=SimpleNamespace(enable_prefix_caching=False, cache_dtype="auto"),
        model_config=SimpleNamespace(dtype=torch.bfloat16, hf_text_config=SimpleNamespace(head_dim=256),
                                     max_model_len=4096),
        kv_transfer_config=None,
        parallel_config=SimpleNamespace(decode_context_parallel_size=1, prefill_context_parallel_size=1,
                                        enable_dbo=False),
        speculative_config=SimpleNamespace(num_speculative_tokens=3),
        scheduler_config=SimpleNamespace(max_num_seqs=4, max_num_batched_tokens=32),
        compilation_config=SimpleNamespace(static_forward_context={}),
    )
    for k, v in over.items():
        setattr(cfg, k, v)
    return cfg


def test_backend_surface():
    from oscar_new_b200.backend import OscarAttentionBackend, OscarAttentionImpl
    from oscar_new_b200.metadata import OscarMetadataBuilder

    assert OscarAttentionBackend.forward_includes_kv_cache_update
    assert OscarAttentionBackend.get_name() == "CUSTOM"
    assert OscarAttentionBackend.get_impl_cls() is OscarAttentionImpl
    assert OscarAttentionBackend.get_builder_cls() is OscarMetadataBuilder
    assert OscarAttentionBackend.get_kv_cache_shape(10, 128, 4, 256) == (2, 10, 128, 4, 256)
    with pytest.raises(NotImplementedError):
        OscarAttentionBackend.copy_blocks()
    with pytest.raises(NotImplementedError):
        OscarAttentionBackend.swap_blocks()


def make_impl(**kw):
    from oscar_new_b200.backend import OscarAttentionImpl

    args = dict(num_heads=24, head_size=256, scale=1 / 16, num_kv_heads=4, alibi_slopes=None, sliding_window=None,
                kv_cache_dtype="auto", logits_soft_cap=None, attn_type="decoder", kv_sharing_target_layer_name=None)
    args.update(kw)
    vc = args.pop("vllm_config", fake_vllm_config())
    return OscarAttentionImpl(**args, vllm_config=vc)


def test_impl_validation_generalises_head_counts():
    impl = make_impl()
    assert (impl.num_heads, impl.num_kv_heads) == (24, 4)
    make_impl(num_heads=6, num_kv_heads=1)
    for bad in ({"head_size": 128}, {"num_heads": 10}, {"sliding_window": 128}, {"logits_soft_cap": 30.0},
                {"attn_type": "encoder"}, {"alibi_slopes": [1.0]}, {"kv_sharing_target_layer_name": "x"}):
        with pytest.raises(ValueError):
            make_impl(**bad)
    for over in ({"cache_config": SimpleNamespace(enable_prefix_caching=True, cache_dtype="auto")},
                 {"kv_transfer_config": object()}):
        with pytest.raises(ValueError):
            make_impl(vllm_config=fake_vllm_config(**over))


def test_forward_without_metadata_zeroes_and_refuses_cpu():
    impl = make_impl()
    out = torch.ones(3, 24 * 256, dtype=torch.bfloat16)
    assert impl.forward(None, out, out, out, None, None, out).eq(0).all()
    impl.rk = impl.rv = torch.eye(256)
    q = torch.zeros(3, 24 * 256, dtype=torch.bfloat16)
    kv = torch.zeros(3, 4 * 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        impl.forward(None, q, kv, kv, None, SimpleNamespace(), q.clone())
    impl.rk = None
    with pytest.raises(RuntimeError, match="rotations"):
        impl.forward(None, q, kv, kv, None, SimpleNamespace(), q.clone())


class FakePlatform:
    @classmethod
    def get_attn_backend_cls(cls, selected_backend, attn_selector_config, num_heads=None):
        return "native.Backend"


def test_plugin_routes_decoder_attention_idempotently(monkeypatch):
    from oscar_new_b200 import plugin

    monkeypatch.setenv("OSCAR_ENABLED", "1")
    monkeypatch.setattr(plugin, "_registered", False)
    plugin.register(FakePlatform)
    plugin.register(FakePlatform)  # second call is a no-op
    sel = SimpleNamespace(head_size=256, attn_type="decoder", use_mla=False, use_sparse=False, use_non_causal=False)
    assert FakePlatform.get_attn_backend_cls(None, sel) == plugin.BACKEND_PATH
    assert FakePlatform.get_attn_backend_cls(None, SimpleNamespace(**{**vars(sel), "head_size": 0})) == \
        plugin.BACKEND_PATH
    for change in ({"use_mla": True}, {"attn_type": "encoder_only"}, {"use_non_causal": True}, {"head_size": 128}):
        assert FakePlatform.get_attn_backend_cls(None, SimpleNamespace(**{**vars(sel), **change})) == "native.Backend"
    with pytest.raises(ValueError):
        FakePlatform.get_attn_backend_cls(None, SimpleNamespace(**{**vars(sel), "has_sink": True}))
    assert plugin.is_draft_layer("mtp.layers.0.attn") and not plugin.is_draft_layer("model.layers.3.attn")


def test_plugin_disabled_by_default(monkeypatch):
    from oscar_new_b200 import plugin

    monkeypatch.delenv("OSCAR_ENABLED", raising=False)
    monkeypatch.delenv("OSCAR_ASCEND_ENABLED", raising=False)
    monkeypatch.setattr(plugin, "_registered", False)

    class Untouched(FakePlatform):
        pass

    plugin.register(Untouched)
    assert "_oscar_selector_installed" not in Untouched.__dict__


def test_attention_hooks_keep_draft_layers_native_and_load_rotations():
    from oscar_new_b200 import plugin

    calls = []

    class FakeAttention:
        def __init__(self, num_heads, prefix="", attn_backend=None):
            self.prefix, self.attn_backend = prefix, attn_backend

        def process_weights_after_loading(self, act_dtype):
            calls.append(act_dtype)

    assert plugin._install_loaded_attention_hooks(FakeAttention)
    assert plugin._install_loaded_attention_hooks(FakeAttention)  # idempotent
    layer = FakeAttention(8, prefix="model.layers.3.attn")
    assert layer.attn_backend is None
    layer.process_weights_after_loading(torch.bfloat16)
    assert calls == [torch.bfloat16]


def test_metadata_builder_sizes_and_rejections():
    from oscar_new_b200.metadata import OscarMetadataBuilder, dummy_run_scope, in_dummy_run

    spec = SimpleNamespace(block_size=768, num_kv_heads=4)
    b = OscarMetadataBuilder(spec, ["model.layers.3.attn"], fake_vllm_config(), torch.device("cpu"))
    assert b.max_reqs == 5 and b.max_tokens == 32 + 7 * 5
    assert b.table.shape == (5, 32 + 6 + 1)
    assert OscarMetadataBuilder.get_cudagraph_support(None, None).name == "UNIFORM_BATCH"
    cm = SimpleNamespace(causal=True, num_reqs=1, num_actual_tokens=4, max_query_len=4,
                         block_table_tensor=torch.zeros(1, 6, dtype=torch.int32))
    with pytest.raises(ValueError, match="shared prefixes"):
        b.build(16, cm)
    with pytest.raises(ValueError, match="causal"):
        b.build(0, SimpleNamespace(**{**vars(cm), "causal": False}))
    with pytest.raises(ValueError, match="capacity"):
        b.build(0, SimpleNamespace(**{**vars(cm), "num_reqs": 9}))
    with pytest.raises(ValueError, match="block table"):
        b.build(0, SimpleNamespace(**{**vars(cm), "block_table_tensor": torch.zeros(1, 99, dtype=torch.int32)}))
    assert not in_dummy_run()
    with dummy_run_scope():
        assert in_dummy_run()
    assert not in_dummy_run()
