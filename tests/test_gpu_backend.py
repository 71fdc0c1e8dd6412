"""The vLLM-facing boundary on the GPU: ``OscarMetadataBuilder.build`` + ``OscarAttentionImpl``
(rotations loaded from a ``.pt`` file after "weight loading") against the CPU oracle,
eagerly and replayed from a CUDA graph captured under the dummy-run scope (reference
tests/test_graph_startup.py and tests/test_npu_kernels.py:197-245, on vLLM's CUDA worker)."""

from dataclasses import replace
from types import SimpleNamespace

import pytest
import torch

from oscar_new_b200.backend import OscarAttentionImpl
from oscar_new_b200.metadata import OscarMetadataBuilder
from tests.helpers import Scenario, make_config
from tests.test_boundary import fake_vllm_config

pytestmark = pytest.mark.gpu
DEV = "cuda"
LAYER = "model.layers.3.self_attn.attn"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.fixture()
def oscar_env(monkeypatch, tmp_path):
    sc = Scenario([300, 2049, 900], [1, 4, 3], hq=24, h=4, cfg=make_config(4, 128, 3), seed=21)
    for name, rot in (("k", sc.rk), ("v", sc.rv)):
        path = tmp_path / f"{name}.pt"
        torch.save({"layers": {3: {"rotation": rot.float()}}}, path)
        monkeypatch.setenv(f"VLLM_OSCAR_{name.upper()}_ROTATION_PATH", str(path))
    monkeypatch.setenv("VLLM_OSCAR_SINK_TOKENS", "4")
    monkeypatch.setenv("VLLM_OSCAR_RECENT_TOKENS", "128")
    vc = fake_vllm_config(
        scheduler_config=SimpleNamespace(max_num_seqs=3, max_num_batched_tokens=16),
        speculative_config=SimpleNamespace(num_speculative_tokens=3),
    )
    impl = OscarAttentionImpl(24, 256, 1 / 16, num_kv_heads=4, vllm_config=vc)
    impl.initialize_layer(SimpleNamespace(layer_name=LAYER))
    builder = OscarMetadataBuilder(SimpleNamespace(block_size=768, num_kv_heads=4), [LAYER], vc, torch.device(DEV))
    return sc, impl, builder


def common_metadata(sc):
    p = sc.plan
    seq = torch.tensor(p.seq_lens, dtype=torch.int32)
    return SimpleNamespace(query_start_loc=p.query_start_loc.to(DEV), seq_lens=seq.to(DEV),
                           block_table_tensor=p.block_tables.to(DEV), slot_mapping=p.slot_mapping.to(DEV),
                           num_reqs=len(p.seq_lens), num_actual_tokens=int(p.counts[1]),
                           max_query_len=max(p.query_lens), max_seq_len=max(p.seq_lens), causal=True)


def test_impl_forward_through_builder_matches_oracle(cuda_lib, oscar_env):
    sc, impl, builder = oscar_env
    assert replace(impl.cfg, k_rotation_path="", v_rotation_path="") == sc.cfg
    torch.testing.assert_close(impl.rk.cpu(), sc.rk)
    meta = builder.build(0, common_metadata(sc))
    q, k, v = sc.current()
    n = q.shape[0]
    out = torch.empty((n, 24 * 256), dtype=torch.bfloat16, device=DEV)
    impl.forward(None, q.view(n, -1), k.view(n, -1), v.view(n, -1), sc.cache, meta, out)
    got = out.view(n, 24, 256).float().cpu()
    expect, _ = sc.expected()
    assert rel_err(got, expect) < 1e-2, rel_err(got, expect)
    torch.testing.assert_close(got, expect, atol=0.035, rtol=0.04)


def test_impl_forward_replays_from_graph_captured_as_dummy(cuda_lib, oscar_env):
    sc, impl, builder = oscar_env
    q, k, v = sc.current()
    n = q.shape[0]
    q2, k2, v2 = (x.view(n, -1).clone() for x in (q, k, v))
    out = torch.zeros((n, 24 * 256), dtype=torch.bfloat16, device=DEV)
    cm = common_metadata(sc)
    capture_meta = builder.build_for_cudagraph_capture(cm)
    assert capture_meta.is_dummy and int(builder.counts.sum()) == 0

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            impl.forward(None, q2, k2, v2, sc.cache, capture_meta, out)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    raw = sc.cache.view(-1).view(torch.uint8)  # packed bytes may read as bf16 NaN
    before = raw.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        impl.forward(None, q2, k2, v2, sc.cache, capture_meta, out)
    torch.cuda.synchronize()
    assert torch.equal(raw, before), "a zero-count (dummy) step touched the cache"
    # a real step refills the builder's fixed buffers; the graph replays with them
    meta = builder.build(0, cm)
    assert meta.counts.data_ptr() == capture_meta.counts.data_ptr()
    graph.replay()
    torch.cuda.synchronize()
    got = out.view(n, 24, 256).float().cpu()
    expect, _ = sc.expected()
    assert rel_err(got, expect) < 1e-2, rel_err(got, expect)
    del graph


def test_first_prefill_uses_the_prefill_kernel_and_writes_the_same_cache(cuda_lib, oscar_env, monkeypatch):
    """A batch whose host length bound equals its query lengths (no history yet) runs
    the tcgen05 prefill kernel; the same batch without the bound runs the general path.
    Outputs match the dense oracle; the caches are byte-identical."""
    _, impl, _ = oscar_env
    vc = fake_vllm_config(scheduler_config=SimpleNamespace(max_num_seqs=3, max_num_batched_tokens=2048),
                          speculative_config=SimpleNamespace(num_speculative_tokens=3))
    builder = OscarMetadataBuilder(SimpleNamespace(block_size=768, num_kv_heads=4), [LAYER], vc, torch.device(DEV))
    results = []
    for with_bound in (True, False):
        sc = Scenario([300, 1100], [300, 1100], hq=24, h=4, cfg=make_config(4, 128, 3), seed=44, fill="none",
                      rk=impl.rk.cpu(), rv=impl.rv.cpu())
        cm = common_metadata(sc)
        cm.query_start_loc_cpu = sc.plan.query_start_loc.clone()
        cm.seq_lens_cpu_upper_bound = torch.tensor(sc.plan.seq_lens, dtype=torch.int32) if with_bound else None
        meta = builder.build(0, cm)
        assert meta.prefill_only == with_bound
        q, k, v = sc.current()
        n = q.shape[0]
        out = torch.empty((n, 24 * 256), dtype=torch.bfloat16, device=DEV)
        impl.forward(None, q.view(n, -1), k.view(n, -1), v.view(n, -1), sc.cache, meta, out)
        got = out.view(n, 24, 256).float().cpu()
        expect, _ = sc.expected()
        assert rel_err(got, expect) < 1e-2, (with_bound, rel_err(got, expect))
        torch.testing.assert_close(got, expect, atol=0.035, rtol=0.04)
        results.append(sc.cache.view(-1).view(torch.uint8).cpu())
    assert torch.equal(results[0], results[1])
