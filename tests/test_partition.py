"""The KV head x request partition of one attention workload over the GPUs of a box
(host logic), and two gloo ranks that each run the CPU oracle on their shard: the
stitched result equals the unsharded one."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import int2_oracle as oo
from oscar_new_b200.partition import balance_requests, head_split, partition, shard_of
from tests.helpers import make_config, oo_outlier


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("kv_heads", [1, 4, 8])
def test_every_request_head_pair_has_exactly_one_rank(world, kv_heads):
    gen = torch.Generator().manual_seed(world * 10 + kv_heads)
    ctx = torch.randint(2048, 262144, (33,), generator=gen).tolist()
    shards = partition(ctx, kv_heads, world)
    assert [s.rank for s in shards] == list(range(world))
    tp = head_split(kv_heads, world)
    owner = {}
    for s in shards:
        assert s.kv_heads == kv_heads // tp
        assert list(s.requests) == sorted(s.requests)
        for r in s.requests:
            for h in range(s.head_begin, s.head_end):
                assert (r, h) not in owner
                owner[(r, h)] = s.rank
    assert len(owner) == len(ctx) * kv_heads
    assert shard_of(world - 1, ctx, kv_heads, world) == shards[-1]


def test_heads_split_first_then_requests():
    assert [head_split(4, w) for w in (1, 2, 4, 8)] == [1, 2, 4, 4]
    assert [head_split(4, w, 2) for w in (1, 2, 4, 8)] == [1, 2, 2, 2]
    assert [head_split(8, w, 2) for w in (1, 2, 4, 8)] == [1, 2, 4, 4]
    assert head_split(6, 6, 2) == 3 and head_split(6, 4, 2) == 2
    shards = partition([100] * 8, 4, 8, 2)  # TP2 x 4 request groups
    assert {(s.head_begin, s.head_end) for s in shards} == {(0, 2), (2, 4)}
    assert len({s.requests for s in shards}) == 4
    shards = partition([100] * 8, 4, 8)  # TP4 (one KV head per rank) x 2 request groups
    assert [(s.head_begin, s.head_end) for s in shards[:4]] == [(0, 1), (1, 2), (2, 3), (3, 4)]
    assert shards[0].requests == shards[3].requests and not set(shards[0].requests) & set(shards[4].requests)
    assert list(shards[1].query_heads(6)) == list(range(6, 12))


def test_requests_balanced_by_total_context():
    gen = torch.Generator().manual_seed(3)
    ctx = torch.exp(torch.empty(32, dtype=torch.float64).uniform_(8 * 0.6931, 18 * 0.6931, generator=gen)).long()
    for groups in (2, 4, 8):
        loads = [sum(int(ctx[r]) for r in g) for g in balance_requests(ctx.tolist(), groups)]
        assert max(loads) - sum(loads) / groups < int(ctx.max())
    with pytest.raises(ValueError):
        balance_requests([1, 2], 0)
    with pytest.raises(ValueError):
        shard_of(2, [1], 1, 2)


# ---------------------------------------------------------------------------
# two gloo ranks, each computing its shard with the oracle
# ---------------------------------------------------------------------------

SEQ = [300, 1000, 2500, 700, 1600]
QLEN = [1, 1, 4, 1, 2]
KV, GROUP = 2, 4


def _problem():
    gen = torch.Generator().manual_seed(2024)
    ks = [oo_outlier(gen, s, KV) for s in SEQ]
    vs = [torch.randn(s, KV, 256, generator=gen).bfloat16() for s in SEQ]
    qs = [torch.randn(q, KV * GROUP, 256, generator=gen).bfloat16() for q in QLEN]
    from oscar_new_b200.synthetic import rotation

    return ks, vs, qs, rotation(1).bfloat16(), rotation(2).bfloat16(), make_config(4, 64, 3)


def _shard_outputs(requests, head_begin, head_end):
    """{request: oracle output [qlen, heads of the shard, 256]} from the shard's own slices."""
    ks, vs, qs, rk, rv, cfg = _problem()
    out = {}
    for r in requests:
        k, v = ks[r][:, head_begin:head_end], vs[r][:, head_begin:head_end]
        q = qs[r][:, head_begin * GROUP:head_end * GROUP]
        out[r] = oo.hybrid_reference(q, k, v, SEQ[r] - QLEN[r], rk, rv, cfg)
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, kv_heads_used, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = shard_of(rank, SEQ, kv_heads_used, world)
        per = KV // kv_heads_used  # real KV heads per partitioned head unit
        mine = _shard_outputs(shard.requests, shard.head_begin * per, shard.head_end * per)
        gathered = [None] * world
        dist.all_gather_object(gathered, (shard, mine))
        if rank == 0:
            torch.save(gathered, os.path.join(outdir, "gathered.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kv_heads_used", [KV, 1])
def test_two_gloo_ranks_stitch_to_the_unsharded_result(tmp_path, kv_heads_used):
    """KV = 2: tensor parallel over the two heads; kv_heads_used = 1 (the heads treated as
    one unit): the two ranks split the requests."""
    mp.spawn(_rank_main, args=(2, _free_port(), kv_heads_used, str(tmp_path)), nprocs=2, join=True)
    gathered = torch.load(tmp_path / "gathered.pt", weights_only=False)
    assert [s.rank for s, _ in gathered] == [0, 1]
    per = KV // kv_heads_used
    full = _shard_outputs(range(len(SEQ)), 0, KV)
    got = {r: torch.zeros_like(full[r]) for r in full}
    seen = torch.zeros(len(SEQ), KV, dtype=torch.int32)
    for shard, outs in gathered:
        hb, he = shard.head_begin * per, shard.head_end * per
        for r, o in outs.items():
            assert o.shape[1] == (he - hb) * GROUP
            got[r][:, hb * GROUP:he * GROUP] = o
            seen[r, hb:he] += 1
    assert (seen == 1).all()
    for r in full:
        torch.testing.assert_close(got[r], full[r], atol=2e-6, rtol=2e-6)
