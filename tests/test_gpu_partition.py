"""The KV head x request partition on the GPU: every rank's shard (its requests, its KV
heads and their query heads, a cache holding only those heads) runs the decode kernels
on its own, and the stitched outputs match the oracle of the unsharded batch.  The ranks
run one after another on one GPU (no kernel waits on another rank)."""

import pytest
import torch

from oscar_new_b200.partition import partition
from tests.helpers import Scenario, make_config, shard_scenario

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_stitches_to_the_unsharded_oracle(cuda_lib, world):
    seq = [700, 5200, 1900, 9000, 300, 2600, 4100]
    qlen = [4, 1, 4, 2, 4, 1, 3]
    sc = Scenario(seq, qlen, hq=24, h=4, cfg=make_config(4, 128, 3), seed=60 + world)
    expect, _ = sc.expected()
    starts = [0]
    for q in qlen:
        starts.append(starts[-1] + q)
    got = torch.full_like(expect, float("nan"))
    for shard in partition(seq, 4, world):
        part = shard_scenario(sc, shard, seed=shard.rank)
        out = part.run_step(splits=16).float().cpu()
        row = 0
        heads = shard.query_heads(6)
        for r in shard.requests:
            got[starts[r]:starts[r + 1], heads.start:heads.stop] = out[row:row + qlen[r]]
            row += qlen[r]
    assert not torch.isnan(got).any()
    assert rel_err(got, expect) < 1e-2, rel_err(got, expect)
    torch.testing.assert_close(got, expect, atol=0.035, rtol=0.04)
