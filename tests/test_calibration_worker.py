"""Calibration worker host logic on CPU: pass/phase rules, token budgets, the covariance
stack, sharding over gloo ranks and the published checkpoint (reference
oscar_ascend/calibration_worker.py:53-180 and tests/test_calibration_math.py).

The device arithmetic is replaced by fp64 CPU restatements from the oracle; the
eigensolver is ``torch.linalg.eigh`` + the oracle's ``U H P_br`` composition."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import calibration_oracle as co
from oscar_new_b200.calibration_worker import CalibrationSession
from oscar_new_b200.rotations import get_rotation, load_checkpoint

D = 256


class CpuOps:
    @staticmethod
    def accumulate_gram(x, cov, weights=None):
        cov += (co.gram(x) if weights is None else co.weighted_gram(x, weights)).float()

    @staticmethod
    def sst_weights(k, q_cov, total):
        w = co.sst_weights(k, q_cov).float()
        total += w.sum()
        return w

    @staticmethod
    def accumulate_gram_grouped(x, covs, weights=None):
        groups = covs.shape[0]
        per = x.shape[1] // groups
        w = None if weights is None else weights.reshape(x.shape[0], x.shape[1])
        for gi in range(groups):
            sl = slice(gi * per, (gi + 1) * per)
            CpuOps.accumulate_gram(x[:, sl], covs[gi], None if w is None else w[:, sl])

    @staticmethod
    def sst_weights_per_head(k, q_covs, totals):
        w = torch.stack([co.sst_weights(k[:, j : j + 1], q_covs[j]).float() for j in range(k.shape[1])], 1)
        totals += w.sum(0)
        return w.reshape(-1)

    @staticmethod
    def normalize(x, denominator):
        if isinstance(denominator, torch.Tensor):
            return x / denominator.clamp_min(1e-30)
        return x / max(float(denominator), 1e-30)


def eigh_rotations(covariances, max_sweeps=12):
    evals, vecs = torch.linalg.eigh(covariances.double())
    rot = torch.stack([co.compose(v) for v in vecs]).float()
    return rot, evals.float(), {"sweeps": 0, "relative_off_diagonal": 0.0}


def activations(layers, tokens, heads, group, seed=0):
    """Seeded Q/K/V with heavy-tailed outlier channels (config 5 generator, small)."""
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for layer in layers:
        q = torch.randn(tokens, heads * group, D, generator=gen)
        k = torch.randn(tokens, heads, D, generator=gen)
        v = torch.randn(tokens, heads, D, generator=gen)
        for x in (q, k, v):
            shape = x[..., :8].shape
            chi2 = torch.randn(*shape, 3, generator=gen).square().sum(-1)  # Student-t, nu = 3
            x[..., :8] = 20 * (torch.randn(*shape, generator=gen) / (chi2 / 3).sqrt()).clamp(-50, 50)
        out[layer] = (q.bfloat16(), k.bfloat16(), v.bfloat16())
    return out


def expected_stack(data, heads, group, head_subset=None):
    """fp64 [Cq, Cv] per layer, averaged over KV heads (reference :131-139)."""
    mats = []
    for layer in sorted(data):
        q, k, v = data[layer]
        n = q.shape[0]
        hs = range(heads) if head_subset is None else head_subset
        cq_sum = cv_sum = 0
        for h in hs:
            cq = co.gram(q[:, h * group : (h + 1) * group]) / (n * group)
            w = co.sst_weights(k[:, h : h + 1], cq)
            cv = co.weighted_gram(v[:, h : h + 1], w) / w.sum()
            cq_sum, cv_sum = cq_sum + cq, cv_sum + cv
        mats.extend((cq_sum / len(hs), cv_sum / len(hs)))
    return torch.stack(mats)


def run_passes(session, data, chunk, rows=None, heads=None):
    for phase in (1, 2):
        for layer, (q, k, v) in data.items():
            sel = slice(None) if rows is None else rows
            qq, kk, vv = q[sel], k[sel], v[sel]
            if heads is not None:
                g = qq.shape[1] // k.shape[1]
                qq = torch.cat([qq[:, h * g : (h + 1) * g] for h in heads], 1)
                kk, vv = kk[:, heads], vv[:, heads]
            for start in range(0, qq.shape[0], chunk):
                session.observe(layer, qq[start : start + chunk], kk[start : start + chunk],
                                vv[start : start + chunk], qq[start : start + chunk].shape[0])
        if phase == 1:
            session.second_pass()


def rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


def test_single_process_stack_matches_fp64_restatement():
    data = activations([0, 5], 400, 2, 3)
    s = CalibrationSession([0, 5], 10**9, "cpu", num_kv_heads=2, group_size=3, ops=CpuOps)
    run_passes(s, data, chunk=128)
    got = s.covariances()
    assert rel(got, expected_stack(data, 2, 3)) < 1e-5


def test_budget_limits_pass_one_and_pass_two_follows_it():
    data = activations([1], 700, 1, 2, seed=3)
    s = CalibrationSession([1, 2], 300, "cpu", num_kv_heads=1, group_size=2, ops=CpuOps)
    with pytest.raises(RuntimeError, match="Insufficient"):
        s.second_pass()  # layer 2 never observed
    s = CalibrationSession([1], 300, "cpu", num_kv_heads=1, group_size=2, ops=CpuOps)
    run_passes(s, data, chunk=128)
    assert s.states[1]["q_tokens"] == 300 and s.states[1]["v_tokens"] == 300
    trimmed = {1: tuple(x[:300] for x in data[1])}
    assert rel(s.covariances(), expected_stack(trimmed, 1, 2)) < 1e-5
    s.observe(7, *data[1], 700)  # unknown layer: ignored


def test_pass_mismatch_is_rejected():
    data = activations([0], 300, 1, 2, seed=4)
    s = CalibrationSession([0], 10**9, "cpu", num_kv_heads=1, group_size=2, ops=CpuOps)
    s.observe(0, *data[0], 300)
    s.second_pass()
    s.observe(0, *(x[:100] for x in data[0]), 100)
    with pytest.raises(RuntimeError, match="mismatch"):
        s.covariances()


def test_finish_publishes_loadable_checkpoints(tmp_path):
    data = activations([2, 3], 300, 1, 2, seed=5)
    s = CalibrationSession([2, 3], 10**9, "cpu", num_kv_heads=1, group_size=2, ops=CpuOps)
    run_passes(s, data, chunk=300)
    info = s.finish(tmp_path, {"model_fingerprint": "synthetic"}, 12, eigensolver=eigh_rotations)
    assert info["published"]
    for kind in ("k", "v"):
        ck = torch.load(tmp_path / f"{kind}_rotation.pt", weights_only=True)
        assert ck["format_version"] == 1 and ck["source_grouping"] == "layer"
        assert sorted(ck["layers"]) == [2, 3] and ck["calibration"]["tokens_per_layer"] == {2: 300, 3: 300}
        # every matrix is stored on its own, not as a view of the K + V stack
        assert all(e["rotation"].untyped_storage().nbytes() == D * D * 4 for e in ck["layers"].values())
        r = get_rotation(str(tmp_path / f"{kind}_rotation.pt"), "model.layers.3.self_attn.attn", "cpu")
        assert r.dtype == torch.bfloat16 and r.shape == (D, D)
    assert not list(tmp_path.glob("*.tmp"))
    load_checkpoint.cache_clear()


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _rank_main(rank, world, port, shard, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        data = activations([0, 4], 512, 2, 3, seed=11)
        if shard == "tokens":
            s = CalibrationSession([0, 4], 10**9, "cpu", 2, 3, shard="tokens", group=dist.group.WORLD, ops=CpuOps)
            run_passes(s, data, chunk=96, rows=slice(rank * 256, (rank + 1) * 256))
        else:
            s = CalibrationSession([0, 4], 10**9, "cpu", 1, 3, shard="heads", group=dist.group.WORLD, ops=CpuOps)
            run_passes(s, data, chunk=96, heads=[rank])
        stack = s.covariances()
        torch.save(stack, os.path.join(outdir, f"{shard}_{rank}.pt"))
        s.finish(os.path.join(outdir, shard), {"model_fingerprint": "x"}, 12, eigensolver=eigh_rotations)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shard", ["tokens", "heads"])
def test_two_rank_gloo_sharding_matches_single_process(tmp_path, shard):
    mp.spawn(_rank_main, args=(2, _free_port(), shard, str(tmp_path)), nprocs=2, join=True)
    data = activations([0, 4], 512, 2, 3, seed=11)
    expect = expected_stack(data, 2, 3)
    stacks = [torch.load(tmp_path / f"{shard}_{r}.pt") for r in range(2)]
    assert torch.equal(stacks[0], stacks[1])
    # finish() all-reduced once more on top of covariances(); the published files come from rank 0
    assert rel(stacks[0], expect) < 1e-5
    ck = torch.load(tmp_path / shard / "k_rotation.pt", weights_only=True)
    assert ck["calibration"]["world_size"] == 2 and ck["calibration"]["shard"] == shard
    assert not (tmp_path / shard / "k_rotation.pt.tmp").exists()


def test_finish_rejects_a_rotation_that_is_not_orthogonal(tmp_path):
    """The publication check (R^T R within 0.005 of I, finite entries) stops finish
    before the failing kind's checkpoint is written (kinds are published in the order
    k, v, as in the reference); the message names the kind and layer."""
    data = activations([3, 7], 300, 1, 2, seed=6)
    s = CalibrationSession([3, 7], 10**9, "cpu", num_kv_heads=1, group_size=2, ops=CpuOps)
    run_passes(s, data, chunk=300)

    def bad_solver(covariances, max_sweeps=12):
        rotations, eigenvalues, info = eigh_rotations(covariances, max_sweeps=max_sweeps)
        rotations = rotations.clone()
        rotations[3] *= 1.01  # layer 7, value rotation: R^T R = 1.0201 I
        return rotations, eigenvalues, info

    with pytest.raises(RuntimeError, match="v rotation for layer 7 failed validation"):
        s.finish(tmp_path, {"model_fingerprint": "x"}, 12, eigensolver=bad_solver)
    assert not (tmp_path / "v_rotation.pt").exists() and not list(tmp_path.glob("*.tmp"))
