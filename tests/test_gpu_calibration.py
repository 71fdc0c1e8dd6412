"""Calibration worker on the GPU: both passes through the CUDA Gram / SST kernels, the
device eigensolver and publication, against fp64 restatements (config-5 generator at a
reduced size: 2 layers, 4 KV heads x 6 query heads, 3 x 1024 tokens).  The NCCL case
shards the tokens over two GPUs, so ``second_pass`` and ``finish`` each all-reduce."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oscar_new_b200.calibration_worker import CalibrationSession
from tests.test_calibration_worker import activations, expected_stack

pytestmark = pytest.mark.gpu
LAYERS, H, G, TOKENS, CHUNK = [3, 9], 4, 6, 3072, 1024


def feed(session, data, device, rows=None):
    for phase in (1, 2):
        for layer, (q, k, v) in data.items():
            sel = slice(None) if rows is None else rows
            qq, kk, vv = (x[sel].to(device) for x in (q, k, v))
            for start in range(0, qq.shape[0], CHUNK):
                end = start + CHUNK
                session.observe(layer, qq[start:end].reshape(-1, H * G * 256), kk[start:end].reshape(-1, H * 256),
                                vv[start:end].reshape(-1, H * 256), qq[start:end].shape[0])
        if phase == 1:
            session.second_pass()


def check_stack(got, expect):
    torch.testing.assert_close(got.cpu().double(), expect, atol=2e-4, rtol=2e-4)


def test_worker_passes_and_publication_on_device(cuda_lib, tmp_path):
    data = activations(LAYERS, TOKENS, H, G, seed=31)
    s = CalibrationSession(LAYERS, 10**9, "cuda", num_kv_heads=H, group_size=G)
    feed(s, data, "cuda")
    stack = s.covariances()
    check_stack(stack, expected_stack(data, H, G))
    info = s.finish(tmp_path, {"model_fingerprint": "synthetic-config5"}, 12)
    assert info["published"] and info["relative_off_diagonal"] < 1e-6
    ref = torch.linalg.eigvalsh(stack.cpu().double())
    eye = torch.eye(256, dtype=torch.float64)
    for kind, offset in (("k", 0), ("v", 1)):
        ck = torch.load(tmp_path / f"{kind}_rotation.pt", weights_only=True)
        for number, layer in enumerate(LAYERS):
            entry = ck["layers"][layer]
            ev = entry["eigenvalues"].double()
            expect = ref[2 * number + offset]
            assert float(((ev - expect).abs() / expect.abs()).max()) < 1e-4
            r = entry["rotation"].double()
            assert float((r.T @ r - eye).norm()) < 1e-5


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _nccl_rank(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        data = activations(LAYERS, TOKENS, H, G, seed=31)
        share = TOKENS // world
        s = CalibrationSession(LAYERS, 10**9, f"cuda:{rank}", H, G, shard="tokens", group=dist.group.WORLD)
        feed(s, data, f"cuda:{rank}", rows=slice(rank * share, (rank + 1) * share))
        torch.save(s.covariances().cpu(), os.path.join(outdir, f"stack_{rank}.pt"))
        info = s.finish(os.path.join(outdir, "pub"), {"model_fingerprint": "x"}, 12)
        torch.save(info, os.path.join(outdir, f"info_{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_token_sharded_calibration_over_nccl(cuda_lib, tmp_path):
    mp.spawn(_nccl_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    data = activations(LAYERS, TOKENS, H, G, seed=31)
    stacks = [torch.load(tmp_path / f"stack_{r}.pt") for r in range(2)]
    assert torch.equal(stacks[0], stacks[1])
    check_stack(stacks[0], expected_stack(data, H, G))
    infos = [torch.load(tmp_path / f"info_{r}.pt") for r in range(2)]
    assert infos[0]["published"] and not infos[1]["published"]
    assert (tmp_path / "pub" / "v_rotation.pt").exists()
