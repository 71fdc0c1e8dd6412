"""The timeout path of the default decode history kernels and the eigensolver on the GPU.

With the test hook `oscar_test_set_wait_fault`, CTA (0, 0, 0) of the history launch never
issues the copy of its second chunk and every bounded device wait gives up after 4096
probes.  The launch must return, store OSCAR_ERR_TIMEOUT (4) in the status word, mark the
aborted CTA's rows empty and leave the context usable: the next step, without the hook,
matches the oracle with a clear status word.  The same hook makes one CTA of the
eigensolver skip its partial-sum pushes of one round, so its cluster's waits run out.
Nothing here faults or hangs the GPU: the withheld copy or push is never issued, so only
the waits run out.
"""

import pytest
import torch

from oscar_new_b200 import _lib, kernels
from tests.helpers import Scenario, make_config

pytestmark = pytest.mark.gpu
DEV = "cuda"


ATTENTION_KERNEL, MTP_KERNEL = 1, 2  # oscar_last_history_kernel codes (include/oscar_b200.h)


@pytest.mark.parametrize(
    "qlen,mtp,kernel",
    [
        ([1, 1], 0, ATTENTION_KERNEL),  # decode: GQA 6 x 4 KV heads, one row tile
        ([4, 4], 3, MTP_KERNEL),  # MTP verify: 4 query tokens x GQA 6 = 3 row tiles
    ],
)
def test_wait_timeout_reports_status_and_context_recovers(cuda_lib, monkeypatch, qlen, mtp, kernel):
    monkeypatch.delenv("OSCAR_HISTORY_F8", raising=False)
    sc = Scenario([1500, 2600], qlen, hq=24, h=4, cfg=make_config(4, 128, mtp), seed=93 + mtp)
    n = sum(qlen)
    q, k, v = sc.current()
    sc.prepare_tasks()
    rk, rv = sc.rk.to(DEV), sc.rv.to(DEV)
    qrot = kernels.rotate_store(k, v, rk, rv, sc.history, sc.meta.slot_mapping, sc.meta.counts, sc.layout, query=q)
    kernels.read_status(DEV)  # start from a clear word
    out = torch.empty((n, 24 * 256), dtype=torch.bfloat16, device=DEV)
    lib = _lib.lib()
    assert lib.oscar_test_set_wait_fault(1, 4096) == 0
    try:
        kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, 8, rv, out,
                                 store_window=False)
        torch.cuda.synchronize()
    finally:
        assert lib.oscar_test_set_wait_fault(-1, 0) == 0
    assert lib.oscar_last_history_kernel() == kernel
    assert kernels.read_status(DEV) == 4
    kernels.decode_attention(qrot, q, k, v, sc.history, sc.window, sc.meta, sc.layout, 1 / 16, 8, rv, out,
                             store_window=False)
    assert kernels.read_status(DEV) == 0
    expect, _ = sc.expected()
    torch.testing.assert_close(out.view(n, 24, 256).float().cpu(), expect, atol=0.035, rtol=0.04)


def test_eigensolver_wait_timeout_reports_status_and_context_recovers(cuda_lib):
    """With the hook, CTA 0 of the first matrix's cluster never pushes its partial sums of
    round 1 and every wait gives up after 4096 probes: that cluster stops with info status
    3 in its first sweep and the host publishes nothing; the other matrices of the launch
    are unaffected, and the next launch without the hook converges to eigvalsh."""
    from oscar_new_b200 import calibration_kernels as ck

    torch.manual_seed(41)
    x = torch.randn(3, 512, 256)
    x[..., :8] *= 5
    cov = (x.transpose(-1, -2) @ x / 512).to(DEV)
    rot = torch.empty_like(cov)
    ev = torch.empty((3, 256), device=DEV)
    info = torch.zeros((3, 4), device=DEV)
    lib = _lib.lib()
    assert lib.oscar_test_set_wait_fault(1, 4096) == 0
    try:
        assert lib.oscar_jacobi_rotations(cov.data_ptr(), 3, 12, 1e-7, rot.data_ptr(), ev.data_ptr(),
                                          info.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        host = info.cpu()
        assert host[0, 2] == 3 and host[0, 0] == 0, host[0]
        assert (host[1:, 2] == 0).all() and (host[1:, 1] < 1e-6).all(), host[1:]
        with pytest.raises(RuntimeError, match="device wait timed out"):
            ck.calibrated_rotations(cov)
    finally:
        assert lib.oscar_test_set_wait_fault(-1, 0) == 0
    _, ev2, result = ck.calibrated_rotations(cov)
    assert result["relative_off_diagonal"] < 1e-6
    ref = torch.linalg.eigvalsh(cov.cpu().double())
    assert float(((ev2.cpu().double() - ref).abs() / ref.abs()).max()) < 1e-4
