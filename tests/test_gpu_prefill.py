"""The tcgen05 first-prefill attention kernel (causal, current tokens only) against the
CPU oracle's dense fp32 attention: ragged lengths around the 128-query / 64-key block
edges (1, 63, 64, 65, 127, 128, 129 tokens), longer requests, GQA 6, a strided query
view (a slice of fused QKV rows), and one 8192-token request against torch's
flash-attention kernel.  Output rel 1e-2 in norm, atol .02 / rtol .02 per element."""

import pytest
import torch

from oracle import int2_oracle as oo
from oscar_new_b200 import kernels

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.mark.parametrize("lens", [[1, 63, 64, 65, 127, 128, 129], [300, 1000, 2500, 17]])
def test_prefill_matches_dense_oracle(cuda_lib, lens):
    g = torch.Generator().manual_seed(sum(lens))
    n, hq, hkv = sum(lens), 24, 4
    qkv = torch.randn(n, hq + 2 * hkv, 256, generator=g)
    qkv[:, hq:hq + hkv, :8] *= 20  # outlier key channels
    qkv = qkv.bfloat16().to(DEV)
    q, k, v = qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:]  # strided views, as in vLLM
    starts = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    out = kernels.prefill_attention(q, k, v, starts, len(lens), max(lens), 1 / 16)
    torch.cuda.synchronize()
    assert kernels.read_status(DEV) == 0
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    for i, ln in enumerate(lens):
        a, b = int(starts[i]), int(starts[i]) + ln
        want = oo.dense_attention(qc[a:b], kc[a:b], vc[a:b], 0)
        got = out[a:b].float().cpu()
        assert rel_err(got, want) < 1e-2, (ln, rel_err(got, want))
        torch.testing.assert_close(got, want, atol=0.02, rtol=0.02)


def test_prefill_long_request_matches_flash_attention(cuda_lib):
    import torch.nn.functional as F

    g = torch.Generator(device=DEV).manual_seed(8)
    n = 8192
    q = torch.randn(n, 24, 256, device=DEV, generator=g).bfloat16()
    k = torch.randn(n, 4, 256, device=DEV, generator=g).bfloat16()
    v = torch.randn(n, 4, 256, device=DEV, generator=g).bfloat16()
    starts = torch.tensor([0, n], dtype=torch.int32, device=DEV)
    out = kernels.prefill_attention(q, k, v, starts, 1, n, 1 / 16)
    ref = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
                                         is_causal=True, enable_gqa=True, scale=1 / 16)[0].transpose(0, 1)
    assert rel_err(out, ref) < 1e-2, rel_err(out, ref)
