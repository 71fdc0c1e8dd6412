"""OSCAR calibration operators on B200 (reference ``oscar_ascend/calibration_kernels.py``).

Same names and meaning as the reference: ``accumulate_gram``, ``sst_weights``,
``normalize``, ``calibrated_rotations``.  The eigensolver runs every Jacobi sweep in a
single launch (one 8-CTA thread-block cluster per matrix) and returns its convergence
info; only that small info vector is read back to decide success, as the reference
reads one residual scalar.
"""

from __future__ import annotations

import torch

from . import _lib
from .kernels import status_word


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("calibration kernels run on a CUDA device only")


def accumulate_gram(x: torch.Tensor, covariance: torch.Tensor, weights: torch.Tensor | None = None):
    """``covariance += X^T X`` over all rows/heads of bf16 ``x`` [n, h, 256], or the
    ``weights``-weighted sum (reference calibration_kernels.py:59-70)."""
    _cuda(x, covariance, weights)
    if covariance.dtype != torch.float32 or covariance.shape != (256, 256) or not covariance.is_contiguous():
        raise ValueError("covariance must be contiguous fp32 [256, 256]")
    n, h, d = x.shape
    if d != 256:
        raise ValueError("head_dim must be 256")
    if x.dtype != torch.bfloat16 or x.stride(2) != 1 or x.stride(0) % 8 or x.stride(1) % 8 or x.data_ptr() % 16:
        x = x.to(torch.bfloat16).contiguous()
    w = None
    if weights is not None:
        w = weights.float().contiguous().view(-1)
        if w.numel() != n * h:
            raise ValueError("weights must have one entry per (token, head) row")
    _lib.call("oscar_accumulate_gram", x.data_ptr(), n, h, x.stride(0), x.stride(1),
              None if w is None else w.data_ptr(), covariance.data_ptr(), _stream(x))


def accumulate_gram_grouped(x: torch.Tensor, covariances: torch.Tensor, weights: torch.Tensor | None = None):
    """``covariances[g] += sum over the rows of head group g`` (x [n, h, 256]; the h
    heads split into ``covariances.shape[0]`` equal groups of consecutive heads) in one
    launch; optional per-row weights [n * h] (or [n, h])."""
    _cuda(x, covariances, weights)
    groups = covariances.shape[0]
    if covariances.dtype != torch.float32 or covariances.shape[1:] != (256, 256) or not covariances.is_contiguous():
        raise ValueError("covariances must be contiguous fp32 [groups, 256, 256]")
    n, h, d = x.shape
    if d != 256 or h % groups:
        raise ValueError("head_dim must be 256 and the heads must split evenly into the groups")
    if x.dtype != torch.bfloat16 or x.stride(2) != 1 or x.stride(0) % 8 or x.stride(1) % 8 or x.data_ptr() % 16:
        x = x.to(torch.bfloat16).contiguous()
    w = None
    if weights is not None:
        w = weights.float().contiguous().view(-1)
        if w.numel() != n * h:
            raise ValueError("weights must have one entry per (token, head) row")
    _lib.call("oscar_accumulate_gram_grouped", x.data_ptr(), n, h, x.stride(0), x.stride(1), groups,
              None if w is None else w.data_ptr(), covariances.data_ptr(), _stream(x))


def prepare_sst_covariances(q_covariances: torch.Tensor) -> torch.Tensor:
    """The three bf16 parts (hi, mid, lo; their sum is each fp32 entry exactly) of every
    query covariance [h, 256, 256], as bf16 [h, 3, 256, 256]: computed once per
    calibration pass and reused by every :func:`sst_weights_per_head` call of it."""
    _cuda(q_covariances)
    c = q_covariances.float().contiguous()
    if c.dim() != 3 or c.shape[1:] != (256, 256):
        raise ValueError("query covariances must be [h, 256, 256]")
    parts = torch.empty((c.shape[0], 3, 256, 256), dtype=torch.bfloat16, device=c.device)
    _lib.call("oscar_split_bf16x3", c.data_ptr(), c.shape[0], parts.data_ptr(), _stream(c))
    return parts


def sst_weights_per_head(key: torch.Tensor, q_covariances: torch.Tensor, totals: torch.Tensor,
                         prepared: torch.Tensor | None = None):
    """Per-head ``w = max(k C_h k^T, 0)`` (key [n, h, 256], q_covariances [h, 256, 256])
    and ``totals[h] += sum w``; returns w as fp32 [n * h] (token-major).  With
    ``prepared`` (:func:`prepare_sst_covariances` of the same covariances) the weights
    come from the tcgen05 kernel, else (or when the key layout does not fit a tensor
    map) from the mma.sync kernel, which splits the covariances itself."""
    _cuda(key, q_covariances, totals)
    n, h, d = key.shape
    if q_covariances.shape != (h, 256, 256) or totals.numel() != h or not totals.is_contiguous():
        raise ValueError("one covariance and one total per head")
    if key.dtype != torch.bfloat16 or key.stride(2) != 1 or key.stride(0) % 8 or key.stride(1) % 8 or key.data_ptr() % 16:
        key = key.to(torch.bfloat16).contiguous()
    weights = torch.empty(n * h, device=key.device, dtype=torch.float32)
    if prepared is not None:
        if prepared.shape != (h, 3, 256, 256) or prepared.dtype != torch.bfloat16 or not prepared.is_contiguous():
            raise ValueError("prepared covariances must come from prepare_sst_covariances")
        rc = _lib.lib().oscar_sst_weights_split(key.data_ptr(), n, h, key.stride(0), key.stride(1),
                                                prepared.data_ptr(), weights.data_ptr(), totals.data_ptr(),
                                                status_word(key.device).data_ptr(), _stream(key))
        if rc != _lib.UNSUPPORTED:
            _lib.check(rc, "oscar_sst_weights_split")
            return weights
    c = q_covariances.float().contiguous()
    _lib.call("oscar_sst_weights_per_head", key.data_ptr(), n, h, key.stride(0), key.stride(1), c.data_ptr(),
              weights.data_ptr(), totals.data_ptr(), _stream(key))
    return weights


def sst_weights(key: torch.Tensor, q_covariance: torch.Tensor, total_weight: torch.Tensor):
    """``w_t = max(k_t C k_t^T, 0)`` per row and ``total_weight += sum w``
    (reference calibration_kernels.py:109-126; any number of KV heads)."""
    _cuda(key, q_covariance, total_weight)
    n, h, d = key.shape
    if key.dtype != torch.bfloat16 or key.stride(2) != 1 or key.stride(0) % 8 or key.stride(1) % 8 or key.data_ptr() % 16:
        key = key.to(torch.bfloat16).contiguous()
    c = q_covariance.float().contiguous()
    weights = torch.empty(n * h, device=key.device, dtype=torch.float32)
    _lib.call("oscar_sst_weights", key.data_ptr(), n, h, key.stride(0), key.stride(1), c.data_ptr(),
              weights.data_ptr(), total_weight.data_ptr(), _stream(key))
    return weights


def normalize(x: torch.Tensor, denominator):
    """``x / max(denominator, 1e-30)`` with a host or device denominator (reference :145-156)."""
    _cuda(x)
    out = torch.empty_like(x)
    xc = x.contiguous()
    dev = isinstance(denominator, torch.Tensor)
    _lib.call("oscar_normalize", xc.data_ptr(), xc.numel(), denominator.data_ptr() if dev else None,
              0.0 if dev else float(denominator), out.data_ptr(), _stream(xc))
    return out


def calibrated_rotations(covariances: torch.Tensor, max_sweeps: int = 12, tolerance: float = 1e-6,
                         refine: float = 1e-7):
    """Batched cyclic Jacobi + ``U H P_br`` (reference :287-327).

    Returns ``(rotations [B,256,256], eigenvalues [B,256], info)``; raises like the
    reference when the result is non-finite or did not converge.  Convergence is the
    reference's ``max|off| / max|diag| < tolerance``; the sweeps continue (within
    ``max_sweeps``) down to ``refine``, because with a wide spectrum an off-diagonal
    left at ``1e-6 * max|diag|`` still moves the small, closely spaced eigenvalues by
    about ``off^2 / gap`` (1e-4 relative on covariances with outlier channels; ~1e-6
    at 1e-7).  The reference's skip rule (no rotation once |a_pq| < 1e-8 (|a_pp| +
    |a_qq|)) keeps the residual near 1e-8, so tighter targets only burn sweeps.
    """
    _cuda(covariances)
    if covariances.dtype != torch.float32:
        raise ValueError("calibration eigensolver requires fp32 covariances")
    batch, dim, last = covariances.shape
    if dim != 256 or last != 256:
        raise ValueError("calibration eigensolver is scoped to D256")
    cov = covariances.contiguous()
    rot = torch.empty_like(cov)
    evals = torch.empty((batch, dim), dtype=torch.float32, device=cov.device)
    info = torch.zeros((batch, 4), dtype=torch.float32, device=cov.device)
    stop = min(float(refine), float(tolerance))
    _lib.call("oscar_jacobi_rotations", cov.data_ptr(), batch, int(max_sweeps), stop, rot.data_ptr(),
              evals.data_ptr(), info.data_ptr(), _stream(cov))
    host = info.cpu()
    status = host[:, 2]
    residual = float(host[:, 1].max())
    result = {"sweeps": int(host[:, 0].max()), "relative_off_diagonal": residual}
    if bool((status == 3).any()):
        raise RuntimeError("calibration eigensolver: a device wait timed out; rotations not published")
    if bool((status == 2).any()):
        raise RuntimeError("non-finite calibration covariance; rotations not published")
    if not residual < tolerance:
        raise RuntimeError(f"calibration eigensolver did not converge: {residual}; rotations not published")
    return rot, evals, result
