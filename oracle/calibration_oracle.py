"""CPU oracle for OSCAR calibration (covariances, Jacobi EVD, U*H*P_br).
TEST INFRASTRUCTURE ONLY -- imported by ``tests/`` and ``bench.py``'s CPU leg, never by
the product package.

Restates, in fp64 torch-CPU code:

* ``gram`` / ``weighted_gram`` — ``oscar_ascend/calibration_kernels.py:14-56``
  (``C += X^T X`` over all rows and heads; ``C += sum_t w_t x_t^T x_t``);
* ``sst_weights`` — ``calibration_kernels.py:73-126`` (``w_t = max(k_t C_q k_t^T, 0)``);
* ``jacobi`` — the parallel cyclic (round-robin) Jacobi of
  ``calibration_kernels.py:170-225`` (pairs ``p = D-1 | (r+j) mod (D-1)``,
  ``q = r | (r-j+D-1) mod (D-1)``, skip rule ``|a_pq| > 1e-8(|a_pp|+|a_qq|) + 1e-20``),
  the same recurrences as the reference's own ``tests/test_calibration_math.py:6-25``;
* ``hadamard`` / ``pbr`` / ``compose`` — ``calibration_kernels.py:270-284`` and
  ``tests/test_calibration_math.py:28-43``: ``R = U_sorted * H / sqrt(D)`` with column
  ``i`` moved to ``bitrev(D-1-i)``.
"""

from __future__ import annotations

import torch


def gram(x: torch.Tensor) -> torch.Tensor:
    """sum over rows and heads of x^T x, fp64; x [N, H, D]."""
    flat = x.double().reshape(-1, x.shape[-1])
    return flat.T @ flat


def weighted_gram(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    flat = x.double().reshape(-1, x.shape[-1])
    return flat.T @ (flat * w.double().reshape(-1)[:, None])


def sst_weights(k: torch.Tensor, q_cov: torch.Tensor) -> torch.Tensor:
    """w_t = max(k_t C k_t^T, 0) per (token, head) row of k [N, H, D]."""
    flat = k.double().reshape(-1, k.shape[-1])
    return ((flat @ q_cov.double()) * flat).sum(-1).clamp_min(0)


def round_robin_pairs(dim: int, round_index: int):
    j = torch.arange(dim // 2)
    p = torch.where(j == 0, torch.full_like(j, dim - 1), (round_index + j) % (dim - 1))
    q = torch.where(j == 0, torch.full_like(j, round_index), (round_index - j + dim - 1) % (dim - 1))
    return p, q


def jacobi(cov: torch.Tensor, sweeps: int = 10, tol: float | None = None):
    """Parallel cyclic Jacobi in fp64.  Returns (U sorted ascending, eigenvalues, sweeps run)."""
    a = cov.double().clone()
    a = (a + a.T) / 2
    dim = a.shape[0]
    u = torch.eye(dim, dtype=torch.float64)
    done = 0
    for sweep in range(sweeps):
        for r in range(dim - 1):
            p, q = round_robin_pairs(dim, r)
            app, aqq, apq = a[p, p], a[q, q], a[p, q]
            delta = (aqq - app) / 2
            sign = torch.where(delta >= 0, 1.0, -1.0).double()
            t = sign * apq / (delta.abs() + (delta * delta + apq * apq).sqrt()).clamp_min(1e-30)
            t = torch.where(apq.abs() > 1e-8 * (app.abs() + aqq.abs()) + 1e-20, t, torch.zeros_like(t))
            c = (1 + t * t).rsqrt()
            s = t * c
            b = a.clone()
            b[:, p], b[:, q] = a[:, p] * c - a[:, q] * s, a[:, p] * s + a[:, q] * c
            nu = u.clone()
            nu[:, p], nu[:, q] = u[:, p] * c - u[:, q] * s, u[:, p] * s + u[:, q] * c
            a = b.clone()
            a[p], a[q] = c[:, None] * b[p] - s[:, None] * b[q], s[:, None] * b[p] + c[:, None] * b[q]
            u = nu
        done = sweep + 1
        if tol is not None:
            off = (a - torch.diag(a.diag())).abs().max()
            if off / a.diag().abs().max().clamp_min(1e-30) < tol:
                break
    order = torch.argsort(a.diag(), stable=True)
    return u[:, order], a.diag()[order], done


def hadamard(dim: int) -> torch.Tensor:
    """Normalised Sylvester Hadamard matrix (fp64)."""
    h = torch.ones((1, 1), dtype=torch.float64)
    while h.shape[0] < dim:
        h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0) / 2**0.5
    return h


def bit_reverse(i: int, bits: int) -> int:
    return int(f"{i:0{bits}b}"[::-1], 2)


def pbr(dim: int) -> torch.Tensor:
    """Permutation matrix: column bitrev(i) takes sorted index D-1-i (descending order)."""
    bits = dim.bit_length() - 1
    perm = torch.empty(dim, dtype=torch.long)
    for i in range(dim):
        perm[bit_reverse(i, bits)] = dim - 1 - i
    return torch.eye(dim, dtype=torch.float64)[:, perm]


def compose(u_sorted: torch.Tensor) -> torch.Tensor:
    """R = U_sorted @ H @ P_br (fp64)."""
    dim = u_sorted.shape[-1]
    return u_sorted.double() @ hadamard(dim) @ pbr(dim)
