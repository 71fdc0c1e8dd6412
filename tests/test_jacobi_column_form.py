"""The eigensolver's column form, restated in numpy, against the oracle's two-sided Jacobi.

`jacobi_kernel` (csrc/calibration.cu) never forms A = V^T C V: it keeps W = C V and V,
takes a_pp, a_qq, a_pq of a pair as the column dot products v_p.w_p, v_q.w_q, v_p.w_q
(each CTA's sum over its 32 rows, the eight CTA sums added as ((c0 + c4) + (c1 + c5)) +
((c2 + c6) + (c3 + c7))), rotates the columns of W and V, and moves every column one seat
down the ring between rounds (group m holds pairs 2m, 2m + 1; the moves of
`test_device_index_math.py`).  This restatement follows that data flow in fp64 and must
reach what the reference's algorithm (`oracle.calibration_oracle.jacobi`, two-sided on A
with the same pair schedule, formula and skip rule) reaches after the same number of
sweeps: the same eigenvalues and eigenvectors.  (Mid-run states are not compared: where
two diagonal entries are nearly equal, the sign of delta picks between two equally valid
45-degree rotations, so two correct fp64 implementations may take different paths.)
"""

import numpy as np
import torch

from oracle.calibration_oracle import jacobi, round_robin_pairs

D, CTAS, GROUPS = 256, 8, 64


def column_form(cov: np.ndarray, sweeps: int):
    a = (cov + cov.T) / 2
    # seats of round 0: pair j = 2m + k holds columns p[j], q[j]
    p0, q0 = (t.numpy() for t in round_robin_pairs(D, 0))
    wp, wq = a[:, p0].T.copy(), a[:, q0].T.copy()  # [pair, row]
    eye = np.eye(D)
    vp, vq = eye[:, p0].T.copy(), eye[:, q0].T.copy()
    for _ in range(sweeps):
        for _r in range(D - 1):
            # per-CTA sums over its 32 rows, then the fixed cross-CTA order
            def cluster_sum(x):
                c = x.reshape(D // 2, CTAS, 32).sum(-1)
                return ((c[:, 0] + c[:, 4]) + (c[:, 1] + c[:, 5])) + ((c[:, 2] + c[:, 6]) + (c[:, 3] + c[:, 7]))

            app, aqq, apq = cluster_sum(vp * wp), cluster_sum(vq * wq), cluster_sum(vp * wq)
            delta = (aqq - app) * 0.5
            sgn = np.where(delta >= 0, 1.0, -1.0)
            h = np.sqrt(delta * delta + apq * apq)
            tang = sgn * apq / np.maximum(np.abs(delta) + h, 1e-300)
            tang = np.where(np.abs(apq) > 1e-8 * (np.abs(app) + np.abs(aqq)) + 1e-20, tang, 0.0)
            cs = 1.0 / np.sqrt(tang * tang + 1.0)
            sn = tang * cs
            cs, sn = cs[:, None], sn[:, None]
            wp, wq = wp * cs - wq * sn, wp * sn + wq * cs
            vp, vq = vp * cs - vq * sn, vp * sn + vq * cs
            # the ring move, per group m of pairs (2m, 2m + 1)
            new = []
            for mats in ((wp, wq), (vp, vq)):
                p, q = mats[0].reshape(GROUPS, 2, D), mats[1].reshape(GROUPS, 2, D)
                np_, nq = p.copy(), q.copy()
                np_[1:, 0] = p[1:, 1]                   # p0 <- p1 (pair 0 keeps column 255)
                nq[1:, 0] = q[:-1, 1]                   # q0 <- group m - 1's q1
                nq[0, 0] = p[0, 1]                      # pair 0: its own p1
                np_[:-1, 1] = p[1:, 0]                  # p1 <- group m + 1's p0
                np_[-1, 1] = q[-1, 1]                   # pair 127: its own q1
                nq[:, 1] = q[:, 0]                      # q1 <- q0
                new += [np_.reshape(D // 2, D), nq.reshape(D // 2, D)]
            wp, wq, vp, vq = new
    # back to columns (round-0 seats), Rayleigh quotients
    w, v = np.empty((D, D)), np.empty((D, D))
    w[:, p0], w[:, q0], v[:, p0], v[:, q0] = wp.T, wq.T, vp.T, vq.T
    ev = (v * w).sum(0)
    order = np.argsort(ev, kind="stable")
    return v[:, order], ev[order]


def test_column_form_converges_like_the_reference_algorithm():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((384, D))
    x[:, :8] *= 5
    cov = x.T @ x / 384
    sweeps = 8
    u_ref, ev_ref, done = jacobi(torch.from_numpy(cov), sweeps=sweeps)
    assert done == sweeps
    u, ev = column_form(cov, sweeps)
    u_ref, ev_ref = u_ref.numpy(), ev_ref.numpy()
    exact = np.linalg.eigvalsh(cov)
    scale = float(np.abs(exact).max())
    assert float(np.abs(ev_ref - exact).max()) < 1e-10 * scale
    assert float(np.abs(ev - exact).max()) < 1e-10 * scale
    # the same eigenvectors (up to sign) and an orthogonal V
    assert float(np.abs(np.abs((u * u_ref).sum(0)) - 1).max()) < 1e-8
    assert float(np.abs(u.T @ u - np.eye(D)).max()) < 1e-12
