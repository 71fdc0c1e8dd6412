"""How `calibrated_rotations` reads the eigensolver's per-matrix info words.

`oscar_jacobi_rotations` writes {sweeps, relative_off_diagonal, status, 0} per matrix
(status 0 ok, 1 not converged, 2 non-finite, 3 a device wait for the cluster's partial
sums timed out).  Here the C ABI call is replaced by a host fake that writes chosen info
words into the buffer it is given, so the host's decisions are checked without a GPU.
"""

import ctypes

import pytest
import torch

from oscar_new_b200 import _lib
from oscar_new_b200 import calibration_kernels as ck


def fake_solver(monkeypatch, words):
    monkeypatch.setattr(ck, "_cuda", lambda *ts: None)
    monkeypatch.setattr(ck, "_stream", lambda t: None)

    def call(name, cov, batch, max_sweeps, stop, rot, evals, info, stream):
        assert name == "oscar_jacobi_rotations" and batch == len(words)
        flat = [float(x) for w in words for x in w]
        ctypes.memmove(info, (ctypes.c_float * len(flat))(*flat), 4 * len(flat))

    monkeypatch.setattr(_lib, "call", call)


@pytest.mark.parametrize("words,error", [
    ([(9, 5e-8, 0, 0), (9, 8e-8, 0, 0)], None),
    ([(9, 5e-8, 0, 0), (12, 3e-6, 1, 0)], "did not converge"),
    ([(2, float("inf"), 2, 0), (9, 5e-8, 0, 0)], "non-finite"),
    ([(3, float("inf"), 3, 0), (3, float("inf"), 3, 0)], "device wait timed out"),
])
def test_info_words_decide_publication(monkeypatch, words, error):
    fake_solver(monkeypatch, words)
    cov = torch.zeros(len(words), 256, 256)
    if error is None:
        _, _, info = ck.calibrated_rotations(cov)
        assert info == {"sweeps": 9, "relative_off_diagonal": pytest.approx(8e-8)}
    else:
        with pytest.raises(RuntimeError, match=error):
            ck.calibrated_rotations(cov)
