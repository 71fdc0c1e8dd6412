"""Loading helpers for the committed golden fixtures (made by ``make_golden.py``)."""

from __future__ import annotations

import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load(name: str):
    return torch.load(HERE / name, weights_only=False)


def unzpack(d) -> torch.Tensor:
    raw = np.frombuffer(zlib.decompress(d["z"]), dtype=np.uint8).copy()
    return torch.from_numpy(raw).view(getattr(torch, d["dtype"])).reshape(d["shape"])
